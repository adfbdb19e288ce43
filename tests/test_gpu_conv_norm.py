"""GPU parity of the conv and gated-norm kernels; rounding matches the eager path bit for bit."""

import pytest
import torch

import jeeves_b200 as gdn
import oracle
from tests.helpers import assert_bf16_matches_cpu, cuda, same_bits

pytestmark = pytest.mark.gpu


def test_golden_conv1d(golden):
    c = golden("conv1d")
    assert same_bits(gdn.causal_conv1d(c["x"].cuda(), c["w"].cuda()), c["y"])


@pytest.mark.parametrize("B,T,C", [(1, 4096, 8192), (2, 300, 8192), (3, 7, 96)])
def test_conv1d_matches_oracle(B, T, C):
    gen = torch.Generator().manual_seed(B + T)
    x = (torch.randn(B, T, C, generator=gen) * 2).to(torch.bfloat16)
    w = (torch.randn(C, 4, generator=gen) * 0.5).to(torch.bfloat16)
    assert_bf16_matches_cpu(gdn.causal_conv1d(x.cuda(), w.cuda()), oracle.causal_conv1d(x, w))


def test_conv1d_special_values_in_either_lane_of_a_channel_pair():
    # signed zeros, |x| > 80 on both sides and NaN, placed at even and odd channels so that they
    # reach both lanes of the packed pairs and the per-element path they fall back to
    gen = torch.Generator().manual_seed(11)
    T, C = 64, 256
    x = (torch.randn(1, T, C, generator=gen) * 2).to(torch.bfloat16)
    w = (torch.randn(C, 4, generator=gen) * 0.5).to(torch.bfloat16)
    w[3::5] = 0
    w[8::11, 3] = 100.0
    x.view(-1)[1::97] = -0.0
    x.view(-1)[2::89] = 0.0
    x.view(-1)[3::83] = 300.0
    x.view(-1)[4::79] = -300.0
    x.view(-1)[5::601] = float("nan")
    y = gdn.causal_conv1d(x.cuda(), w.cuda()).cpu()
    ref = oracle.causal_conv1d(x, w)
    assert torch.equal(y.isnan(), ref.isnan())
    assert_bf16_matches_cpu(torch.nan_to_num(y), torch.nan_to_num(ref))
    assert torch.equal(torch.signbit(y[y == 0]), torch.signbit(ref[y == 0]))


def test_conv1d_varlen_restarts_each_sequence():
    gen = torch.Generator().manual_seed(3)
    lens = [5, 40, 1, 70]
    x = (torch.randn(1, sum(lens), 256, generator=gen) * 2).to(torch.bfloat16)
    w = (torch.randn(256, 4, generator=gen) * 0.5).to(torch.bfloat16)
    cu = torch.tensor([0, 5, 45, 46, 116], dtype=torch.int32)
    y = gdn.causal_conv1d(x.cuda(), w.cuda(), cu_seqlens=cu.cuda()).cpu()
    for i in range(4):
        s, e = int(cu[i]), int(cu[i + 1])
        assert_bf16_matches_cpu(y[:, s:e], oracle.causal_conv1d(x[:, s:e], w))


def test_golden_conv1d_step(golden):
    c = golden("conv1d_step")
    st = c["state"].cuda()
    y = gdn.causal_conv1d_step(c["x"].cuda(), st, c["w"].cuda())
    assert same_bits(y, c["y"]) and same_bits(st, c["state_after"])


def test_conv1d_step_matches_oracle_at_model_width():
    gen = torch.Generator().manual_seed(4)
    x = (torch.randn(16, 8192, generator=gen) * 2).to(torch.bfloat16)
    st = torch.randn(16, 8192, 4, generator=gen).to(torch.bfloat16)
    w = (torch.randn(8192, 4, generator=gen) * 0.5).to(torch.bfloat16)
    st_ref, st_gpu = st.clone(), st.cuda()
    y_ref = oracle.causal_conv1d_step(x, st_ref, w)
    y = gdn.causal_conv1d_step(x.cuda(), st_gpu, w.cuda())
    assert_bf16_matches_cpu(y, y_ref)
    assert same_bits(st_gpu, st_ref)


def test_golden_conv_step(golden):
    c = golden("conv_step")
    out = gdn.conv_step(c["state"].cuda(), c["qkv"].cuda(), c["w"].cuda(), c["key_dim"], c["value_dim"], c["head_dim"],
                        c["head_dim"])
    for a, b in zip(out, (c["ext"], c["q"], c["k"], c["v"])):
        assert same_bits(a, b)


@pytest.mark.parametrize("B,T", [(1, 4), (4, 5), (2, 8), (2, 9)])  # taps + T up to 12 take the 16-byte path
def test_conv_step_matches_oracle_and_writes_ext_out_only(B, T):
    gen = torch.Generator().manual_seed(10 + B * T)
    key_dim, value_dim, hd, taps = 2048, 4096, 128, 4
    C = 2 * key_dim + value_dim
    merged = (torch.randn(B, T, C + 64, generator=gen) * 2).to(torch.bfloat16)
    st = torch.randn(B, C, taps, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C, 1, taps, generator=gen) * 0.5).to(torch.bfloat16)
    ref = oracle.conv_step(st, merged[..., :C], w, key_dim, value_dim, hd, hd)
    mc = merged.cuda()
    out = gdn.conv_step(st.cuda(), mc[..., :C], w.cuda(), key_dim, value_dim, hd, hd)
    assert same_bits(out[0], ref[0])
    for a, b in zip(out[1:], ref[1:]):
        assert_bf16_matches_cpu(a, b)
    stacked = torch.zeros(3, B, C, taps + T, dtype=torch.bfloat16, device="cuda")
    stacked[1] = float("nan")
    out2 = gdn.conv_step(st.cuda(), mc[..., :C], w.cuda(), key_dim, value_dim, hd, hd, ext_out=stacked[1])
    assert out2[0].data_ptr() == stacked[1].data_ptr()
    assert all(same_bits(a, b) for a, b in zip(out2, out))
    assert not stacked[0].any() and not stacked[2].any()


def test_golden_gated_norm(golden):
    c = golden("gated_norm")
    y = gdn.gated_rms_norm(c["x"].cuda(), c["z"].cuda(), c["w"].cuda()).cpu()
    # silu(z) is evaluated in fp32 on both sides; the CPU's vectorised exp can move a
    # bf16 rounding by one ulp, so allow a rare one-ulp difference.
    assert (y != c["y"]).float().mean().item() < 0.01
    assert ((y.float() - c["y"].float()).abs() <= c["y"].float().abs() * 2 ** -6).all()


@pytest.mark.parametrize("rows,scale", [(4096 * 32, 2.0), (65536 + 37, 2.0), (64, 1e-3), (1536, 2.0)])
def test_gated_norm_matches_oracle(rows, scale):
    gen = torch.Generator().manual_seed(rows)
    x = (torch.randn(rows, 128, generator=gen) * scale).to(torch.bfloat16)
    z = (torch.randn(rows, 128, generator=gen) * 3).to(torch.bfloat16)
    w = (torch.rand(128, generator=gen) + 0.5).to(torch.bfloat16)
    y = gdn.gated_rms_norm(*cuda(x, z, w)).cpu()
    ref = oracle.gated_rms_norm(x, z, w)
    assert (y != ref).float().mean().item() < 1e-3
    # a one-ulp flip of the normalised value can move the product with the weight by two
    # ulps (bf16 rounding after each step), so the bound is two bf16 ulps
    assert ((y.float() - ref.float()).abs() <= ref.float().abs() * 2 ** -6 + 1e-30).all()


def test_gated_norm_module_dropin():
    norm = gdn.GatedRMSNorm(128).cuda().to(torch.bfloat16)
    x = torch.randn(10, 128, device="cuda", dtype=torch.bfloat16)
    z = torch.randn(10, 128, device="cuda", dtype=torch.bfloat16)
    ref = oracle.gated_rms_norm(x.cpu(), z.cpu(), norm.weight.detach().cpu())
    assert (norm(x, z).cpu() != ref).float().mean().item() < 0.01
