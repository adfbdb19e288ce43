"""GPU parity of the fused decode and prefill layers against the composition of the oracle's ops,
and of the norm-fused chunked prefill against the separate chunk and norm calls."""

import pytest
import torch

import jeeves_b200 as gdn
import oracle
from tests.helpers import gdn_inputs, maxabs, rel, same_bits

pytestmark = pytest.mark.gpu


def reference_layer(qkv, conv_state, w, g, beta, state, z, nw, H, HV):
    B, C = qkv.shape
    y = oracle.causal_conv1d_step(qkv, conv_state, w)  # updates conv_state
    kd = H * 128
    q = y[:, :kd].reshape(B, 1, H, 128)
    k = y[:, kd:2 * kd].reshape(B, 1, H, 128)
    v = y[:, 2 * kd:].reshape(B, 1, HV, 128)
    o, S = oracle.recurrent_gated_delta_rule(q, k, v, g.reshape(B, 1, HV), beta.reshape(B, 1, HV),
                                             initial_state=state, output_final_state=True)
    out = oracle.gated_rms_norm(o.reshape(-1, 128), z.reshape(-1, 128), nw).reshape(B, HV, 128)
    return out, S


@pytest.mark.parametrize("B,H,HV,taps", [(4, 16, 32, 4), (3, 2, 4, 3)])
def test_decode_layer_matches_composition(B, H, HV, taps):
    gen = torch.Generator().manual_seed(B * 10 + taps)
    C = 2 * H * 128 + HV * 128
    qkv = (torch.randn(B, C, generator=gen) * 2).to(torch.bfloat16)
    cs = torch.randn(B, C, taps, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C, 4, generator=gen) * 0.5).to(torch.bfloat16)
    g = -torch.exp(torch.randn(B, HV, generator=gen) * 0.5 - 3.0)
    beta = torch.sigmoid(torch.randn(B, HV, generator=gen)).to(torch.bfloat16)
    state = torch.randn(B, HV, 128, 128, generator=gen) * 0.02
    z = torch.randn(B, HV, 128, generator=gen).to(torch.bfloat16)
    nw = (torch.rand(128, generator=gen) + 0.5).to(torch.bfloat16)
    cs_ref = cs.clone()
    if taps == 4:
        out_ref, S_ref = reference_layer(qkv, cs_ref, w, g, beta, state, z, nw, H, HV)
    else:  # the eager step keeps K taps; with 3 live taps the state holds the last 3 inputs
        full = torch.cat([torch.zeros(B, C, 1, dtype=cs.dtype), cs], dim=-1)
        out_ref, S_ref = reference_layer(qkv, full, w, g, beta, state, z, nw, H, HV)
        cs_ref = full[..., 1:]
    cs_gpu, st_gpu = cs.cuda(), state.cuda()
    out = gdn.decode_layer_step(qkv.cuda(), cs_gpu, w.cuda(), g.cuda(), beta.cuda(), st_gpu, z.cuda(), nw.cuda(), H)
    assert same_bits(cs_gpu, cs_ref)
    assert rel(st_gpu, S_ref) < 1e-5
    assert maxabs(out, out_ref) < 2e-2
    assert (out.cpu() != out_ref).float().mean().item() < 0.02


def reference_prefill_layer(qkv, w, g, beta, z, nw, H, HV, h0=None):
    B, T, C = qkv.shape
    y = oracle.causal_conv1d(qkv, w)
    kd = H * 128
    q = y[..., :kd].reshape(B, T, H, 128)
    k = y[..., kd:2 * kd].reshape(B, T, H, 128)
    v = y[..., 2 * kd:].reshape(B, T, HV, 128)
    o, S = oracle.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    out = oracle.gated_rms_norm(o.reshape(-1, 128), z.reshape(-1, 128), nw).reshape(B, T, HV, 128)
    return out, S


def layer_inputs(seed, B, T, H, HV):
    gen = torch.Generator().manual_seed(seed)
    C = 2 * H * 128 + HV * 128
    qkv = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C, 4, generator=gen) * 0.5).to(torch.bfloat16)
    g = -torch.exp(torch.randn(B, T, HV, generator=gen) * 0.5 - 3.0)
    beta = torch.sigmoid(torch.randn(B, T, HV, generator=gen)).to(torch.bfloat16)
    z = torch.randn(B, T, HV, 128, generator=gen).to(torch.bfloat16)
    nw = (torch.rand(128, generator=gen) + 0.5).to(torch.bfloat16)
    h0 = torch.randn(B, HV, 128, 128, generator=gen) * 0.02
    return qkv, w, g, beta, z, nw, h0


@pytest.mark.parametrize("B,T,H,HV", [(1, 700, 16, 32), (2, 130, 2, 4), (1, 4096, 16, 32)])
def test_prefill_layer_matches_oracle_composition(B, T, H, HV):
    """conv + SiLU, chunked gated delta rule and gated norm (the prefill branch of the layer)
    against the oracle's ops, up to config 1's full shape (B=1, T=4096, 16 / 32 heads). The norm
    divides each row by its rms (about 0.01 with these inputs), which magnifies the chunk output's
    absolute error about a hundredfold, so the layer is checked step by step: the conv bit for bit,
    the chunk output within the bf16 output bound (max-abs 2e-2) and the state within 1e-3
    relative, the norm of that output within 2^-6 relative of the oracle's norm of the same values
    (under 1% of the elements differing at all), and the whole output within 1e-2 relative
    (Frobenius)."""
    qkv, w, g, beta, z, nw, h0 = layer_inputs(B * 100 + T, B, T, H, HV)
    out_ref, S_ref = reference_prefill_layer(qkv, w, g, beta, z, nw, H, HV, h0)
    qkv_d, w_d, g_d, b_d, z_d, nw_d, h0_d = (t.cuda() for t in (qkv, w, g, beta, z, nw, h0))
    out, S = gdn.prefill_layer(qkv_d, w_d, g_d, b_d, z_d, nw_d, H, initial_state=h0_d)
    assert out.shape == (B, T, HV, 128)
    assert torch.isfinite(out.float()).all()
    assert rel(S, S_ref) < 1e-3, rel(S, S_ref)
    # the steps: conv, chunk output, norm of that output
    y = gdn.causal_conv1d(qkv_d, w_d)
    assert same_bits(y, oracle.causal_conv1d(qkv, w))
    kd = H * 128
    o, S2 = gdn.gated_delta_rule_chunk(y[..., :kd].view(B, T, H, 128), y[..., kd:2 * kd].view(B, T, H, 128),
                                       y[..., 2 * kd:].view(B, T, HV, 128), g_d, b_d, initial_state=h0_d,
                                       output_final_state=True)
    assert same_bits(S2, S)
    o_ref, _ = oracle.chunk_gated_delta_rule(*(t.cpu() for t in (y[..., :kd].reshape(B, T, H, 128),
                                                                 y[..., kd:2 * kd].reshape(B, T, H, 128),
                                                                 y[..., 2 * kd:].reshape(B, T, HV, 128))),
                                             g, beta, initial_state=h0)
    assert maxabs(o, o_ref) < 2e-2, maxabs(o, o_ref)
    normed = oracle.gated_rms_norm(o.cpu().reshape(-1, 128), z.reshape(-1, 128), nw).reshape(B, T, HV, 128)
    # the norm kernel's bound, as in test_gpu_conv_norm: the reference rounds to bf16 three times
    # (the normalised value, its product with the weight, the product with silu(z)); the kernel's
    # rsqrt can move the first rounding by one ulp and the CPU's exp in silu(z) the last, so an
    # element can land up to 2^-6 relative away (two to four bf16 ulps). A CPU simulation of those
    # two flips over the 16.8 M elements of config 1 gives 4 elements three ulps away, at most 0.8
    # of this bound.
    d = (out.cpu().float() - normed.float()).abs()
    lim = normed.float().abs() * 2 ** -6 + 1e-30
    assert (d <= lim).all(), float((d / lim).max())
    assert (out.cpu() != normed).float().mean().item() < 0.01
    assert rel(out, out_ref) < 1e-2, rel(out, out_ref)


def _chunk_then_norm(q, k, v, g, beta, z, nw, h0, cu=None):
    o, S = gdn.gated_delta_rule_chunk(q, k, v, g, beta, initial_state=h0, output_final_state=True, cu_seqlens=cu)
    y = gdn.gated_rms_norm(o.reshape(-1, 128), z.reshape(-1, 128), nw).reshape(o.shape)
    return y, S


@pytest.mark.parametrize("B,T,H,HV,state", [
    (1, 1000, 16, 32, True),   # 64 scan CTAs: the cooperative launch, then the norm
    (2, 300, 16, 32, False),   # 128 scan CTAs: still one chunk launch, two sequences in chunk-major order
    (1, 65, 2, 4, True),       # 8 scan CTAs, a ragged last chunk
    (3, 130, 16, 32, True),    # 192 scan CTAs: factor kernel, scan kernel, then the norm
])
def test_chunk_gated_norm_equals_chunk_then_norm_bitwise(B, T, H, HV, state):
    q, k, v, g, beta, h0 = gdn_inputs(B * 7 + T, B, T, H, HV, state=state, normalise=False)
    gen = torch.Generator().manual_seed(T)
    z = torch.randn(B, T, HV, 128, generator=gen).to(torch.bfloat16).cuda()
    nw = (torch.rand(128, generator=gen) + 0.5).to(torch.bfloat16).cuda()
    q, k, v, g, beta = (t.cuda() for t in (q, k, v, g, beta))
    h0 = None if h0 is None else h0.cuda()
    y_ref, S_ref = _chunk_then_norm(q, k, v, g, beta, z, nw, h0)
    y, S = gdn.gated_delta_rule_chunk_gated_norm(q, k, v, g, beta, z, nw, initial_state=h0, output_final_state=True)
    assert same_bits(y, y_ref) and same_bits(S, S_ref)
    out = torch.full_like(y, float("nan"))  # a caller-given output buffer
    y2, _ = gdn.gated_delta_rule_chunk_gated_norm(q, k, v, g, beta, z, nw, initial_state=h0, out=out)
    assert y2.data_ptr() == out.data_ptr() and same_bits(out, y_ref)


@pytest.mark.parametrize("lens", [[300, 77], [1, 64, 0, 129, 400, 33, 2, 90]])
def test_packed_chunk_gated_norm_equals_chunk_then_norm_bitwise(lens):
    """Two packed sequences (128 scan CTAs: one chunk launch, chunks of the shorter sequence
    skipped in chunk-major order) and eight (512 scan CTAs: factor, order and scan kernels)."""
    H, HV, T = 16, 32, sum(lens)
    q, k, v, g, beta, _ = gdn_inputs(len(lens), 1, T, H, HV, normalise=False)
    gen = torch.Generator().manual_seed(len(lens) + 1)
    h0 = (torch.randn(len(lens), HV, 128, 128, generator=gen) * 0.02).cuda()
    z = torch.randn(1, T, HV, 128, generator=gen).to(torch.bfloat16).cuda()
    nw = (torch.rand(128, generator=gen) + 0.5).to(torch.bfloat16).cuda()
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32).cuda()
    q, k, v, g, beta = (t.cuda() for t in (q, k, v, g, beta))
    y_ref, S_ref = _chunk_then_norm(q, k, v, g, beta, z, nw, h0, cu)
    y, S = gdn.gated_delta_rule_chunk_gated_norm(q, k, v, g, beta, z, nw, initial_state=h0, output_final_state=True,
                                                 cu_seqlens=cu)
    assert same_bits(y, y_ref) and same_bits(S, S_ref)


def test_prefill_layer_leaves_no_device_error():
    from jeeves_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.load().gdn_device_error(None, 0) == 0


@pytest.mark.parametrize("B,H,HV,taps", [(8, 16, 32, 3), (64, 16, 32, 4), (256, 16, 32, 3), (128, 4, 4, 4),
                                         (3, 2, 4, 3)])
def test_decode_layer_equals_the_three_separate_calls(B, H, HV, taps):
    """gdn_decode_layer's output, recurrent state and conv state equal the separate conv-step,
    recurrent-step and gated-norm calls bit for bit, with both slice widths of the step."""
    gen = torch.Generator().manual_seed(B + H + taps)
    C = 2 * H * 128 + HV * 128
    qkv = (torch.randn(B, C, generator=gen) * 2).to(torch.bfloat16).cuda()
    cs = torch.randn(B, C, taps, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(C, 4, generator=gen) * 0.5).to(torch.bfloat16).cuda()
    g = (-torch.exp(torch.randn(B, HV, generator=gen) * 0.5 - 3.0)).cuda()
    beta = torch.sigmoid(torch.randn(B, HV, generator=gen)).to(torch.bfloat16).cuda()
    state = (torch.randn(B, HV, 128, 128, generator=gen) * 0.02).cuda()
    z = torch.randn(B, HV, 128, generator=gen).to(torch.bfloat16).cuda()
    nw = (torch.rand(128, generator=gen) + 0.5).to(torch.bfloat16).cuda()

    cs_sep, st_sep = cs.clone(), state.clone()
    y = gdn.causal_conv1d_step(qkv, cs_sep, w)
    kd = H * 128
    q, k, v = y[:, :kd].view(B, 1, H, 128), y[:, kd:2 * kd].view(B, 1, H, 128), y[:, 2 * kd:].view(B, 1, HV, 128)
    o, st_sep = gdn.gated_delta_rule_step(q, k, v, g.view(B, 1, HV), beta.view(B, 1, HV), initial_state=st_sep,
                                          output_final_state=True)
    out_sep = gdn.gated_rms_norm(o.view(-1, 128), z.view(-1, 128), nw).view(B, HV, 128)

    cs_f, st_f = cs.clone(), state.clone()
    out_f = gdn.decode_layer_step(qkv, cs_f, w, g, beta, st_f, z, nw, H)
    assert same_bits(cs_f, cs_sep)
    assert same_bits(st_f, st_sep)
    assert same_bits(out_f, out_sep)


def test_decode_layer_rejects_bad_arguments_before_any_launch():
    """Non-bf16 activations or weights (which the kernels would read as bf16), and z, norm
    weight, g or beta of the wrong size, raise ValueError; the states are left untouched."""
    B, H, HV, taps = 4, 2, 4, 3
    C = 2 * H * 128 + HV * 128
    dev = "cuda"
    ok = dict(qkv=torch.randn(B, C, device=dev).to(torch.bfloat16),
              conv_state=torch.zeros(B, C, taps, device=dev, dtype=torch.bfloat16),
              conv_weight=torch.randn(C, 4, device=dev).to(torch.bfloat16),
              g=-torch.rand(B, HV, device=dev), beta=torch.rand(B, HV, device=dev).to(torch.bfloat16),
              state=torch.zeros(B, HV, 128, 128, device=dev),
              z=torch.randn(B, HV, 128, device=dev).to(torch.bfloat16),
              norm_weight=torch.ones(128, device=dev, dtype=torch.bfloat16))
    bad = [("qkv", ok["qkv"].float()), ("conv_weight", ok["conv_weight"].float()), ("z", ok["z"].float()),
           ("norm_weight", ok["norm_weight"].float()), ("norm_weight", ok["norm_weight"][:64]),
           ("z", ok["z"][:, :2]), ("g", ok["g"][:, :2]), ("beta", ok["beta"][:2])]
    for name, value in bad:
        args = dict(ok, **{name: value})
        with pytest.raises(ValueError):
            gdn.decode_layer_step(args["qkv"], args["conv_state"], args["conv_weight"], args["g"], args["beta"],
                                  args["state"], args["z"], args["norm_weight"], H)
    torch.cuda.synchronize()
    assert not ok["state"].any() and not ok["conv_state"].any()
