"""Delta-rule gates on the GPU against PyTorch's CUDA eager ops (bit for bit, the comparison
the reference makes for its own kernel, model/triton_kernels_test.py:78-100) and against the
CPU reference's golden vectors."""

import pytest
import torch

import jeeves_b200 as gdn
import oracle
from tests.helpers import bf16_ulps, same_bits

pytestmark = pytest.mark.gpu


def _edge_inputs():
    gen = torch.Generator().manual_seed(6)
    HV = 32
    merged = (torch.randn(3, 5, 64 + 2 * HV, generator=gen) * 12).to(torch.bfloat16)
    b, a = merged[..., 64:64 + HV], merged[..., 64 + HV:]
    # softplus of about -103 to -87 is subnormal: a flush to zero would differ from PyTorch
    a[0, 0] = torch.linspace(-110, -80, HV)
    b[0, 0] = torch.linspace(-100, 100, HV)
    a[0, 1, :4] = torch.tensor([float("inf"), float("-inf"), 30.0, -30.0])
    b[0, 1, :2] = torch.tensor([float("inf"), float("-inf")])
    a[1, 0, 0] = b[1, 0, 1] = float("nan")
    rate = -torch.rand(HV, generator=gen).exp()
    valid = torch.rand(3, 5, generator=gen) < 0.7
    dts = (torch.randn(HV, generator=gen), torch.randn(HV, generator=gen).to(torch.bfloat16))
    return merged, HV, rate, valid, dts


@pytest.mark.parametrize("with_valid", [False, True])
@pytest.mark.parametrize("dt_index", [0, 1])
def test_delta_gates_bitwise_equal_to_cuda_eager(with_valid, dt_index):
    merged, HV, rate, valid, dts = _edge_inputs()
    m = merged.cuda()
    b, a = m[..., 64:64 + HV], m[..., 64 + HV:]  # strided views, as the engine passes them
    dt, r = dts[dt_index].cuda(), rate.cuda()
    v = valid.cuda() if with_valid else None
    beta, g = gdn.delta_gates(b, a, dt, r, v)
    beta_ref, g_ref = oracle.delta_gates(b, a, dt, r, v)  # the eager formula, run by torch on CUDA
    assert same_bits(beta, beta_ref)
    assert same_bits(g, g_ref)


def test_delta_gates_golden(golden):
    c = golden("delta_gates")
    args = [c[k].cuda() for k in ("b", "a", "dt_bias", "rate")]
    valid = c.get("valid")
    beta, g = gdn.delta_gates(*args, valid.cuda() if valid is not None else None)
    # CPU and CUDA exp / log1p may differ in the last fp32 bit
    n, ulp = bf16_ulps(beta, c["beta"])
    assert ulp <= 1 and n <= max(1, beta.numel() // 1000)
    ref = c["g"].float()
    assert torch.allclose(g.cpu(), ref, rtol=4 * 2 ** -23, atol=0)


def test_delta_gates_rejects_bad_inputs():
    b = torch.zeros(2, 4, dtype=torch.bfloat16, device="cuda")
    dt, r = torch.zeros(4, device="cuda"), -torch.ones(4, device="cuda")
    with pytest.raises(ValueError, match="bfloat16"):
        gdn.delta_gates(b.float(), b, dt, r)
    with pytest.raises(ValueError, match="valid"):
        gdn.delta_gates(b, b, dt, r, torch.ones(2, device="cuda"))
    with pytest.raises(ValueError, match="dt_bias"):
        gdn.delta_gates(b, b, torch.zeros(3, device="cuda"), r)


def _gated_inputs(seed, B, T, H, HV, dt_f32=True, with_valid=False):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, 128, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, T, H, 128, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, T, HV, 128, generator=gen).to(torch.bfloat16)
    proj = (torch.randn(B, T, 2 * HV + 8, generator=gen) * 3).to(torch.bfloat16)  # one merged projection
    proj[..., 0, 8 + HV:8 + HV + 4] = 25.0  # softplus beyond 20 takes the identity branch
    b, a = proj[..., 8:8 + HV], proj[..., 8 + HV:]
    dt = torch.randn(HV, generator=gen) if dt_f32 else torch.randn(HV, generator=gen).to(torch.bfloat16)
    rate = -torch.rand(HV, generator=gen).exp() * 0.05
    valid = (torch.rand(B, T, generator=gen) < 0.8) if with_valid else None
    h0 = torch.randn(B, HV, 128, 128, generator=gen) * 0.02
    dev = [None if t is None else t.cuda() for t in (q, k, v, b, a, dt, rate, valid, h0)]
    return dev


@pytest.mark.parametrize("B,T,H,HV,dt_f32,with_valid", [
    (1, 700, 16, 32, True, False),   # the cooperative launch (64 scan CTAs)
    (3, 130, 16, 32, False, True),   # factor kernel + scan kernel, bf16 dt_bias, a valid mask
    (2, 65, 2, 4, True, True),
])
def test_chunk_gates_equal_gates_then_chunk_bitwise(B, T, H, HV, dt_f32, with_valid):
    """The gates computed by the prefill's factor work give the same bits as delta_gates followed
    by gated_delta_rule_chunk (the engine's extend pass, inference/engine.py:378-379)."""
    q, k, v, b, a, dt, rate, valid, h0 = _gated_inputs(B * 10 + T, B, T, H, HV, dt_f32, with_valid)
    beta, g = gdn.delta_gates(b, a, dt, rate, valid)
    o_ref, s_ref = gdn.gated_delta_rule_chunk(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    o, s = gdn.gated_delta_rule_chunk_gates(q, k, v, b, a, dt, rate, valid, initial_state=h0, output_final_state=True)
    assert same_bits(o, o_ref) and same_bits(s, s_ref)


def test_packed_chunk_gates_equal_gates_then_chunk_bitwise():
    lens = [70, 300, 1, 129, 0, 257]
    q, k, v, b, a, dt, rate, valid, _ = _gated_inputs(5, 1, sum(lens), 16, 32, True, True)
    h0 = (torch.randn(len(lens), 32, 128, 128, generator=torch.Generator().manual_seed(6)) * 0.02).cuda()
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32).cuda()
    beta, g = gdn.delta_gates(b, a, dt, rate, valid)
    o_ref, s_ref = gdn.gated_delta_rule_chunk(q, k, v, g, beta, initial_state=h0, output_final_state=True, cu_seqlens=cu)
    o, s = gdn.gated_delta_rule_chunk_gates(q, k, v, b, a, dt, rate, valid, initial_state=h0, output_final_state=True,
                                            cu_seqlens=cu)
    assert same_bits(o, o_ref) and same_bits(s, s_ref)


@pytest.mark.parametrize("B,T,with_valid", [(4, 1, False), (3, 5, True)])
def test_step_gates_equal_gates_then_step_bitwise(B, T, with_valid):
    """Decode (T = 1) and verify (T = 5) steps with the gates computed in the recurrent kernel."""
    q, k, v, b, a, dt, rate, valid, h0 = _gated_inputs(B + T, B, T, 16, 32, True, with_valid)
    beta, g = gdn.delta_gates(b, a, dt, rate, valid)
    o_ref, s_ref = gdn.gated_delta_rule_step(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    o, s = gdn.gated_delta_rule_step_gates(q, k, v, b, a, dt, rate, valid, initial_state=h0, output_final_state=True)
    assert same_bits(o, o_ref) and same_bits(s, s_ref)


def test_fp32_chunk_gates_equal_gates_then_chunk_bitwise():
    q, k, v, b, a, dt, rate, _, h0 = _gated_inputs(9, 2, 40, 2, 4)
    q, k, v = q.float(), k.float(), v.float()
    beta, g = gdn.delta_gates(b, a, dt, rate)
    o_ref, s_ref = gdn.gated_delta_rule_chunk(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    o, s = gdn.gated_delta_rule_chunk_gates(q, k, v, b, a, dt, rate, initial_state=h0, output_final_state=True)
    assert same_bits(o, o_ref) and same_bits(s, s_ref)
