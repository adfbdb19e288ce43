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
