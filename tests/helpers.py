"""Shared input generators and comparisons for the tests."""

import torch


def gdn_inputs(seed, B, T, H, HV, dtype=torch.bfloat16, D=128, state=True, normalise=True):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, D, generator=gen)
    k = torch.randn(B, T, H, D, generator=gen)
    if normalise:
        q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6)
        k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    v = torch.randn(B, T, HV, D, generator=gen)
    g = -torch.exp(torch.randn(B, T, HV, generator=gen) * 0.5 - 3.0)
    beta = torch.sigmoid(torch.randn(B, T, HV, generator=gen))
    h0 = torch.randn(B, HV, D, D, generator=gen) * 0.02 if state else None
    return q.to(dtype), k.to(dtype), v.to(dtype), g, beta.to(dtype), h0


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp(min=1e-30)).item()


def maxabs(a, b):
    return (a.detach().double().cpu() - b.detach().double().cpu()).abs().max().item()


def cuda(*ts):
    return [None if t is None else t.cuda() for t in ts]


def same_bits(x, y):
    x, y = x.detach().cpu(), y.detach().cpu()
    if x.dtype != y.dtype or x.shape != y.shape:
        return False
    view = {torch.float32: torch.int32, torch.bfloat16: torch.int16}[x.dtype]
    nan = x.isnan()
    if not torch.equal(nan, y.isnan()):
        return False
    return torch.equal(x.view(view)[~nan], y.view(view)[~nan])


def bf16_ulps(x, y):
    """Number of differing bf16 elements and the largest distance in units of the last place."""
    x, y = x.detach().cpu().contiguous(), y.detach().cpu().contiguous()
    assert x.dtype == y.dtype == torch.bfloat16 and x.shape == y.shape
    a = x.view(torch.int16).to(torch.int32)
    b = y.view(torch.int16).to(torch.int32)
    # map sign-magnitude bit patterns to a monotonic integer line
    a = torch.where(a < 0, -(a & 0x7FFF), a)
    b = torch.where(b < 0, -(b & 0x7FFF), b)
    d = (a - b).abs()
    return int((d > 0).sum()), int(d.max()) if d.numel() else 0


def assert_bf16_matches_cpu(gpu, cpu, max_frac=1e-6):
    """GPU output against the CPU oracle: bitwise, except that SiLU's exp may differ in the
    last fp32 bit between the CPU's vectorised exp and CUDA's expf, which can move a bf16
    rounding by one ulp on rare elements."""
    n, ulp = bf16_ulps(gpu, cpu)
    assert ulp <= 1 and n <= max(1, int(max_frac * cpu.numel())), (n, ulp, cpu.numel())
