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
