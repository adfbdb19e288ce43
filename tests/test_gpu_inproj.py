"""GPU parity of the merged input projection with the causal conv in the GEMM epilogue: the
projection against PyTorch's bf16 matmul (the reference's nn.Linear on CUDA, fp32 accumulation),
and the conv part against the library's conv kernel on that matmul's output (same rounding), so
that only a different summation order of the GEMM can move a bf16 value, by one ulp; and both
against a float64 product and conv computed on the CPU, within the reference's bf16 roundings."""

import pytest
import torch

import jeeves_b200 as gdn
from tests.helpers import bf16_ulps

pytestmark = pytest.mark.gpu


def _case(seed, T, K, C, rest):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(T, K, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(C + rest, K, generator=gen) * K ** -0.5).to(torch.bfloat16).cuda()
    cw = (torch.randn(C, 4, generator=gen) * 0.5).to(torch.bfloat16).cuda()
    return x, w, cw


def _close(got, want, max_ulps=1, frac=0.01):
    """At most `frac` of the values differ, each by at most `max_ulps` bf16 ulps of the larger
    magnitude (values near zero, where a tiny absolute difference spans many ulps, by 1e-3)."""
    g, w = got.float().cpu(), want.float().cpu()
    tol = max_ulps * 2.0 ** -7 * torch.maximum(g.abs(), w.abs()) + 1e-3
    assert bool(((g - w).abs() <= tol).all()), float(((g - w).abs() - tol).max())
    n, _ = bf16_ulps(got, want)
    assert n <= max(1, int(frac * got.numel())), (n, got.numel())


# The kernel (single CTAs, or CTA pairs once the pair tiles fill the GPU) and the tile width
# (tokens per tile, 64 .. 256) follow the shape; on a 148-SM B200 these shapes reach every width of
# both: single 64 (the first three), 256, 224, 160, 128, 96, 192; pairs 224, 64, 96, 128, 160, 192,
# 224, 256 (the 9B-shaped projection, 4096 tokens x 12,352 channels, takes pairs of 256).
SHAPES = [(300, 256, 512, 264), (125, 128, 256, 0), (1, 64, 8, 8), (2024, 128, 2048, 256), (571, 128, 4096, 768),
          (382, 128, 4096, 768), (284, 128, 4096, 768), (200, 128, 4096, 768), (321, 128, 4096, 2304),
          (4096, 512, 1024, 520), (2206, 128, 256, 128), (3350, 128, 256, 128), (516, 128, 4096, 2176),
          (516, 128, 4096, 3456), (659, 128, 4096, 3456), (763, 128, 4096, 3456), (893, 128, 4096, 3456)]


@pytest.mark.parametrize("T,K,C,rest", SHAPES)
def test_in_proj_conv_matches_matmul_then_conv(T, K, C, rest):
    x, w, cw = _case(T + K, T, K, C, rest)
    out = gdn.in_proj_conv(x, w, cw, C)
    y = x @ w.T  # bf16 output, fp32 accumulation
    _close(out[:, C:], y[:, C:])
    if C:
        _close(out[:, :C], gdn.causal_conv1d(y[None, :, :C].contiguous(), cw)[0], max_ulps=2, frac=0.02)


@pytest.mark.parametrize("T", [1, 63, 64, 65, 127, 128, 129, 253, 256, 257, 700])
def test_in_proj_without_conv_channels_matches_matmul(T):
    """A projection with no conv channels (the decode-time projections, the output projection):
    its tiles carry no window tokens, so every column of a tile is an output token. Token counts
    on both sides of the tile edges."""
    x, w, cw = _case(T, T, 256, 0, 1152)
    out = gdn.in_proj_conv(x, w, cw, 0)
    _close(out, x @ w.T)


@pytest.mark.parametrize("T,K,N", [(1, 4096, 8192), (32, 4096, 8192), (256, 4096, 8192), (100, 4096, 4096),
                                   (17, 4288, 1152), (256, 2048, 640)])
def test_in_proj_split_k_decode_batches(T, K, N):
    """Decode-sized batches without conv channels split K over a cluster of 2 to 8 CTAs (so that
    the tiles, one per 128 weight rows, cover the SMs) and add the partial sums through distributed
    shared memory in a fixed order: against matmul, and the same bits on a repeated call. K = 4288
    gives the CTAs K ranges of unequal length."""
    x, w, cw = _case(T + N, T, K, 0, N)
    out = gdn.in_proj_conv(x, w, cw, 0)
    _close(out, x @ w.T)
    assert torch.equal(out, gdn.in_proj_conv(x, w, cw, 0))


@pytest.mark.parametrize("lens,K,C,rest", [([70, 1, 129, 0, 100, 3], 192, 256, 72),        # single CTAs
                                           ([700, 2, 900, 0, 3, 419, 1], 128, 2048, 256),  # pairs, 160 tokens
                                           ([1000, 1, 0, 700, 3, 502], 128, 256, 128),     # pairs, 64 tokens
                                           ([400, 1, 0, 300, 192], 128, 4096, 3456)])      # pairs, 256 tokens
def test_in_proj_conv_packed_sequences_and_conv_state(lens, K, C, rest):
    T = sum(lens)
    x, w, cw = _case(7, T, K, C, rest)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    out, state = gdn.in_proj_conv(x, w, cw, C, cu_seqlens=cu, conv_state=True)
    y = x @ w.T
    _close(out[:, C:], y[:, C:])
    _close(out[:, :C], gdn.causal_conv1d(y[None, :, :C].contiguous(), cw, cu_seqlens=cu)[0], max_ulps=2, frac=0.02)
    for n, (a, b) in enumerate(zip(cu[:-1].tolist(), cu[1:].tolist())):
        want = torch.zeros(C, 4, dtype=torch.bfloat16, device="cuda")
        m = min(4, b - a)
        if m:
            want[:, 4 - m:] = y[b - m:b, :C].T
        _close(state[n], want)


@pytest.mark.parametrize("T,C,rest", [(2, 512, 136), (700, 512, 136), (893, 4096, 3456)])
def test_in_proj_conv_dense_conv_state(T, C, rest):
    x, w, cw = _case(11, T, 128, C, rest)
    out, state = gdn.in_proj_conv(x, w, cw, C, conv_state=True)
    y = x @ w.T
    want = torch.zeros(1, C, 4, dtype=torch.bfloat16, device="cuda")
    want[0, :, 4 - min(4, T):] = y[-min(4, T):, :C].T
    _close(state, want)
    _close(out[:, C:], y[:, C:])


def _bf16_ulp(v):
    """One bf16 unit in the last place of each value (2^(e-8) for |v| = m 2^e, 0.5 <= m < 1)."""
    return torch.ldexp(torch.ones_like(v), torch.frexp(v)[1] - 8)


def _conv64(y, cw):
    """The causal depthwise conv + SiLU of model/model.py:199-204 in float64, zeros before the
    first token, on a [T, C] float64 projection: (SiLU output, conv sum)."""
    T, C = y.shape
    taps = cw.shape[-1]
    yp = torch.cat([torch.zeros(taps - 1, C, dtype=torch.float64), y])
    acc = sum(cw[:, i].double()[None, :] * yp[i:i + T] for i in range(taps))
    return acc * torch.sigmoid(acc), acc


@pytest.mark.parametrize("T,K,C,rest", [(700, 4096, 2048, 512),     # single CTAs
                                        (4096, 4096, 8192, 4160),   # the 9B-shaped projection, CTA pairs
                                        (256, 4096, 0, 8192),       # decode batch, K split over clusters
                                        (32, 4096, 0, 8192)])
def test_in_proj_conv_matches_float64_cpu_product(T, K, C, rest):
    """The projection and its conv against a float64 product and conv computed on the CPU (no
    intermediate rounding): each projected channel within one bf16 ulp (or 1e-3) of the exactly
    rounded product, under 1 % of them off at all; each conv channel within the bound that the
    reference's roundings allow (the projection, the conv sum and the SiLU output are each rounded
    to bf16, model/model.py:199-204): one ulp of the output, plus 1.1 (the largest slope of SiLU)
    times one ulp of the conv sum and the sum over the window of |w| times one ulp of the
    projected value, plus 1e-5. Each ulp term is twice the half-ulp rounding error it covers."""
    x, w, cw = _case(T * 3 + K + C, T, K, C, rest)
    out = gdn.in_proj_conv(x, w, cw, C).cpu()
    y64 = x.cpu().double() @ w.cpu().double().T
    _close(out[:, C:], y64[:, C:].to(torch.bfloat16))
    if C:
        got = out[:, :C].double()
        want, acc = _conv64(y64[:, :C], cw.cpu())
        taps = cw.shape[-1]
        uy = _bf16_ulp(y64[:, :C].abs())
        uyp = torch.cat([torch.zeros(taps - 1, C, dtype=torch.float64), uy])
        spread = sum(cw[:, i].cpu().double().abs()[None, :] * uyp[i:i + T] for i in range(taps))
        bound = _bf16_ulp(torch.maximum(got.abs(), want.abs())) + 1.1 * (_bf16_ulp(acc.abs()) + spread) + 1e-5
        excess = (got - want).abs() - bound
        assert bool((excess <= 0).all()), float(excess.max())


def test_in_proj_conv_leaves_no_device_error():
    from jeeves_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.load().gdn_device_error(None, 0) == 0
