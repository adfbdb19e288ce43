"""GPU parity of the fp8-weight projection (the reference's FP8Linear / fp8_matmul,
inference/fp8.py:62-190) on the tcgen05 kernel, to the reference's own bar
(inference/cuda_test.py:75-95): on its four weight shapes and nine row counts, with outlier
columns in odd rows and tiny rows, at least 99.5 % of the outputs equal the exact result
(x @ codes^T * scale in float64) rounded once to bf16, every output is finite, and a second call
gives the same bits. With the conv in the epilogue, the conv columns against the conv kernel on
the plain fp8 output (within the fused kernel's one-ulp SiLU), the rest bit-identical."""

import pytest
import torch

import jeeves_b200 as gdn
from tests.helpers import bf16_ulps

pytestmark = pytest.mark.gpu

FP8 = torch.float8_e4m3fn
FP8_MAX_RECIPROCAL = float(torch.tensor(1 / torch.finfo(FP8).max, dtype=torch.float32))


def quantize_rows(weight):
    """Per-row e4m3 codes and fp32 scales as inference/fp8_weights.py:15-18 makes them."""
    w = weight.float()
    scale = w.abs().amax(1).clamp(min=1e-12) * FP8_MAX_RECIPROCAL
    return (w / scale[:, None]).to(FP8).contiguous(), scale.contiguous()


def _weights(N, K, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.rand(N, K, generator=gen, device="cuda") * 2 - 1) * K ** -0.5  # nn.Linear's uniform init
    return quantize_rows(w.to(torch.bfloat16))


def _rows(M, K, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, generator=gen, device="cuda").to(torch.bfloat16)
    x[1::2, 0] = 1e5        # outliers: the activation scaling
    x[2::4] *= 2 ** -20     # tiny rows: fp16 subnormals unless scaled up
    return x


@pytest.mark.parametrize("N,K", [(4096, 4096), (1024, 12288), (1040, 4096), (17408, 4096)])
def test_fp8_linear_matches_the_exact_result(N, K):
    codes, scale = _weights(N, K, N + K)
    for M in (1, 4, 12, 16, 17, 48, 256, 300, 1024):
        x = _rows(M, K, M)
        out = gdn.fp8_linear(x, codes, scale)
        exact = ((x.double() @ codes.double().t()) * scale.double()).to(torch.bfloat16)
        same = (out == exact).double().mean().item()
        assert out.isfinite().all(), (N, K, M)
        assert same >= 0.995, (N, K, M, same)
        assert torch.equal(out, gdn.fp8_linear(x, codes, scale)), (N, K, M)


def test_fp8_linear_keeps_leading_dims():
    codes, scale = _weights(1024, 512, 3)
    x = _rows(24, 512, 4).view(2, 12, 512)
    out = gdn.fp8_linear(x, codes, scale)
    assert out.shape == (2, 12, 1024)
    assert torch.equal(out.view(24, 1024), gdn.fp8_linear(x.view(24, 512), codes, scale))


def _close(got, want, max_ulps=2, frac=0.02):
    g, w = got.float().cpu(), want.float().cpu()
    tol = max_ulps * 2.0 ** -7 * torch.maximum(g.abs(), w.abs()) + 1e-3
    assert bool(((g - w).abs() <= tol).all()), float(((g - w).abs() - tol).max())
    n, _ = bf16_ulps(got, want)
    assert n <= max(1, int(frac * got.numel())), (n, got.numel())


@pytest.mark.parametrize("T,K,C,rest", [(300, 256, 512, 264), (1, 128, 256, 0), (2024, 512, 2048, 256)])
def test_fp8_in_proj_conv(T, K, C, rest):
    codes, scale = _weights(C + rest, K, T)
    x = _rows(T, K, K)
    x[1::2, 0] = 3.0  # moderate outliers: the conv sums stay in range
    gen = torch.Generator(device="cuda").manual_seed(7)
    cw = (torch.randn(C, 4, generator=gen, device="cuda") * 0.5).to(torch.bfloat16)
    out = gdn.in_proj_conv(x, codes, cw, C, weight_scale=scale)
    plain = gdn.fp8_linear(x, codes, scale)
    assert torch.equal(out[:, C:], plain[:, C:])
    _close(out[:, :C], gdn.causal_conv1d(plain[None, :, :C].contiguous(), cw)[0])


def test_fp8_in_proj_conv_packed_sequences_and_state():
    lens = [300, 1, 0, 257, 3]
    T, K, C, rest = sum(lens), 256, 512, 136
    codes, scale = _weights(C + rest, K, 11)
    x = _rows(T, K, 12)
    x[1::2, 0] = 3.0
    cw = (torch.randn(C, 4, device="cuda") * 0.5).to(torch.bfloat16)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    out, state = gdn.in_proj_conv(x, codes, cw, C, cu_seqlens=cu, conv_state=True, weight_scale=scale)
    plain = gdn.fp8_linear(x, codes, scale)
    assert torch.equal(out[:, C:], plain[:, C:])
    _close(out[:, :C], gdn.causal_conv1d(plain[None, :, :C].contiguous(), cw, cu_seqlens=cu)[0])
    for n, (a, b) in enumerate(zip(cu[:-1].tolist(), cu[1:].tolist())):
        want = torch.zeros(C, 4, dtype=torch.bfloat16, device="cuda")
        m = min(4, b - a)
        if m:
            want[:, 4 - m:] = plain[b - m:b, :C].T
        assert torch.equal(state[n], want), n


def _fp8_call(lib, x, codes, scale, cw, C, ws_bytes):
    T, K = x.shape
    N = codes.shape[0]
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
    st = lib.gdn_in_proj_conv_fp8(x.data_ptr(), K, codes.data_ptr(), K, scale.data_ptr(),
                                  cw.data_ptr() if C else None, None, out.data_ptr(), N, None, ws.data_ptr(),
                                  ws_bytes, T, K, N, C, 1, 4, torch.cuda.current_stream().cuda_stream)
    assert st == 0, st
    return out


def test_fp8_prefill_on_cta_pairs_and_on_single_ctas():
    """With the prefill workspace (gdn_in_proj_fp8_prefill_workspace_size) a shape whose token
    tiles fill the GPU converts the codes to fp16 once and runs its products on CTA pairs; with
    the base workspace the same call runs on single CTAs that convert tile by tile. Both meet the
    reference's bar; with the conv in the epilogue, the conv columns against the conv kernel on the
    plain output and the rest bit-identical to it."""
    from jeeves_b200 import _lib
    lib = _lib.load()
    T, K, C, rest = 2048, 1024, 8192, 256
    N = C + rest
    codes, scale = _weights(N, K, 21)
    x = _rows(T, K, 22)
    x[1::2, 0] = 3.0
    cw = (torch.randn(C, 4, generator=torch.Generator(device="cuda").manual_seed(5), device="cuda") * 0.5).to(
        torch.bfloat16)
    exact = ((x.double() @ codes.double().t()) * scale.double()).to(torch.bfloat16)
    small = lib.gdn_in_proj_fp8_workspace_size(T, K)
    for conv in (0, C):
        big = lib.gdn_in_proj_fp8_prefill_workspace_size(T, K, N, conv)
        assert big == small + (256 - small % 256) % 256 + N * K * 2  # this shape runs on CTA pairs
        plain_pair = _fp8_call(lib, x, codes, scale, cw, 0, big)
        plain_single = _fp8_call(lib, x, codes, scale, cw, 0, small)
        for out in (plain_pair, plain_single):
            assert out.isfinite().all()
            assert (out == exact).double().mean().item() >= 0.995
        if conv:
            for ws_bytes, plain in ((big, plain_pair), (small, plain_single)):
                out = _fp8_call(lib, x, codes, scale, cw, C, ws_bytes)
                assert torch.equal(out[:, C:], plain[:, C:])
                _close(out[:, :C], gdn.causal_conv1d(plain[None, :, :C].contiguous(), cw)[0])
    assert torch.equal(plain_pair, _fp8_call(lib, x, codes, scale, cw, 0, big))


def test_fp8_rejects_bad_arguments():
    codes, scale = _weights(256, 128, 1)
    x = _rows(8, 128, 2)
    with pytest.raises(ValueError):
        gdn.in_proj_conv(x, codes, None, 0)  # no scales
    with pytest.raises(ValueError):
        gdn.in_proj_conv(x, codes, None, 0, weight_scale=scale[:10])


def test_fp8_leaves_no_device_error():
    from jeeves_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.load().gdn_device_error(None, 0) == 0
