"""The drafter's attention-side kernels of a gated-delta layer (CUDA only).

* ``decode_attention(q, k_cache, v_cache, mask, scale)`` replaces ``decode_attention``
  (``model/model.py:354-361``; CUDA kernel ``model/triton_kernels.py:117-211``): attention of a
  few query rows per key head over a KV cache with an additive mask, on tcgen05;
* ``rotary(x, cos, sin)`` replaces ``apply_rotary`` with per-row (3-D) cos / sin
  (``model/model.py:182-196``; ``model/triton_kernels.py:54-75``), bit for bit;
* ``rotate_into_cache(...)`` replaces ``rotate_into_cache`` (``model/model.py:342-351``;
  ``model/triton_kernels.py:214-262``), bit for bit.

Errors are ``ValueError`` with the reference's wording where the reference raises one.
"""

from __future__ import annotations

import torch

from . import _lib
from .gated_delta import _ptr, _require_cuda, _stream

MAX_ROWS = 64  # query rows per key head (R * H / Hkv), as DECODE_ATTENTION_MAX_ROWS


def decode_attention_supported(q, k_cache, v_cache, mask) -> bool:
    """The configurations the kernel runs: bf16, head dim 128 or 256, H a multiple of Hkv, at most
    64 query rows per key head, a ``(B, 1, R, L)`` mask, caches with at least B rows and L
    positions, unit inner strides and 16-byte aligned rows."""
    if q.dim() != 4 or k_cache.dim() != 4 or mask.dim() != 4:
        return False
    B, R, H, D = q.shape
    Hkv, L = k_cache.shape[2], mask.shape[-1]
    tensors = (q, k_cache, v_cache, mask)
    return (all(t.dtype == torch.bfloat16 and t.is_cuda for t in tensors) and D in (128, 256) and H % Hkv == 0
            and R * (H // Hkv) <= MAX_ROWS and tuple(mask.shape) == (B, 1, R, L) and v_cache.shape == k_cache.shape
            and k_cache.shape[0] >= B and k_cache.shape[1] >= L and k_cache.shape[3] == D
            and all(t.stride(-1) == 1 for t in tensors)
            and all(_rows_aligned(t, dims) for t, dims in ((q, (0, 1, 2)), (k_cache, (0, 1, 2)),
                                                           (v_cache, (0, 1, 2)), (mask, (0, 2)))))


def _rows_aligned(t: torch.Tensor, dims) -> bool:
    """Every row start 16-byte aligned: the base, and the strides of ``dims`` in 8-element steps
    (an empty tensor has no rows to read)."""
    return t.numel() == 0 or (t.data_ptr() % 16 == 0 and all(t.stride(d) % 8 == 0 for d in dims))


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, mask: torch.Tensor,
                     scale: float) -> torch.Tensor:
    """``o[b, r, h] = softmax(scale q k^T + mask) v`` over the first ``mask.shape[-1]`` keys of cache
    rows ``0..B-1``, key head ``h // (H // Hkv)``; q ``[B, R, H, D]``, caches ``[rows, slots, Hkv,
    D]``, mask ``[B, 1, R, L]``, all bf16. Rows whose keys are all masked get zeros."""
    what = "decode_attention"
    _require_cuda(what, q, k_cache, v_cache, mask)
    if not decode_attention_supported(q, k_cache, v_cache, mask):
        raise ValueError(f"decode_attention needs bfloat16 inputs with contiguous last dims, a head dim of 128 or 256, "
                         f"query heads a multiple of the key heads, at most {MAX_ROWS} query rows per key head, a "
                         f"(B, 1, R, L) mask and caches with at least B rows and L positions; got q {tuple(q.shape)}, "
                         f"k_cache {tuple(k_cache.shape)}, v_cache {tuple(v_cache.shape)}, mask {tuple(mask.shape)}")
    B, R, H, D = q.shape
    Hkv, L = k_cache.shape[2], mask.shape[-1]
    o = torch.empty(B, R, H, D, dtype=q.dtype, device=q.device)
    lib = _lib.load()
    ws_bytes = lib.gdn_decode_attention_workspace_size(B, Hkv, L, D)
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
    status = lib.gdn_decode_attention(
        q.data_ptr(), *q.stride()[:3], k_cache.data_ptr(), *k_cache.stride()[:3], v_cache.data_ptr(),
        *v_cache.stride()[:3], mask.data_ptr(), mask.stride(0), mask.stride(2), o.data_ptr(), B, R, H, Hkv, D, L,
        k_cache.shape[0], k_cache.shape[1], float(scale), _ptr(workspace), ws_bytes, _stream())
    _lib.check(status, what)
    return o


def _cos_rows(t: torch.Tensor, B: int, T: int, F: int) -> torch.Tensor:
    return t.float().expand(B, T, F).contiguous()


def rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``apply_rotary(x, cos, sin)`` for x ``[B, T, H, D]`` bf16 and cos / sin broadcastable to
    ``[B, T, F]`` (2F <= D), with the eager path's bf16 rounding."""
    what = "rotary"
    _require_cuda(what, x, cos, sin)
    B, T, H, D = x.shape
    n_freqs = cos.shape[-1]
    if x.dtype != torch.bfloat16:
        raise ValueError(f"x: expected bfloat16, got {x.dtype}")
    if 2 * n_freqs > D:
        raise ValueError(f"x: head dim {D} is smaller than the {2 * n_freqs} rotary dims")
    x = x.contiguous()
    cos, sin = _cos_rows(cos, B, T, n_freqs), _cos_rows(sin, B, T, n_freqs)
    out = torch.empty_like(x)
    status = _lib.load().gdn_rotary(x.data_ptr(), cos.data_ptr(), sin.data_ptr(), out.data_ptr(), B, T, H, D, n_freqs,
                                    _stream())
    _lib.check(status, what)
    return out


def rotate_into_cache(k, v, qm, km, vm, cos_c, sin_c, cos_m, sin_m, k_cache, v_cache, rows, positions,
                      tail_start: int) -> torch.Tensor:
    """Rotated keys and values of the K candidate rows into ``k_cache`` / ``v_cache`` at ``(rows,
    positions)``, rotated mask-row keys and values at cache row b, positions ``tail_start + m``;
    returns the rotated mask-row queries ``[B, M, H, D]``."""
    what = "rotate_into_cache"
    _require_cuda(what, k, v, qm, km, vm, cos_c, sin_c, cos_m, sin_m, k_cache, v_cache, rows, positions)
    B, K, H, D = k.shape
    M = qm.shape[1]
    n_freqs = cos_c.shape[-1]
    if any(t.dtype != torch.bfloat16 for t in (k, v, qm, km, vm, k_cache, v_cache)):
        raise ValueError("k, v, qm, km, vm and the caches must be bfloat16")
    if v.shape != k.shape or not qm.shape == km.shape == vm.shape == (B, M, H, D) or rows.shape != (B, K) \
            or positions.shape != (B, K):
        raise ValueError(f"expected k and v of shape (B, K, H, D), qm, km and vm of shape (B, M, H, D), and rows and "
                         f"positions of shape (B, K); got k {tuple(k.shape)}, v {tuple(v.shape)}, qm {tuple(qm.shape)}, "
                         f"km {tuple(km.shape)}, vm {tuple(vm.shape)}, rows {tuple(rows.shape)}, "
                         f"positions {tuple(positions.shape)}")
    if not (qm.stride() == km.stride() == vm.stride() and qm.stride()[2:] == (D, 1)):
        raise ValueError("qm, km and vm must share strides, with each head's D values contiguous")
    if k_cache.stride() != v_cache.stride() or k_cache.stride()[2:] != (D, 1) or 2 * n_freqs > D:
        raise ValueError("the caches must share strides with contiguous heads, and the rotary dims must fit the head dim")
    q_out = torch.empty(B, M, H, D, dtype=qm.dtype, device=qm.device)
    cos_c, sin_c = _cos_rows(cos_c, B, K, n_freqs), _cos_rows(sin_c, B, K, n_freqs)
    cos_m, sin_m = _cos_rows(cos_m, B, M, n_freqs), _cos_rows(sin_m, B, M, n_freqs)
    k, v = k.contiguous(), v.contiguous()
    rows = rows.to(torch.int64)
    positions = positions.to(torch.int64).contiguous()
    status = _lib.load().gdn_rotate_into_cache(
        k.data_ptr(), v.data_ptr(), qm.data_ptr(), km.data_ptr(), vm.data_ptr(), qm.stride(0), qm.stride(1),
        cos_c.data_ptr(), sin_c.data_ptr(), cos_m.data_ptr(), sin_m.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        k_cache.stride(0), k_cache.stride(1), q_out.data_ptr(), rows.data_ptr(), rows.stride(0), rows.stride(1),
        positions.data_ptr(), int(tail_start), B, K, M, H, D, n_freqs, _stream())
    _lib.check(status, what)
    return q_out
