"""Causal depthwise conv1d + SiLU with the reference's call signatures (CUDA only).

Replaces ``causal_conv1d`` / ``causal_conv1d_step`` (``model/model.py:199-214``) and
``conv_step`` / ``eager_conv_step`` (``model/model.py:324-339``,
``model/triton_kernels.py:303-325``). Errors follow ``model/triton_kernels.py:311-318``:
``ValueError`` with the expected and actual dtype and shape.
"""

from __future__ import annotations

import torch

from . import _lib
from .gated_delta import _require_cuda, _stream


def causal_conv1d(x: torch.Tensor, weight: torch.Tensor, cu_seqlens: torch.Tensor | None = None) -> torch.Tensor:
    """silu(depthwise causal conv(x)) for x ``[B, T, C]`` bf16 and weight ``[C, K]`` (or ``[C, 1, K]``)."""
    what = "causal_conv1d"
    _require_cuda(what, x, weight, cu_seqlens)
    if x.dim() != 3:
        raise ValueError(f"x: expected [B, T, C], got {tuple(x.shape)}")
    B, T, C = x.shape
    w = weight.reshape(C, -1)
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError(f"x, weight: expected bfloat16, got {x.dtype}, {w.dtype}")
    if x.stride(-1) != 1:
        x = x.contiguous()
    w = w.contiguous()
    y = torch.empty(B, T, C, dtype=x.dtype, device=x.device)
    cu = None
    rows = B
    if cu_seqlens is not None:
        if B != 1:
            raise ValueError(f"{what}: with cu_seqlens x is packed into a batch of 1, got batch {B}")
        cu = cu_seqlens.to(dtype=torch.int32).contiguous()
        rows = cu.numel() - 1
    status = _lib.load().gdn_conv1d_silu(x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), y.data_ptr(),
                                         None if cu is None else cu.data_ptr(), rows, T, C, w.shape[1], _stream())
    _lib.check(status, what)
    return y


def causal_conv1d_step(x: torch.Tensor, state: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """One decode token: x ``[B, C]``, state ``[B, C, taps]`` bf16 (updated in place), weight ``[C, K]``."""
    what = "causal_conv1d_step"
    _require_cuda(what, x, state, weight)
    B, C = x.shape
    w = weight.reshape(C, -1).contiguous()
    taps = state.shape[-1]
    if state.shape != (B, C, taps) or not state.is_contiguous() or state.dtype != torch.bfloat16:
        raise ValueError(f"state: expected a contiguous bfloat16 tensor of shape {(B, C, taps)}, got {state.dtype} "
                         f"{tuple(state.shape)}")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError(f"x, weight: expected bfloat16, got {x.dtype}, {w.dtype}")
    if x.stride(-1) != 1:
        x = x.contiguous()
    y = torch.empty(B, C, dtype=x.dtype, device=x.device)
    status = _lib.load().gdn_conv1d_silu_step(x.data_ptr(), x.stride(0), state.data_ptr(), w.data_ptr(), y.data_ptr(),
                                              B, C, taps, w.shape[1], _stream())
    _lib.check(status, what)
    return y


def conv_step(state, qkv, weight, key_dim: int, value_dim: int, head_k_dim: int, head_v_dim: int, ext_out=None):
    """Conv over the state window + T new tokens; returns ``(ext, q, k, v)`` like ``model/model.py:335-339``.

    q and k come back repeat-interleaved to the value heads, v ``[B, T, HV, head_v_dim]``, all
    contiguous; ``ext`` ``[B, C, taps + T]`` is written to ``ext_out`` when given.
    """
    what = "conv_step"
    _require_cuda(what, state, qkv, weight, ext_out)
    B, T, C = qkv.shape
    taps = state.shape[-1]
    k_heads, v_heads = key_dim // head_k_dim, value_dim // head_v_dim
    if key_dim % head_k_dim or value_dim % head_v_dim or v_heads % k_heads:
        raise ValueError(f"the key and value dims must hold whole heads, and the value heads a whole number per key head; "
                         f"got {key_dim}, {value_dim}")
    if qkv.stride(-1) != 1 or not state.is_contiguous() or C != 2 * key_dim + value_dim:
        raise ValueError("qkv needs contiguous channels, state and weight must be contiguous, and qkv must hold q, k and v")
    w = weight.reshape(C, -1)
    if state.shape != (B, C, taps) or any(t.dtype != torch.bfloat16 for t in (state, qkv, w)):
        raise ValueError(f"expected bfloat16 state of shape {(B, C, taps)} and weight of shape {(C, 1, w.shape[-1])}, got "
                         f"{state.dtype} {tuple(state.shape)} and {w.dtype} {tuple(weight.shape)}")
    w = w.contiguous()
    ext = torch.empty(B, C, taps + T, dtype=qkv.dtype, device=qkv.device) if ext_out is None else ext_out
    if ext.shape != (B, C, taps + T) or ext.dtype != torch.bfloat16 or not ext.is_contiguous():
        raise ValueError(f"ext_out: expected a contiguous bfloat16 tensor of shape {(B, C, taps + T)}, got {ext.dtype} "
                         f"{tuple(ext.shape)}")
    q = torch.empty(B, T, v_heads, head_k_dim, dtype=qkv.dtype, device=qkv.device)
    k = torch.empty_like(q)
    v = torch.empty(B, T, v_heads, head_v_dim, dtype=qkv.dtype, device=qkv.device)
    status = _lib.load().gdn_conv_step(state.data_ptr(), qkv.data_ptr(), qkv.stride(0), qkv.stride(1), w.data_ptr(),
                                       ext.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), B, T, taps, w.shape[1],
                                       key_dim, value_dim, head_k_dim, head_v_dim, _stream())
    _lib.check(status, what)
    return ext, q, k, v


eager_conv_step = conv_step


def conv_state_commit(ext: torch.Tensor, state: torch.Tensor, accepted: torch.Tensor) -> None:
    """After a verify step, keep the conv window of the accepted tokens: ``state[..., b, :, :] =
    ext[..., b, :, j : j + taps]`` with ``j = clamp(accepted[b], 0, T)`` (the gather of
    ``inference/engine.py:473-474``). ext ``[B, C, taps + T]`` or ``[layers, B, C, taps + T]`` (as
    ``conv_step`` writes it; the layer and row dims may be strided slices), state ``[B, C, taps]`` or
    ``[layers, B, C, taps]`` bf16 (same layout rule), accepted ``[B]`` integers. One launch for
    every layer."""
    what = "conv_state_commit"
    _require_cuda(what, ext, state, accepted)
    e4, s4 = (ext[None], state[None]) if ext.dim() == 3 else (ext, state)
    if e4.dim() != 4 or s4.dim() != 4 or e4.shape[:3] != s4.shape[:3]:
        raise ValueError(f"{what}: expected ext [layers, B, C, taps + T] and state [layers, B, C, taps], got "
                         f"{tuple(ext.shape)} and {tuple(state.shape)}")
    L, B, C, taps = s4.shape
    T = e4.shape[3] - taps
    if T < 0 or ext.dtype != torch.bfloat16 or state.dtype != torch.bfloat16:
        raise ValueError(f"{what}: expected bfloat16 ext with at least {taps} columns, got {ext.dtype} "
                         f"{tuple(ext.shape)} and state {state.dtype}")
    if e4.stride(3) != 1 or e4.stride(2) != taps + T or s4.stride(3) != 1 or s4.stride(2) != taps:
        raise ValueError(f"{what}: each row's channels and taps must be contiguous in ext and state")
    if accepted.shape != (B,) or accepted.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"accepted: expected {B} integers, got {accepted.dtype} {tuple(accepted.shape)}")
    status = _lib.load().gdn_conv_state_commit(e4.data_ptr(), s4.data_ptr(), accepted.to(torch.int64).contiguous().data_ptr(),
                                               L, B, C, taps, T, e4.stride(0), e4.stride(1), s4.stride(0), s4.stride(1),
                                               _stream())
    _lib.check(status, what)
