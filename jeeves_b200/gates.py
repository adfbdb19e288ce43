"""Delta-rule gates from the layer's raw projections (CUDA only).

Replaces ``delta_gates`` (``model/model.py:314-321``) and its CUDA kernel
(``model/triton_kernels.py:76-114``): ``beta = sigmoid(b)`` in bf16 and
``g = log_decay_rate * softplus(a + dt_bias)`` in fp32, zeroed on rows whose ``valid`` is
False. Rounds as PyTorch's CUDA eager ops (expf, log1pf, IEEE division, subnormals kept).

``gated_delta_rule_chunk_gates`` and ``gated_delta_rule_step_gates`` take the raw projections
instead of ``g`` and ``beta`` and compute the gates inside the prefill / recurrent kernels (the
engine's ``delta_gates`` followed by ``delta_extend`` / ``delta_outputs``,
``inference/engine.py:378-379``, ``:429-430``), with the same bits as the two calls.
"""

from __future__ import annotations

import torch

from . import _lib
from .gated_delta import (HEAD_DIM, _check_qkv, _chunk_prefill, _cu_seqlens_arg, _ptr, _recurrent, _require_cuda,
                          _state_arg, _stream)


def _gate_inputs(what, b, a, dt_bias, log_decay_rate, valid, shape=None):
    """Checked ``(b2, a2, dt, rate, valid_rows)``: b and a as [rows, HV] with unit inner stride."""
    _require_cuda(what, b, a, dt_bias, log_decay_rate, valid)
    *lead, HV = b.shape
    if shape is not None and tuple(b.shape) != tuple(shape):
        raise ValueError(f"b: expected shape {tuple(shape)}, got {tuple(b.shape)}")
    if b.dtype != torch.bfloat16 or a.dtype != torch.bfloat16:
        raise ValueError(f"b, a: expected bfloat16, got {b.dtype}, {a.dtype}")
    if a.shape != b.shape:
        raise ValueError(f"a: expected shape {tuple(b.shape)}, got {tuple(a.shape)}")
    if valid is not None and (valid.shape != tuple(lead) or valid.dtype != torch.bool):
        raise ValueError(f"valid: expected a bool tensor of shape {tuple(lead)}, got {valid.dtype} {tuple(valid.shape)}")
    if dt_bias.shape != (HV,) or dt_bias.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"dt_bias: expected float32 or bfloat16 of shape {(HV,)}, got {dt_bias.dtype} "
                         f"{tuple(dt_bias.shape)}")
    if log_decay_rate.numel() != HV:
        raise ValueError(f"log_decay_rate: expected {HV} values, got {tuple(log_decay_rate.shape)}")
    b2, a2 = b.reshape(-1, HV), a.reshape(-1, HV)
    if b2.stride(-1) != 1 or a2.stride(-1) != 1:
        b2, a2 = b2.contiguous(), a2.contiguous()
    rows = b2.shape[0]
    valid_rows = None if valid is None else valid.reshape(rows).contiguous().view(torch.uint8)
    return b2, a2, dt_bias.contiguous(), log_decay_rate.float().contiguous(), valid_rows


def _gate_struct(b2, a2, dt, rate, valid_rows):
    HV = b2.shape[1]
    return _lib.GateInputs(b2.data_ptr(), b2.stride(0) if b2.shape[0] else HV, a2.data_ptr(),
                           a2.stride(0) if a2.shape[0] else HV, dt.data_ptr(),
                           _lib.F32 if dt.dtype == torch.float32 else _lib.BF16, rate.data_ptr(), _ptr(valid_rows))


def delta_gates(b: torch.Tensor, a: torch.Tensor, dt_bias: torch.Tensor, log_decay_rate: torch.Tensor,
                valid: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    what = "delta_gates"
    b2, a2, dt, rate, valid_rows = _gate_inputs(what, b, a, dt_bias, log_decay_rate, valid)
    *lead, HV = b.shape
    rows = b2.shape[0]
    beta = torch.empty(*lead, HV, dtype=torch.bfloat16, device=b.device)
    g = torch.empty(*lead, HV, dtype=torch.float32, device=b.device)
    status = _lib.load().gdn_delta_gates(
        b2.data_ptr(), b2.stride(0) if rows else HV, a2.data_ptr(), a2.stride(0) if rows else HV, dt.data_ptr(),
        _lib.F32 if dt.dtype == torch.float32 else _lib.BF16, rate.data_ptr(), _ptr(valid_rows), beta.data_ptr(),
        g.data_ptr(), rows, HV, _stream())
    _lib.check(status, what)
    return beta, g


def gated_delta_rule_chunk_gates(q, k, v, b, a, dt_bias, log_decay_rate, valid=None, initial_state=None,
                                 output_final_state=False, scale=None, cu_seqlens=None):
    """``gated_delta_rule_chunk(q, k, v, g, beta, ...)`` with ``beta, g = delta_gates(b, a, dt_bias,
    log_decay_rate, valid)`` computed inside the prefill (bf16) or recurrent (fp32) kernel;
    returns ``(o, final_state or None)``. b, a: ``[B, T, HV]`` bf16; valid: ``[B, T]`` bool."""
    what = "gated_delta_rule_chunk_gates"
    _require_cuda(what, q, k, v, initial_state)
    B, T, H, HV = _check_qkv(what, q, k, v)
    gate_args = _gate_inputs(what, b, a, dt_bias, log_decay_rate, valid, shape=(B, T, HV))
    gates = _gate_struct(*gate_args)  # gate_args keeps the tensors it points at alive until the launch
    cu, rows = _cu_seqlens_arg(what, cu_seqlens, B, T)
    h0 = _state_arg(what, initial_state, rows, HV)
    o = torch.empty(B, T, HV, HEAD_DIM, dtype=q.dtype, device=q.device)
    final = torch.empty(rows, HV, HEAD_DIM, HEAD_DIM, dtype=torch.float32, device=q.device) if output_final_state else None
    if q.dtype == torch.float32:
        _recurrent(what, q, k, v, None, None, state_in=h0, state_out=final, o=o, cu_seqlens=cu, rows=rows, scale=scale,
                   gates=gates)
    else:
        _chunk_prefill(what, q, k, v, None, None, h0, final, o, cu, rows, scale, gates=gates)
    return o, final


def gated_delta_rule_step_gates(q, k, v, b, a, dt_bias, log_decay_rate, valid=None, initial_state=None,
                                output_final_state=True, scale=None, cu_seqlens=None):
    """``gated_delta_rule_step(q, k, v, g, beta, ...)`` with the gates computed in the recurrent
    kernel from the raw projections; returns ``(o, final_state or None)``."""
    what = "gated_delta_rule_step_gates"
    _require_cuda(what, q, k, v, initial_state)
    B, T, H, HV = _check_qkv(what, q, k, v)
    gate_args = _gate_inputs(what, b, a, dt_bias, log_decay_rate, valid, shape=(B, T, HV))
    gates = _gate_struct(*gate_args)  # gate_args keeps the tensors it points at alive until the launch
    cu, rows = _cu_seqlens_arg(what, cu_seqlens, B, T)
    h0 = _state_arg(what, initial_state, rows, HV)
    o = torch.empty(B, T, HV, HEAD_DIM, dtype=q.dtype, device=q.device)
    final = torch.empty(rows, HV, HEAD_DIM, HEAD_DIM, dtype=torch.float32, device=q.device) if output_final_state else None
    _recurrent(what, q, k, v, None, None, state_in=h0, state_out=final, o=o, cu_seqlens=cu, rows=rows, scale=scale,
               gates=gates)
    return o, final
