"""Delta-rule gates from the layer's raw projections (CUDA only).

Replaces ``delta_gates`` (``model/model.py:314-321``) and its CUDA kernel
(``model/triton_kernels.py:76-114``): ``beta = sigmoid(b)`` in bf16 and
``g = log_decay_rate * softplus(a + dt_bias)`` in fp32, zeroed on rows whose ``valid`` is
False. Rounds as PyTorch's CUDA eager ops (expf, log1pf, IEEE division, subnormals kept).
"""

from __future__ import annotations

import torch

from . import _lib
from .gated_delta import _ptr, _require_cuda, _stream


def delta_gates(b: torch.Tensor, a: torch.Tensor, dt_bias: torch.Tensor, log_decay_rate: torch.Tensor,
                valid: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    what = "delta_gates"
    _require_cuda(what, b, a, dt_bias, log_decay_rate, valid)
    *lead, HV = b.shape
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
    dt = dt_bias.contiguous()
    rate = log_decay_rate.float().contiguous()
    beta = torch.empty(*lead, HV, dtype=torch.bfloat16, device=b.device)
    g = torch.empty(*lead, HV, dtype=torch.float32, device=b.device)
    valid_rows = None if valid is None else valid.reshape(rows).contiguous().view(torch.uint8)
    status = _lib.load().gdn_delta_gates(
        b2.data_ptr(), b2.stride(0) if rows else HV, a2.data_ptr(), a2.stride(0) if rows else HV, dt.data_ptr(),
        _lib.F32 if dt.dtype == torch.float32 else _lib.BF16, rate.data_ptr(), _ptr(valid_rows), beta.data_ptr(),
        g.data_ptr(), rows, HV, _stream())
    _lib.check(status, what)
    return beta, g
