"""Output-gated RMSNorm with the reference's module interface (CUDA only).

Replaces ``GatedRMSNorm`` (``model/model.py:144-161``): ``forward(x, z)`` returns
``bf16(bf16(w * bf16(x * rsqrt(mean(x^2) + eps))) * silu(z))`` per row of 128.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib
from .gated_delta import _require_cuda, _stream


def gated_rms_norm(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    what = "gated_rms_norm"
    _require_cuda(what, x, z, weight)
    D = x.shape[-1]
    if z.shape != x.shape:
        raise ValueError(f"z: expected shape {tuple(x.shape)}, got {tuple(z.shape)}")
    if x.dtype != torch.bfloat16 or z.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or weight.shape != (D,):
        raise ValueError(f"x, z, weight: expected bfloat16 with weight of shape {(D,)}, got {x.dtype}, {z.dtype}, "
                         f"{weight.dtype} {tuple(weight.shape)}")
    x, z, w = x.contiguous(), z.contiguous(), weight.contiguous()
    if w.data_ptr() % 16:  # the kernel reads the weight with 16-byte loads
        w = w.clone()
    y = torch.empty_like(x)
    rows = x.numel() // D if D else 0
    status = _lib.load().gdn_gated_rmsnorm(x.data_ptr(), z.data_ptr(), w.data_ptr(), y.data_ptr(), rows, D, float(eps),
                                           _stream())
    _lib.check(status, what)
    return y


class GatedRMSNorm(nn.Module):
    """Drop-in for ``model.model.GatedRMSNorm`` (same parameter name and init)."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor, z: torch.Tensor) -> torch.Tensor:
        return gated_rms_norm(x, z, self.weight, self.eps)

    def extra_repr(self) -> str:
        return f"{tuple(self.weight.shape)}, eps={self.eps}"
