"""Drop-in for the reference's ``model/fla_inplace.py`` (same two functions, same errors).

``gated_delta_rule_step_inplace`` (``model/fla_inplace.py:17-26``) runs the decode step
with the state read and written in place; ``gated_delta_rule_advance_inplace``
(``:63-74``) advances each row by its own number of tokens without outputs.
"""

from __future__ import annotations

import torch

from .gated_delta import (HEAD_DIM, _check_qkv, _check_state_inplace, _gates, _recurrent, _require_cuda,
                          gated_delta_rule_advance_inplace)

__all__ = ["gated_delta_rule_step_inplace", "gated_delta_rule_advance_inplace"]


def gated_delta_rule_step_inplace(q, k, v, g, beta, state) -> torch.Tensor:
    what = "gated_delta_rule_step_inplace"
    _require_cuda(what, q, k, v, g, beta, state)
    B, T, H, HV = _check_qkv(what, q, k, v)
    _check_state_inplace(what, state, B, HV)
    g, beta = _gates(what, g, beta, B, T, HV)
    o = torch.empty(B, T, HV, HEAD_DIM, dtype=q.dtype, device=q.device)
    _recurrent(what, q, k, v, g, beta, state_in=state, state_out=state, o=o)
    return o
