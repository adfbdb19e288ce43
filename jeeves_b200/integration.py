"""Route the reference's kernel dispatch to this library.

The reference picks its GPU kernels in ``model/model.py:64-94``: ``_on(name, x)`` is true
when kernel family ``name`` is available and enabled and ``x`` is on CUDA, and the
dispatchers then call fla's functions through module attributes (``_fla_chunk_gdr``,
``_fla_recurrent_gdr``, ``fla_inplace``, ``_fla_causal_conv1d``,
``_fla_causal_conv1d_update``, ``_fla_rms_norm_gated``). ``install`` replaces those
attributes with adapters that have fla's signatures, marks the families available, and
wraps the dispatchers whose CUDA branch needs Triton (``conv_step``,
``gated_delta_rule_advance_inplace``, ``delta_gates``). CPU tensors still take the reference's eager path,
so ``set_kernels(gdn=False)`` and friends keep working.
"""

from __future__ import annotations

from types import ModuleType

import torch

from . import fla_inplace as _fla_inplace
from .conv import causal_conv1d as _conv1d
from .conv import causal_conv1d_step as _conv1d_step
from .conv import conv_step as _conv_step
from .gated_delta import gated_delta_rule_chunk, gated_delta_rule_step
from .attention import decode_attention as _decode_attention
from .attention import decode_attention_supported as _attention_supported
from .attention import rotary as _rotary
from .attention import rotate_into_cache as _rotate_into_cache
from .gates import delta_gates as _delta_gates
from .norm import gated_rms_norm

KERNEL_FAMILIES = ("gdn", "causal_conv1d", "rms_norm_gated")
IMPORTED_NAMES = ("gated_delta_rule_chunk", "gated_delta_rule_step", "gated_delta_rule_advance_inplace", "conv_step",
                  "eager_conv_step", "causal_conv1d", "causal_conv1d_step", "delta_gates", "decode_attention",
                  "rotate_into_cache", "apply_rotary")


def fla_chunk_gated_delta_rule(q, k, v, g=None, beta=None, scale=None, initial_state=None, output_final_state=False,
                               use_qk_l2norm_in_kernel=False, cu_seqlens=None, **unused):
    """fla's ``chunk_gated_delta_rule`` signature (called at ``model/model.py:291``)."""
    _need_l2norm(use_qk_l2norm_in_kernel)
    return gated_delta_rule_chunk(q, k, v, g, beta, initial_state=initial_state, output_final_state=output_final_state,
                                  scale=scale, cu_seqlens=cu_seqlens)


def fla_fused_recurrent_gated_delta_rule(q, k, v, g=None, beta=None, scale=None, initial_state=None,
                                         output_final_state=False, use_qk_l2norm_in_kernel=False, cu_seqlens=None,
                                         **unused):
    """fla's ``fused_recurrent_gated_delta_rule`` signature (called at ``model/model.py:299``)."""
    _need_l2norm(use_qk_l2norm_in_kernel)
    return gated_delta_rule_step(q, k, v, g, beta, initial_state=initial_state, output_final_state=output_final_state,
                                 scale=scale, cu_seqlens=cu_seqlens)


def fla_causal_conv1d(x, weight, bias=None, activation="silu", cu_seqlens=None, **unused):
    """fla's ``causal_conv1d`` as called at ``model/model.py:201``; returns ``(y, None)``."""
    if bias is not None or activation not in ("silu", "swish"):
        raise ValueError("only bias=None with a SiLU activation is implemented")
    return _conv1d(x, weight, cu_seqlens=cu_seqlens), None


def fla_causal_conv1d_update(x, cache, residual=None, weight=None, bias=None, activation="silu", **unused):
    """fla's ``causal_conv1d_update`` as called at ``model/model.py:209``; returns ``(y, cache)``."""
    if residual is not None or bias is not None or activation not in ("silu", "swish"):
        raise ValueError("only residual=None, bias=None with a SiLU activation is implemented")
    return _conv1d_step(x, cache, weight), cache


def fla_rms_norm_gated(x, g, weight, bias=None, activation="swish", eps=1e-6, **unused):
    """fla's ``rms_norm_gated`` as called at ``model/model.py:152`` (gate ``g`` with a swish)."""
    if bias is not None or activation not in ("swish", "silu"):
        raise ValueError("only bias=None with a swish gate is implemented")
    return gated_rms_norm(x, g, weight, eps)


def _need_l2norm(flag: bool) -> None:
    if not flag:
        raise ValueError("the kernels L2-normalise q and k themselves; call with use_qk_l2norm_in_kernel=True "
                         "(as model/model.py:292 and :300 do)")


class Installed:
    """Handle returned by ``install``; ``uninstall()`` restores every replaced attribute."""

    def __init__(self):
        self._saved: list[tuple[object, str, object, bool]] = []

    def set(self, obj, name, value):
        had = hasattr(obj, name)
        self._saved.append((obj, name, getattr(obj, name, None), had))
        setattr(obj, name, value)

    def uninstall(self) -> None:
        for obj, name, old, had in reversed(self._saved):
            if had:
                setattr(obj, name, old)
            else:
                delattr(obj, name)
        self._saved.clear()


def install(model_module: ModuleType, *importers: ModuleType) -> Installed:
    """Route ``model_module`` (the reference's ``model.model``) to this library.

    ``importers`` are modules that imported dispatchers by name (``inference.engine``
    imports ``conv_step``, ``eager_conv_step``, ``gated_delta_rule_chunk`` ... at
    ``inference/engine.py:16-18``); their copies are pointed at the wrapped dispatchers.
    """
    m = model_module
    handle = Installed()
    handle.set(m, "_fla_chunk_gdr", fla_chunk_gated_delta_rule)
    handle.set(m, "_fla_recurrent_gdr", fla_fused_recurrent_gated_delta_rule)
    handle.set(m, "fla_inplace", _fla_inplace)
    handle.set(m, "_fla_causal_conv1d", fla_causal_conv1d)
    handle.set(m, "_fla_causal_conv1d_update", fla_causal_conv1d_update)
    handle.set(m, "_fla_rms_norm_gated", fla_rms_norm_gated)
    available = dict(m._AVAILABLE)
    kernels = dict(m.KERNELS)
    for family in KERNEL_FAMILIES:
        available[family] = True
        kernels[family] = bool(getattr(m, "_ENABLED_BY_ENV", True))
    handle.set(m, "_AVAILABLE", available)
    handle.set(m, "KERNELS", kernels)

    eager_conv = m.eager_conv_step
    conv_dispatch = m.conv_step
    advance_dispatch = m.gated_delta_rule_advance_inplace

    def conv_step(state, qkv, weight, key_dim, value_dim, head_k_dim, head_v_dim, ext_out=None):
        if m._on("causal_conv1d", qkv):
            return _conv_step(state, qkv, weight, key_dim, value_dim, head_k_dim, head_v_dim, ext_out)
        return conv_dispatch(state, qkv, weight, key_dim, value_dim, head_k_dim, head_v_dim, ext_out)

    def eager_conv_step(state, qkv, weight, key_dim, value_dim, head_k_dim, head_v_dim, ext_out=None):
        if m._on("causal_conv1d", qkv):
            return _conv_step(state, qkv, weight, key_dim, value_dim, head_k_dim, head_v_dim, ext_out)
        return eager_conv(state, qkv, weight, key_dim, value_dim, head_k_dim, head_v_dim, ext_out)

    def gated_delta_rule_advance_inplace(k, v, g, beta, state, steps):
        if m._on("gdn", k):
            return _fla_inplace.gated_delta_rule_advance_inplace(k, v, g, beta, state, steps)
        return advance_dispatch(k, v, g, beta, state, steps)

    handle.set(m, "conv_step", conv_step)
    handle.set(m, "eager_conv_step", eager_conv_step)
    handle.set(m, "gated_delta_rule_advance_inplace", gated_delta_rule_advance_inplace)
    if hasattr(m, "delta_gates"):
        gates_dispatch = m.delta_gates

        def delta_gates(b, a, dt_bias, log_decay_rate, valid=None):
            if m._on("gdn", b):
                return _delta_gates(b, a, dt_bias, log_decay_rate, valid)
            return gates_dispatch(b, a, dt_bias, log_decay_rate, valid)

        handle.set(m, "delta_gates", delta_gates)
    # The drafter's attention-side dispatchers (model/model.py:182, :342, :354), under the "gdn"
    # family: the supported CUDA cases run here, everything else keeps the reference's path.
    if hasattr(m, "decode_attention"):
        attention_dispatch = m.decode_attention

        def decode_attention(q, k_cache, v_cache, mask, scale):
            if m._on("gdn", q) and _attention_supported(q, k_cache, v_cache, mask):
                return _decode_attention(q, k_cache, v_cache, mask, scale)
            return attention_dispatch(q, k_cache, v_cache, mask, scale)

        handle.set(m, "decode_attention", decode_attention)
    if hasattr(m, "rotate_into_cache"):
        rotate_dispatch = m.rotate_into_cache

        def rotate_into_cache(k, v, qm, km, vm, cos_c, sin_c, cos_m, sin_m, k_cache, v_cache, rows, positions,
                              tail_start):
            if m._on("gdn", k) and k.dtype == k_cache.dtype == torch.bfloat16:
                return _rotate_into_cache(k, v, qm, km, vm, cos_c, sin_c, cos_m, sin_m, k_cache, v_cache, rows,
                                          positions, tail_start)
            return rotate_dispatch(k, v, qm, km, vm, cos_c, sin_c, cos_m, sin_m, k_cache, v_cache, rows, positions,
                                   tail_start)

        handle.set(m, "rotate_into_cache", rotate_into_cache)
    if hasattr(m, "apply_rotary"):
        rotary_dispatch = m.apply_rotary

        def apply_rotary(x, cos, sin):
            if x.dim() == 4 and cos.dim() == 3 and x.dtype == torch.bfloat16 and m._on("gdn", x):
                return _rotary(x, cos, sin)
            return rotary_dispatch(x, cos, sin)

        handle.set(m, "apply_rotary", apply_rotary)
    # Keep the reference's norm module class but let its fla branch reach our kernel: done
    # through _fla_rms_norm_gated above, since GatedRMSNorm.forward calls it under _on.
    for mod in importers:
        for name in IMPORTED_NAMES:
            if hasattr(mod, name) and hasattr(m, name):
                handle.set(mod, name, getattr(m, name))
    return handle
