"""Gated delta rule operators with the reference's call signatures.

Each function mirrors one dispatcher of ``model/model.py`` (PostHog/jeeves) and runs on
the CUDA kernels of ``libgdn_b200.so``. Inputs must be CUDA tensors: there is no CPU or
eager fallback, and a missing library raises. Shapes: q, k ``[B, T, H, 128]`` (H key
heads; H may be smaller than HV, value head hv then reads key head hv // (HV // H), the
repeat-interleave mapping of ``model/model.py:487-490``), v ``[B, T, HV, 128]``, g
``[B, T, HV]`` (log decay), beta ``[B, T, HV]``, states ``[B, HV, 128, 128]`` fp32.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

HEAD_DIM = 128
_DTYPES = {torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(what: str, *tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError(f"{what}: expected CUDA tensors, got a tensor on {t.device}")


def _heads_last_contiguous(x: torch.Tensor) -> torch.Tensor:
    return x if x.stride(-1) == 1 else x.contiguous()


def _check_qkv(what: str, q, k, v):
    if k.dim() != 4 or v.dim() != 4:
        raise ValueError(f"{what}: expected k [B, T, H, D] and v [B, T, HV, D], got {tuple(k.shape)} and {tuple(v.shape)}")
    B, T, H, Dk = k.shape
    HV, Dv = v.shape[2], v.shape[3]
    if v.shape[:2] != (B, T) or (q is not None and q.shape != k.shape):
        raise ValueError(f"{what}: q {None if q is None else tuple(q.shape)}, k {tuple(k.shape)} and v {tuple(v.shape)} "
                         f"do not agree")
    if HV % H:
        raise ValueError(f"{what}: {HV} value heads are not a multiple of {H} key heads")
    if Dk != HEAD_DIM or Dv != HEAD_DIM:
        raise ValueError(f"{what}: head dims must be {HEAD_DIM}, got {Dk} and {Dv}")
    dtypes = {t.dtype for t in (q, k, v) if t is not None}
    if len(dtypes) != 1 or next(iter(dtypes)) not in _DTYPES:
        raise ValueError(f"{what}: q, k, v must all be bfloat16 or all float32, got {sorted(map(str, dtypes))}")
    return B, T, H, HV


def _gates(what: str, g, beta, B, T, HV):
    if g.shape != (B, T, HV) or beta.shape != (B, T, HV):
        raise ValueError(f"{what}: g and beta must be {(B, T, HV)}, got {tuple(g.shape)} and {tuple(beta.shape)}")
    g = g.to(torch.float32).contiguous()
    if beta.dtype not in _DTYPES:
        beta = beta.to(torch.float32)
    return g, beta.contiguous()


def _state_arg(what: str, state, rows, HV, *, name="initial_state"):
    if state is None:
        return None
    if state.shape != (rows, HV, HEAD_DIM, HEAD_DIM):
        raise ValueError(f"{what}: {name} must be {(rows, HV, HEAD_DIM, HEAD_DIM)}, got {tuple(state.shape)}")
    return state.to(torch.float32).contiguous()


def _recurrent(what, q, k, v, g, beta, *, state_in=None, state_out=None, snapshots=None, o=None, steps=None,
               cu_seqlens=None, rows=None, scale=None, gates=None):
    """One gdn_recurrent call, or gdn_recurrent_gates when ``gates`` (a ``_lib.GateInputs``) is given."""
    B, T = k.shape[:2]
    H, HV = k.shape[2], v.shape[2]
    q = None if q is None else _heads_last_contiguous(q)
    k, v = _heads_last_contiguous(k), _heads_last_contiguous(v)
    if scale is None:
        scale = HEAD_DIM ** -0.5
    qs = (0, 0, 0) if q is None else (q.stride(0), q.stride(1), q.stride(2))
    tail = (_ptr(state_in), _ptr(state_out), _ptr(snapshots), _ptr(o), _ptr(steps), _ptr(cu_seqlens),
            B if rows is None else rows, T, H, HV, HEAD_DIM, HEAD_DIM,
            *qs, k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1), v.stride(2), float(scale), _stream())
    lib = _lib.load()
    if gates is None:
        status = lib.gdn_recurrent(_ptr(q), _ptr(k), _ptr(v), _DTYPES[k.dtype], _ptr(g), _ptr(beta),
                                   _DTYPES[beta.dtype], *tail)
    else:
        status = lib.gdn_recurrent_gates(_ptr(q), _ptr(k), _ptr(v), _DTYPES[k.dtype], gates, *tail)
    _lib.check(status, what)


def _cu_seqlens_arg(what, cu_seqlens, B, T):
    if cu_seqlens is None:
        return None, B
    if B != 1:
        raise ValueError(f"{what}: with cu_seqlens the inputs are packed into a batch of 1, got batch {B}")
    if cu_seqlens.dim() != 1 or cu_seqlens.numel() < 1 or cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"{what}: cu_seqlens must be a 1-D int32/int64 tensor, got {cu_seqlens.dtype} {tuple(cu_seqlens.shape)}")
    if not cu_seqlens.is_cuda:
        # A host copy can be checked without a device sync: offsets must rise from 0 to T.
        steps = cu_seqlens[1:] - cu_seqlens[:-1]
        if int(cu_seqlens[0]) != 0 or bool((steps < 0).any()) or int(cu_seqlens[-1]) > T:
            raise ValueError(f"{what}: cu_seqlens must rise from 0 to at most {T}, got {cu_seqlens.tolist()}")
        return cu_seqlens.to(dtype=torch.int32).pin_memory().to("cuda", non_blocking=True), cu_seqlens.numel() - 1
    return cu_seqlens.to(dtype=torch.int32).contiguous(), cu_seqlens.numel() - 1


def gated_delta_rule_step(q, k, v, g, beta, initial_state=None, output_final_state=True, scale=None, cu_seqlens=None):
    """Recurrent gated delta rule over T tokens; returns ``(o, final_state or None)``.

    Replaces ``gated_delta_rule_step`` (``model/model.py:297-302``): the verify outputs of
    ``inference/engine.py:250-252`` and the decode step of the non-static cache path.
    """
    what = "gated_delta_rule_step"
    _require_cuda(what, q, k, v, g, beta, initial_state)
    B, T, H, HV = _check_qkv(what, q, k, v)
    g, beta = _gates(what, g, beta, B, T, HV)
    cu, rows = _cu_seqlens_arg(what, cu_seqlens, B, T)
    h0 = _state_arg(what, initial_state, rows, HV)
    o = torch.empty(B, T, HV, HEAD_DIM, dtype=q.dtype, device=q.device)
    final = torch.empty(rows, HV, HEAD_DIM, HEAD_DIM, dtype=torch.float32, device=q.device) if output_final_state else None
    _recurrent(what, q, k, v, g, beta, state_in=h0, state_out=final, o=o, cu_seqlens=cu, rows=rows, scale=scale)
    return o, final


def gated_delta_rule_chunk(q, k, v, g, beta, initial_state=None, output_final_state=False, scale=None, cu_seqlens=None):
    """Chunked prefill; returns ``(o, final_state or None)``.

    Replaces ``gated_delta_rule_chunk`` (``model/model.py:289-294``). ``cu_seqlens`` (int32 or
    int64, ``[N + 1]``) packs N sequences into a batch of 1, as fla 0.5.x's
    ``chunk_gated_delta_rule(..., cu_seqlens=...)``; ``initial_state`` and the final state
    then have N rows. bf16 inputs run the tcgen05 chunk kernel; fp32 inputs (the fp32 mode
    of the parity bound) run the fp32 recurrent kernel on CUDA cores.
    """
    what = "gated_delta_rule_chunk"
    _require_cuda(what, q, k, v, g, beta, initial_state)
    B, T, H, HV = _check_qkv(what, q, k, v)
    g, beta = _gates(what, g, beta, B, T, HV)
    cu, rows = _cu_seqlens_arg(what, cu_seqlens, B, T)
    h0 = _state_arg(what, initial_state, rows, HV)
    o = torch.empty(B, T, HV, HEAD_DIM, dtype=q.dtype, device=q.device)
    final = torch.empty(rows, HV, HEAD_DIM, HEAD_DIM, dtype=torch.float32, device=q.device) if output_final_state else None
    if q.dtype == torch.float32:
        _recurrent(what, q, k, v, g, beta, state_in=h0, state_out=final, o=o, cu_seqlens=cu, rows=rows, scale=scale)
        return o, final
    _chunk_prefill(what, q, k, v, g, beta, h0, final, o, cu, rows, scale)
    return o, final


def _chunk_prefill(what, q, k, v, g, beta, h0, final, o, cu, rows, scale, norm=None, gates=None):
    """One gdn_chunk_prefill call (gdn_chunk_prefill_gated_norm when ``norm`` = (z, weight, eps,
    out); gdn_chunk_prefill_gates when ``gates`` is a ``_lib.GateInputs``), with the workspace
    taken from PyTorch's caching allocator."""
    B, T, H = k.shape[:3]
    HV = v.shape[2]
    if T == 0:
        if final is not None:
            final.copy_(h0) if h0 is not None else final.zero_()
        return
    q, k, v = (_heads_last_contiguous(t) for t in (q, k, v))
    lib = _lib.load()
    ws_bytes = lib.gdn_chunk_prefill_workspace_size(rows, T, HV, int(cu is not None))
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    tail = (_ptr(h0), _ptr(final), o.data_ptr(), _ptr(cu), rows, T, H, HV, HEAD_DIM, HEAD_DIM,
            q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1),
            v.stride(2), float(HEAD_DIM ** -0.5 if scale is None else scale))
    if gates is not None:
        status = lib.gdn_chunk_prefill_gates(q.data_ptr(), k.data_ptr(), v.data_ptr(), gates, *tail,
                                             workspace.data_ptr(), ws_bytes, _stream())
        _lib.check(status, what)
        return
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), _DTYPES[beta.dtype], *tail)
    if norm is None:
        status = lib.gdn_chunk_prefill(*args, workspace.data_ptr(), ws_bytes, _stream())
    else:
        z, w, eps, out = norm
        status = lib.gdn_chunk_prefill_gated_norm(*args, z.data_ptr(), w.data_ptr(), float(eps), out.data_ptr(),
                                                  workspace.data_ptr(), ws_bytes, _stream())
    _lib.check(status, what)


def gated_delta_rule_chunk_gated_norm(q, k, v, g, beta, z, norm_weight, eps=1e-6, initial_state=None,
                                      output_final_state=False, scale=None, cu_seqlens=None, out=None):
    """Chunked prefill and the output-gated RMSNorm of its output; returns ``(y, final_state or None)``.

    Equals ``gated_rms_norm(gated_delta_rule_chunk(...)[0], z, norm_weight, eps)`` bit for bit:
    the prefill branch of ``GatedDeltaNet.forward`` from ``gated_delta_rule_chunk`` to
    ``self.norm`` (``model/model.py:505-506``, ``:516``). bf16 only. ``z`` holds
    ``B * T * HV * 128`` bf16 values in the output's order (``[B, T, HV, 128]``); ``out``
    (``[B, T, HV, 128]`` bf16) receives ``y`` and is allocated when not given. The un-normed
    output is not kept.
    """
    what = "gated_delta_rule_chunk_gated_norm"
    _require_cuda(what, q, k, v, g, beta, z, norm_weight, initial_state, out)
    B, T, H, HV = _check_qkv(what, q, k, v)
    if q.dtype != torch.bfloat16:
        raise ValueError(f"{what}: expected bfloat16 q, k, v, got {q.dtype}")
    shape = (B, T, HV, HEAD_DIM)
    if z.dtype != torch.bfloat16 or z.numel() != B * T * HV * HEAD_DIM:
        raise ValueError(f"z: expected {B * T * HV * HEAD_DIM} bfloat16 values {shape}, got {z.dtype} {tuple(z.shape)}")
    if norm_weight.dtype != torch.bfloat16 or norm_weight.shape != (HEAD_DIM,):
        raise ValueError(f"norm_weight: expected bfloat16 of shape {(HEAD_DIM,)}, got {norm_weight.dtype} "
                         f"{tuple(norm_weight.shape)}")
    if out is not None and (out.shape != shape or out.dtype != torch.bfloat16 or not out.is_contiguous()):
        raise ValueError(f"out: expected a contiguous bfloat16 tensor of shape {shape}, got {out.dtype} "
                         f"{tuple(out.shape)}")
    g, beta = _gates(what, g, beta, B, T, HV)
    cu, rows = _cu_seqlens_arg(what, cu_seqlens, B, T)
    h0 = _state_arg(what, initial_state, rows, HV)
    z = z.reshape(shape).contiguous()
    w = norm_weight.contiguous()
    if w.data_ptr() % 16:  # read with 16-byte loads
        w = w.clone()
    if out is None:
        out = torch.empty(shape, dtype=torch.bfloat16, device=q.device)
    final = torch.empty(rows, HV, HEAD_DIM, HEAD_DIM, dtype=torch.float32, device=q.device) if output_final_state else None
    # the scan's output goes to `out` and is normalised there in place
    _chunk_prefill(what, q, k, v, g, beta, h0, final, out, cu, rows, scale, norm=(z, w, eps, out))
    return out, final


def _check_state_inplace(what, state, B, HV):
    if state.dtype != torch.float32 or not state.is_contiguous() or state.shape != (B, HV, HEAD_DIM, HEAD_DIM):
        raise ValueError(f"state: expected a contiguous float32 tensor of shape {(B, HV, HEAD_DIM, HEAD_DIM)}, "
                         f"got {state.dtype} {tuple(state.shape)}")


def gated_delta_rule_advance_inplace(k, v, g, beta, state, steps) -> None:
    """Advance ``state[b]`` by ``clamp(steps[b], 0, T)`` tokens in place, without outputs.

    Replaces ``gated_delta_rule_advance_inplace`` (``model/model.py:305-311``,
    ``model/fla_inplace.py:63-74``); same errors (ValueError) for a bad state or steps.
    """
    what = "gated_delta_rule_advance_inplace"
    _require_cuda(what, k, v, g, beta, state, steps)
    B, T, H, HV = _check_qkv(what, None, k, v)
    _check_state_inplace(what, state, B, HV)
    if steps.shape != (B,) or steps.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"steps: expected {B} integers, got {steps.dtype} {tuple(steps.shape)}")
    g, beta = _gates(what, g, beta, B, T, HV)
    _recurrent(what, None, k, v, g, beta, state_in=state, state_out=state, steps=steps.to(torch.int64).contiguous())


def gated_delta_rule_verify(q, k, v, g, beta, state, snapshots=None, scale=None):
    """Score T drafted tokens; returns ``(o, snapshots)`` with ``snapshots[b, t]`` the state after token t.

    ``state`` is read, not written. After acceptance, ``gated_delta_rule_rollback`` makes
    ``snapshots[b, accepted[b] - 1]`` the live state (the rollback of
    ``inference/engine.py:471-472`` without recomputing the accepted tokens).
    """
    what = "gated_delta_rule_verify"
    _require_cuda(what, q, k, v, g, beta, state, snapshots)
    B, T, H, HV = _check_qkv(what, q, k, v)
    g, beta = _gates(what, g, beta, B, T, HV)
    h0 = _state_arg(what, state, B, HV, name="state")
    shape = (B, T, HV, HEAD_DIM, HEAD_DIM)
    if snapshots is None:
        snapshots = torch.empty(shape, dtype=torch.float32, device=q.device)
    elif snapshots.shape != shape or snapshots.dtype != torch.float32 or not snapshots.is_contiguous():
        raise ValueError(f"snapshots: expected a contiguous float32 tensor of shape {shape}, got {snapshots.dtype} "
                         f"{tuple(snapshots.shape)}")
    o = torch.empty(B, T, HV, HEAD_DIM, dtype=q.dtype, device=q.device)
    _recurrent(what, q, k, v, g, beta, state_in=h0, snapshots=snapshots, o=o, scale=scale)
    return o, snapshots


def gated_delta_rule_verify_deltas(q, k, v, g, beta, state, deltas=None, scale=None):
    """Score T drafted tokens from ``state`` (read, not written) and keep each token's update vector;
    returns ``(o, deltas)`` with ``deltas [B, T, HV, 128]`` fp32 = beta_t (v_t - e^{g_t} S_{t-1}^T k_t).

    Replaces the engine's ``delta_outputs`` (``inference/engine.py:249-252``). With bf16 rows and
    T <= 8 the block runs on the tensor cores: one product of the state (as two bf16 parts, within
    2^-18 of fp32) with the 2T raw k and q rows, the rows' Gram products, and the token recurrence
    unrolled per column; ``o`` and ``deltas`` agree with the recurrent kernel to fp32 rounding.
    Otherwise the recurrent kernel runs and ``o`` is ``gated_delta_rule_step(...)[0]`` bit for bit.
    ``gated_delta_rule_delta_commit`` then makes the accepted tokens' state live without re-running
    their reductions."""
    what = "gated_delta_rule_verify_deltas"
    _require_cuda(what, q, k, v, g, beta, state, deltas)
    B, T, H, HV = _check_qkv(what, q, k, v)
    g, beta = _gates(what, g, beta, B, T, HV)
    h0 = _state_arg(what, state, B, HV, name="state")
    shape = (B, T, HV, HEAD_DIM)
    if deltas is None:
        deltas = torch.empty(shape, dtype=torch.float32, device=q.device)
    elif deltas.shape != shape or deltas.dtype != torch.float32 or not deltas.is_contiguous():
        raise ValueError(f"deltas: expected a contiguous float32 tensor of shape {shape}, got {deltas.dtype} "
                         f"{tuple(deltas.shape)}")
    q, k, v = _heads_last_contiguous(q), _heads_last_contiguous(k), _heads_last_contiguous(v)
    o = torch.empty(B, T, HV, HEAD_DIM, dtype=q.dtype, device=q.device)
    status = _lib.load().gdn_recurrent_deltas(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), _DTYPES[k.dtype], g.data_ptr(), beta.data_ptr(), _DTYPES[beta.dtype],
        _ptr(h0), o.data_ptr(), deltas.data_ptr(), B, T, H, HV, HEAD_DIM, HEAD_DIM,
        q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1),
        v.stride(2), float(HEAD_DIM ** -0.5 if scale is None else scale), _stream())
    _lib.check(status, what)
    return o, deltas


def gated_delta_rule_verify_deltas_gated_norm(q, k, v, g, beta, state, z, norm_weight, eps=1e-6, deltas=None,
                                              scale=None):
    """``gated_delta_rule_verify_deltas`` with the output-gated RMSNorm (``GatedRMSNorm.forward``,
    ``model/model.py:150-158``; the engine's ``self.norm`` after ``delta_outputs``,
    ``inference/engine.py:435``) fused into the tensor-core block's drain: returns
    ``(y, deltas)`` with ``y [B, T, HV, 128]`` bf16 equal to ``gated_rms_norm(o, z, norm_weight)`` of
    the unfused call bit for bit. Needs bf16 rows and 1 <= T <= 8."""
    what = "gated_delta_rule_verify_deltas_gated_norm"
    _require_cuda(what, q, k, v, g, beta, state, z, norm_weight, deltas)
    B, T, H, HV = _check_qkv(what, q, k, v)
    if q.dtype != torch.bfloat16 or not 1 <= T <= 8:
        raise ValueError(f"{what}: expected bfloat16 rows and 1 to 8 tokens, got {q.dtype}, {T}")
    g, beta = _gates(what, g, beta, B, T, HV)
    h0 = _state_arg(what, state, B, HV, name="state")
    if h0 is None:
        raise ValueError(f"{what}: a state is required")
    shape = (B, T, HV, HEAD_DIM)
    z = z.reshape(shape)
    if z.dtype != torch.bfloat16:
        raise ValueError(f"z: expected bfloat16, got {z.dtype}")
    z = z.contiguous()
    w = norm_weight.reshape(HEAD_DIM).to(torch.bfloat16).contiguous()
    if deltas is None:
        deltas = torch.empty(shape, dtype=torch.float32, device=q.device)
    elif deltas.shape != shape or deltas.dtype != torch.float32 or not deltas.is_contiguous():
        raise ValueError(f"deltas: expected a contiguous float32 tensor of shape {shape}, got {deltas.dtype} "
                         f"{tuple(deltas.shape)}")
    q, k, v = _heads_last_contiguous(q), _heads_last_contiguous(k), _heads_last_contiguous(v)
    y = torch.empty(shape, dtype=torch.bfloat16, device=q.device)
    status = _lib.load().gdn_recurrent_deltas_gated_norm(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), _DTYPES[beta.dtype], h0.data_ptr(),
        z.data_ptr(), w.data_ptr(), float(eps), y.data_ptr(), deltas.data_ptr(), B, T, H, HV, HEAD_DIM, HEAD_DIM,
        q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1),
        v.stride(2), float(HEAD_DIM ** -0.5 if scale is None else scale), _stream())
    _lib.check(status, what)
    return y, deltas


def gated_delta_rule_delta_commit(k, g, deltas, state, accepted) -> None:
    """Advance ``state[b]`` in place by ``clamp(accepted[b], 0, T)`` tokens from the update vectors of
    ``gated_delta_rule_verify_deltas`` (run on the same state, k and g), with one streaming pass over
    the state: the advance's own update arithmetic without its reductions (the engine's
    ``delta_commit``, ``inference/engine.py:254-258``). With update vectors from the recurrent kernel
    the state is ``gated_delta_rule_advance_inplace``'s bit for bit; from the tensor-core block, to
    fp32 rounding."""
    what = "gated_delta_rule_delta_commit"
    _require_cuda(what, k, g, deltas, state, accepted)
    if k.dim() != 4 or k.shape[-1] != HEAD_DIM:
        raise ValueError(f"k: expected [B, T, H, {HEAD_DIM}], got {tuple(k.shape)}")
    if deltas.dim() != 4 or deltas.dtype != torch.float32 or not deltas.is_contiguous():
        raise ValueError(f"deltas: expected a contiguous float32 [B, T, HV, {HEAD_DIM}] tensor")
    B, T, H = k.shape[:3]
    HV = deltas.shape[2]
    if deltas.shape != (B, T, HV, HEAD_DIM) or HV % H:
        raise ValueError(f"deltas: expected {(B, T, HV, HEAD_DIM)} with HV a multiple of {H}, got {tuple(deltas.shape)}")
    _check_state_inplace(what, state, B, HV)
    if g.shape != (B, T, HV) or g.dtype != torch.float32:
        raise ValueError(f"g: expected float32 {(B, T, HV)}, got {g.dtype} {tuple(g.shape)}")
    if accepted.shape != (B,) or accepted.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"accepted: expected {B} integers, got {accepted.dtype} {tuple(accepted.shape)}")
    k = _heads_last_contiguous(k)
    g = g.contiguous()
    status = _lib.load().gdn_delta_commit(state.data_ptr(), k.data_ptr(), _DTYPES[k.dtype], g.data_ptr(),
                                          deltas.data_ptr(), accepted.to(torch.int64).contiguous().data_ptr(), B, T,
                                          H, HV, HEAD_DIM, HEAD_DIM, k.stride(0), k.stride(1), k.stride(2), _stream())
    _lib.check(status, what)


def gated_delta_rule_delta_commit_layers(ks, gs, deltas, states, accepted) -> None:
    """``gated_delta_rule_delta_commit`` for every layer of a model in one launch: layer l's
    ``states[l]`` advances by ``clamp(accepted[b], 0, T)`` tokens from ``ks[l]``, ``gs[l]`` and
    ``deltas[l]`` (the engine's commit loop over its layers, ``inference/engine.py:471-472``). Every
    layer has the same shapes and k strides; each state ends as the one-layer commit leaves it, bit
    for bit."""
    what = "gated_delta_rule_delta_commit_layers"
    ks, gs, deltas, states = list(ks), list(gs), list(deltas), list(states)
    L = len(states)
    if not (len(ks) == len(gs) == len(deltas) == L):
        raise ValueError(f"{what}: expected as many k, g and deltas tensors as states, got {len(ks)}, {len(gs)}, "
                         f"{len(deltas)} and {L}")
    if L == 0:
        return
    _require_cuda(what, *ks, *gs, *deltas, *states, accepted)
    k0 = ks[0]
    if k0.dim() != 4 or k0.shape[-1] != HEAD_DIM:
        raise ValueError(f"k: expected [B, T, H, {HEAD_DIM}], got {tuple(k0.shape)}")
    B, T, H = k0.shape[:3]
    HV = deltas[0].shape[2] if deltas[0].dim() == 4 else -1
    if HV <= 0 or HV % H:
        raise ValueError(f"deltas: expected [B, T, HV, {HEAD_DIM}] with HV a multiple of {H}, got "
                         f"{tuple(deltas[0].shape)}")
    if accepted.shape != (B,) or accepted.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"accepted: expected {B} integers, got {accepted.dtype} {tuple(accepted.shape)}")
    k_dtype = k0.dtype
    strides = None
    kk, gg = [], []
    for l in range(L):
        k = _heads_last_contiguous(ks[l])
        if k.shape != k0.shape or k.dtype != k_dtype:
            raise ValueError(f"k[{l}]: expected {k_dtype} {tuple(k0.shape)}, got {k.dtype} {tuple(k.shape)}")
        if strides is None:
            strides = k.stride()[:3]
        elif k.stride()[:3] != strides:
            k = k.contiguous()
            if k.stride()[:3] != strides:
                raise ValueError(f"k[{l}]: the layers' k tensors need the same strides")
        d = deltas[l]
        if d.shape != (B, T, HV, HEAD_DIM) or d.dtype != torch.float32 or not d.is_contiguous():
            raise ValueError(f"deltas[{l}]: expected a contiguous float32 tensor of shape {(B, T, HV, HEAD_DIM)}")
        _check_state_inplace(what, states[l], B, HV)
        g = gs[l]
        if g.shape != (B, T, HV) or g.dtype != torch.float32:
            raise ValueError(f"g[{l}]: expected float32 {(B, T, HV)}, got {g.dtype} {tuple(g.shape)}")
        kk.append(k)
        gg.append(g.contiguous())
    arr = ctypes.c_void_p * L
    status = _lib.load().gdn_delta_commit_layers(
        arr(*[s.data_ptr() for s in states]), arr(*[k.data_ptr() for k in kk]), _DTYPES[k_dtype],
        arr(*[g.data_ptr() for g in gg]), arr(*[d.data_ptr() for d in deltas]), L,
        accepted.to(torch.int64).contiguous().data_ptr(), B, T, H, HV, HEAD_DIM, HEAD_DIM, *strides, _stream())
    _lib.check(status, what)


def gated_delta_rule_rollback(state, snapshots, accepted) -> None:
    """``state[b] <- snapshots[b, accepted[b] - 1]`` for rows with ``accepted[b] >= 1`` (clamped to T)."""
    what = "gated_delta_rule_rollback"
    _require_cuda(what, state, snapshots, accepted)
    if snapshots.dim() != 5:
        raise ValueError(f"snapshots: expected [B, T, HV, 128, 128], got {tuple(snapshots.shape)}")
    B, T, HV = snapshots.shape[:3]
    _check_state_inplace(what, state, B, HV)
    if snapshots.dtype != torch.float32 or not snapshots.is_contiguous():
        raise ValueError("snapshots: expected a contiguous float32 tensor")
    if accepted.shape != (B,) or accepted.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"accepted: expected {B} integers, got {accepted.dtype} {tuple(accepted.shape)}")
    status = _lib.load().gdn_snapshot_commit(state.data_ptr(), snapshots.data_ptr(),
                                             accepted.to(torch.int64).contiguous().data_ptr(), B, T, HV, HEAD_DIM,
                                             HEAD_DIM, _stream())
    _lib.check(status, what)
