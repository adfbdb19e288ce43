"""One gated-delta layer between the input projections and ``out_proj`` (CUDA only).

``decode_layer_step`` does, for one new token per row, what the StaticCache decode branch
of ``GatedDeltaNet.forward`` (``model/model.py:465-467``, ``:496-499``, ``:516``) does:
conv step + SiLU, q/k L2 norm, gated delta rule step on the state in place, and the
output-gated RMSNorm. ``prefill_layer`` does the same for a prompt (the prefill branch,
``:478-479``, ``:482-489``, ``:505-506``, ``:516``): causal conv1d + SiLU, then the chunked
gated delta rule with the output-gated RMSNorm fused into the same call.
"""

from __future__ import annotations

import torch

from . import _lib
from .conv import causal_conv1d, conv_state_commit, conv_step
from .gated_delta import (_DTYPES, HEAD_DIM, _require_cuda, _stream, gated_delta_rule_advance_inplace,
                          gated_delta_rule_chunk_gated_norm, gated_delta_rule_delta_commit,
                          gated_delta_rule_delta_commit_layers, gated_delta_rule_rollback, gated_delta_rule_step,
                          gated_delta_rule_verify, gated_delta_rule_verify_deltas)
from .norm import gated_rms_norm


def prefill_layer(qkv, conv_weight, g, beta, z, norm_weight, key_heads: int, eps: float = 1e-6, initial_state=None,
                  output_final_state: bool = True, scale: float | None = None, cu_seqlens=None):
    """qkv ``[B, T, C]`` pre-conv bf16 (q | k | v channels, C = 2 * key_heads * 128 + HV * 128),
    conv_weight ``[C, taps]`` (or ``[C, 1, taps]``), g ``[B, T, HV]`` fp32, beta ``[B, T, HV]``,
    z ``[B, T, HV, 128]`` bf16, norm_weight ``[128]`` bf16; returns ``(y [B, T, HV, 128] bf16,
    final_state [rows, HV, 128, 128] fp32 or None)``. With ``cu_seqlens`` (B = 1) the packed
    sequences are convolved and scanned separately. q and k are read as views of the conv
    output; the key heads are never repeated in memory."""
    what = "prefill_layer"
    _require_cuda(what, qkv, conv_weight, g, beta, z, norm_weight)
    if qkv.dim() != 3:
        raise ValueError(f"qkv: expected [B, T, C], got {tuple(qkv.shape)}")
    B, T, C = qkv.shape
    kd = key_heads * HEAD_DIM
    if C <= 2 * kd or (C - 2 * kd) % HEAD_DIM:
        raise ValueError(f"qkv: {C} channels do not split into 2 x {kd} key channels and whole value heads")
    HV = (C - 2 * kd) // HEAD_DIM
    y = causal_conv1d(qkv, conv_weight.reshape(C, -1), cu_seqlens=cu_seqlens)
    q = y[..., :kd].view(B, T, key_heads, HEAD_DIM)
    k = y[..., kd:2 * kd].view(B, T, key_heads, HEAD_DIM)
    v = y[..., 2 * kd:].view(B, T, HV, HEAD_DIM)
    return gated_delta_rule_chunk_gated_norm(q, k, v, g, beta, z, norm_weight, eps=eps, initial_state=initial_state,
                                             output_final_state=output_final_state, scale=scale,
                                             cu_seqlens=cu_seqlens)


def decode_layer_step(qkv, conv_state, conv_weight, g, beta, state, z, norm_weight, key_heads: int,
                      eps: float = 1e-6, scale: float | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """qkv ``[B, C]`` pre-conv bf16 (q | k | v channels); conv_state ``[B, C, taps]`` and state
    ``[B, HV, 128, 128]`` are updated in place; g ``[B, HV]`` fp32, beta ``[B, HV]`` bf16, z
    ``[B, HV, 128]``; returns the normed output ``[B, HV, 128]`` bf16. ``workspace`` (``[B, C]``
    bf16, allocated here when not given) receives the post-conv activations."""
    what = "decode_layer_step"
    _require_cuda(what, qkv, conv_state, conv_weight, g, beta, state, z, norm_weight)
    B, C = qkv.shape
    HV = state.shape[1]
    if C != 2 * key_heads * HEAD_DIM + HV * HEAD_DIM:
        raise ValueError(f"qkv: expected {2 * key_heads * HEAD_DIM + HV * HEAD_DIM} channels, got {C}")
    for name, t in (("qkv", qkv), ("conv_weight", conv_weight), ("z", z), ("norm_weight", norm_weight)):
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name}: expected bfloat16, got {t.dtype}")
    if z.numel() != B * HV * HEAD_DIM or norm_weight.numel() != HEAD_DIM:
        raise ValueError(f"z, norm_weight: expected {(B, HV, HEAD_DIM)} and {(HEAD_DIM,)}, got {tuple(z.shape)} and "
                         f"{tuple(norm_weight.shape)}")
    if g.numel() != B * HV or beta.numel() != B * HV:
        raise ValueError(f"g, beta: expected {(B, HV)}, got {tuple(g.shape)} and {tuple(beta.shape)}")
    taps = conv_state.shape[-1]
    w = conv_weight.reshape(C, -1).contiguous()
    if conv_state.shape != (B, C, taps) or not conv_state.is_contiguous() or conv_state.dtype != torch.bfloat16:
        raise ValueError(f"conv_state: expected a contiguous bfloat16 tensor of shape {(B, C, taps)}, got "
                         f"{conv_state.dtype} {tuple(conv_state.shape)}")
    if state.dtype != torch.float32 or not state.is_contiguous() or state.shape != (B, HV, HEAD_DIM, HEAD_DIM):
        raise ValueError(f"state: expected a contiguous float32 tensor of shape {(B, HV, HEAD_DIM, HEAD_DIM)}, got "
                         f"{state.dtype} {tuple(state.shape)}")
    if qkv.stride(-1) != 1:
        qkv = qkv.contiguous()
    g = g.reshape(B, HV).to(torch.float32).contiguous()
    beta = beta.reshape(B, HV).to(torch.bfloat16).contiguous()
    z = z.reshape(B, HV, HEAD_DIM).contiguous()
    out = torch.empty(B, HV, HEAD_DIM, dtype=torch.bfloat16, device=qkv.device)
    if workspace is None:
        workspace = torch.empty(B, C, dtype=torch.bfloat16, device=qkv.device)
    elif workspace.shape != (B, C) or workspace.dtype != torch.bfloat16 or not workspace.is_contiguous():
        raise ValueError(f"workspace: expected a contiguous bfloat16 tensor of shape {(B, C)}, got {workspace.dtype} "
                         f"{tuple(workspace.shape)}")
    status = _lib.load().gdn_decode_layer(
        qkv.data_ptr(), qkv.stride(0), conv_state.data_ptr(), w.data_ptr(), g.data_ptr(), beta.data_ptr(),
        state.data_ptr(), z.data_ptr(), norm_weight.contiguous().data_ptr(), out.data_ptr(), workspace.data_ptr(),
        B, key_heads, HV,
        HEAD_DIM, HEAD_DIM, taps, w.shape[1], float(HEAD_DIM ** -0.5 if scale is None else scale), float(eps), _stream())
    _lib.check(status, what)
    return out


def verify_layer_step(qkv, conv_state, conv_weight, g, beta, state, z, norm_weight, key_heads: int, ext_out=None,
                      eps: float = 1e-6, scale: float | None = None, snapshots=None, deltas=None):
    """The verify branch of one delta layer for T drafted tokens per row (``inference/engine.py:427-435``
    without the drafter's mask rows): ``conv_step`` over the conv-state window and the T new tokens
    (the window ``ext [B, C, taps + T]`` goes to ``ext_out``), the gated delta rule outputs from
    ``state`` (``delta_outputs``, ``:250-252``; the state is read, not written) and the output-gated
    RMSNorm. qkv ``[B, T, C]`` pre-conv bf16; conv_state ``[B, C, taps]``; g, beta ``[B, T, HV]``;
    z ``[B, T, HV, 128]``. Returns ``(y [B, T, HV, 128] bf16, pending)``; ``pending`` goes to
    ``verify_layer_commit`` once the accepted lengths are known.

    With ``snapshots`` (a ``[B, T, HV, 128, 128]`` fp32 buffer) the verify also writes the state after
    every token, and the commit copies the accepted one instead of advancing the state again. With
    ``deltas`` (a ``[B, T, HV, 128]`` fp32 buffer) the verify runs as one tensor-core block per state
    (for bf16 rows and T <= 8) and keeps each token's update vector, and the commit advances the state
    by the accepted tokens in one streaming pass, without the advance's reductions (states agree with
    the advance to fp32 rounding). At most one of the two."""
    what = "verify_layer_step"
    _require_cuda(what, qkv, conv_state, conv_weight, g, beta, state, z, norm_weight, ext_out, snapshots, deltas)
    if qkv.dim() != 3:
        raise ValueError(f"qkv: expected [B, T, C], got {tuple(qkv.shape)}")
    B, T, C = qkv.shape
    kd = key_heads * HEAD_DIM
    if C <= 2 * kd or (C - 2 * kd) % HEAD_DIM:
        raise ValueError(f"qkv: {C} channels do not split into 2 x {kd} key channels and whole value heads")
    vd = C - 2 * kd
    if snapshots is not None and deltas is not None:
        raise ValueError(f"{what}: pass snapshots or deltas, not both")
    if deltas is not None and qkv.dtype == torch.bfloat16 and 1 <= T <= 8:
        return _verify_layer_deltas(what, qkv, conv_state, conv_weight, g, beta, state, z, norm_weight, key_heads,
                                    ext_out, eps, scale, deltas)
    _, q, k, v = conv_step(conv_state, qkv, conv_weight, kd, vd, HEAD_DIM, HEAD_DIM, ext_out=ext_out)
    if snapshots is not None:
        o, snapshots = gated_delta_rule_verify(q, k, v, g, beta, state, snapshots=snapshots, scale=scale)
    elif deltas is not None:
        o, deltas = gated_delta_rule_verify_deltas(q, k, v, g, beta, state, deltas=deltas, scale=scale)
    else:
        o, _ = gated_delta_rule_step(q, k, v, g, beta, initial_state=state, output_final_state=False, scale=scale)
    y = gated_rms_norm(o.view(-1, HEAD_DIM), z.reshape(-1, HEAD_DIM), norm_weight, eps).view(o.shape)
    return y, (k, v, g, beta, snapshots, deltas)


def _verify_layer_deltas(what, qkv, conv_state, conv_weight, g, beta, state, z, norm_weight, key_heads, ext_out, eps,
                         scale, deltas):
    """The kept-update-vector verify of bf16 rows and 1 <= T <= 8 tokens as one library call
    (``gdn_verify_layer_deltas``): the conv step, then the tensor-core block verify as its
    programmatic dependent, with the gated norm (in the block's drain for few states)."""
    B, T, C = qkv.shape
    kd = key_heads * HEAD_DIM
    HV = (C - 2 * kd) // HEAD_DIM
    taps = conv_state.shape[-1]
    w = conv_weight.reshape(C, -1)
    if qkv.stride(-1) != 1:
        qkv = qkv.contiguous()
    if conv_state.shape != (B, C, taps) or conv_state.dtype != torch.bfloat16 or not conv_state.is_contiguous():
        raise ValueError(f"conv_state: expected a contiguous bfloat16 tensor of shape {(B, C, taps)}, got "
                         f"{conv_state.dtype} {tuple(conv_state.shape)}")
    if w.dtype != torch.bfloat16:
        raise ValueError(f"conv_weight: expected bfloat16, got {w.dtype}")
    w = w.contiguous()
    ext = torch.empty(B, C, taps + T, dtype=torch.bfloat16, device=qkv.device) if ext_out is None else ext_out
    if ext.shape != (B, C, taps + T) or ext.dtype != torch.bfloat16 or not ext.is_contiguous():
        raise ValueError(f"ext_out: expected a contiguous bfloat16 tensor of shape {(B, C, taps + T)}, got {ext.dtype} "
                         f"{tuple(ext.shape)}")
    if state.dtype != torch.float32 or not state.is_contiguous() or state.shape != (B, HV, HEAD_DIM, HEAD_DIM):
        raise ValueError(f"state: expected a contiguous float32 tensor of shape {(B, HV, HEAD_DIM, HEAD_DIM)}, got "
                         f"{state.dtype} {tuple(state.shape)}")
    shape = (B, T, HV, HEAD_DIM)
    if deltas.shape != shape or deltas.dtype != torch.float32 or not deltas.is_contiguous():
        raise ValueError(f"deltas: expected a contiguous float32 tensor of shape {shape}, got {deltas.dtype} "
                         f"{tuple(deltas.shape)}")
    if g.shape != (B, T, HV) or beta.shape != (B, T, HV):
        raise ValueError(f"g, beta: expected {(B, T, HV)}, got {tuple(g.shape)} and {tuple(beta.shape)}")
    g = g.to(torch.float32).contiguous()
    if beta.dtype not in (torch.bfloat16, torch.float32):
        beta = beta.to(torch.float32)
    beta = beta.contiguous()
    z = z.reshape(shape)
    if z.dtype != torch.bfloat16:
        raise ValueError(f"z: expected bfloat16, got {z.dtype}")
    z = z.contiguous()
    nw = norm_weight.reshape(HEAD_DIM).to(torch.bfloat16).contiguous()
    q = torch.empty(shape, dtype=torch.bfloat16, device=qkv.device)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    y = torch.empty_like(q)
    status = _lib.load().gdn_verify_layer_deltas(
        qkv.data_ptr(), qkv.stride(0), qkv.stride(1), conv_state.data_ptr(), w.data_ptr(), ext.data_ptr(),
        q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), _DTYPES[beta.dtype],
        state.data_ptr(), z.data_ptr(), nw.data_ptr(), y.data_ptr(), deltas.data_ptr(), B, T, key_heads, HV,
        HEAD_DIM, HEAD_DIM, taps, w.shape[1], float(HEAD_DIM ** -0.5 if scale is None else scale), float(eps),
        _stream())
    _lib.check(status, what)
    return y, (k, v, g, beta, None, deltas)


def verify_layer_commit(pending, state, accepted, ext=None, conv_state=None) -> None:
    """Keep the first ``accepted[b]`` verified tokens of row b in ``state`` (the commit of
    ``inference/engine.py:471-472``): advance the state by them again (the reference's design,
    ``delta_commit``), copy the snapshot after them when the verify wrote snapshots, or apply the kept
    update vectors when it kept them. With ``ext``
    and ``conv_state`` the conv state is rolled forward too (``conv_state_commit``; the engine runs
    that once over every layer's stacked conv state, ``:473-474``)."""
    k, v, g, beta, snapshots, deltas = pending
    if snapshots is not None:
        gated_delta_rule_rollback(state, snapshots, accepted)
    elif deltas is not None:
        gated_delta_rule_delta_commit(k, g, deltas, state, accepted)
    else:
        gated_delta_rule_advance_inplace(k, v, g, beta, state, accepted)
    if ext is not None:
        conv_state_commit(ext, conv_state, accepted)


def verify_layers_commit(pendings, states, accepted, ext=None, conv_states=None) -> None:
    """``verify_layer_commit`` for every layer of a verify step (the engine's commit loop,
    ``inference/engine.py:471-474``): the layers whose verify kept update vectors are committed by
    one launch (``gated_delta_rule_delta_commit_layers``), the others one by one; with ``ext`` and
    ``conv_states`` (stacked ``[layers, B, C, ..]``) the conv states follow in one more launch."""
    pendings, states = list(pendings), list(states)
    if len(pendings) != len(states):
        raise ValueError(f"verify_layers_commit: {len(pendings)} pending verifies for {len(states)} states")
    kept = [i for i, p in enumerate(pendings) if p[5] is not None and p[4] is None]
    if kept:
        gated_delta_rule_delta_commit_layers([pendings[i][0] for i in kept], [pendings[i][2] for i in kept],
                                             [pendings[i][5] for i in kept], [states[i] for i in kept], accepted)
    for i, p in enumerate(pendings):
        if i not in kept:
            verify_layer_commit(p, states[i], accepted)
    if ext is not None:
        conv_state_commit(ext, conv_states, accepted)


def in_proj_conv(x, weight, conv_weight, conv_channels: int, cu_seqlens=None, conv_state: bool = False,
                 weight_scale=None):
    """The merged input projection of a gated-delta layer with the causal conv + SiLU fused into the
    GEMM: ``y = x @ weight.T`` (bf16, fp32 accumulation), then ``silu(causal_conv1d)`` over the first
    ``conv_channels`` columns (the qkv channels; ``weight`` holds their rows first, then z, b, a).
    x ``[T, hidden]`` or ``[1, T, hidden]`` bf16; conv_weight ``[conv_channels, 4]`` (or ``[C, 1,
    4]``). Returns ``out [.., T, N]``, and with ``conv_state`` also the last 4 pre-conv rows of
    every sequence ``[sequences, conv_channels, 4]`` (the cache's conv state).

    ``weight`` may be fp8 (``torch.float8_e4m3fn`` codes with ``weight_scale`` [N] fp32, the
    reference's ``FP8Linear`` buffers): then ``y = (x @ codes.T) * weight_scale`` computed as
    ``inference/fp8.py`` does (fp16 activation rows with a power-of-two scale per row, fp16 codes,
    fp32 accumulation)."""
    what = "in_proj_conv"
    _require_cuda(what, x, weight, conv_weight, cu_seqlens, weight_scale)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    T, K = x2.shape
    N = weight.shape[0]
    if weight.dim() != 2 or weight.shape[1] != K:
        raise ValueError(f"weight: expected [N, {K}], got {tuple(weight.shape)}")
    fp8 = weight.dtype == torch.float8_e4m3fn
    if x.dtype != torch.bfloat16 or not (fp8 or weight.dtype == torch.bfloat16):
        raise ValueError(f"x, weight: expected bfloat16 and bfloat16 or float8_e4m3fn, got {x.dtype}, {weight.dtype}")
    if fp8 and (weight_scale is None or weight_scale.dtype != torch.float32 or weight_scale.numel() != N):
        raise ValueError(f"weight_scale: expected {N} float32 row scales for an fp8 weight")
    if conv_channels:
        if conv_weight is None or conv_weight.dtype != torch.bfloat16:
            raise ValueError("conv_weight: expected bfloat16")
        cw = conv_weight.reshape(conv_channels, -1).contiguous()
        if cw.shape[1] != 4:
            raise ValueError(f"conv_weight: expected {conv_channels} channels of 4 taps, got {tuple(conv_weight.shape)}")
    else:
        cw = None
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    cu = None
    seqs = 1
    if cu_seqlens is not None:
        cu = cu_seqlens.to(device=x.device, dtype=torch.int32).contiguous()
        seqs = cu.numel() - 1
    out = torch.empty(*lead, N, dtype=torch.bfloat16, device=x.device)
    state = torch.empty(seqs, conv_channels, 4, dtype=torch.bfloat16, device=x.device) if conv_state else None
    lib = _lib.load()
    common = (None if cw is None else cw.data_ptr(), None if cu is None else cu.data_ptr(), out.data_ptr(), N,
              None if state is None else state.data_ptr())
    if fp8:
        ws_bytes = lib.gdn_in_proj_fp8_prefill_workspace_size(T, K, N, conv_channels)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        scale = weight_scale.contiguous()
        status = lib.gdn_in_proj_conv_fp8(x2.data_ptr(), x2.stride(0), w.data_ptr(), w.stride(0), scale.data_ptr(),
                                          *common, ws.data_ptr(), ws_bytes, T, K, N, conv_channels, seqs, 4, _stream())
    else:
        status = lib.gdn_in_proj_conv(x2.data_ptr(), x2.stride(0), w.data_ptr(), w.stride(0), *common, T, K, N,
                                      conv_channels, seqs, 4, _stream())
    _lib.check(status, what)
    return (out, state) if conv_state else out


def fp8_linear(x, weight, scale):
    """The reference's fp8 GEMM (``fp8_matmul`` / ``FP8Linear.forward``, inference/fp8.py:112-148,
    :177-184): x ``[.., K]`` (cast to bf16) times e4m3 codes ``[N, K]`` with fp32 row scales
    ``[N]`` -> bf16 ``[.., N]``, on the tcgen05 kernel without a conv."""
    shape = x.shape
    y = in_proj_conv(x.reshape(-1, shape[-1]).to(torch.bfloat16), weight, None, 0, weight_scale=scale)
    return y.view(*shape[:-1], weight.shape[0])
