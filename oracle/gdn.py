"""fp32 CPU restatement of the reference's gated delta rule (test infrastructure only).

Shapes follow the reference: q, k ``[B, T, H, Dk]`` with H equal to the number of
value heads (the reference's caller has already repeat-interleaved them, see
``model/model.py:487-490``), v ``[B, T, HV, Dv]``, g ``[B, T, HV]`` (log decay, fp32),
beta ``[B, T, HV]``, state ``[B, HV, Dk, Dv]`` fp32. ``expand_heads`` gives the
repeat-interleave mapping for callers that hold q, k at fewer key heads.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def expand_heads(x: torch.Tensor, heads: int) -> torch.Tensor:
    """Repeat-interleave key heads up to ``heads`` value heads (``model/model.py:487-490``)."""
    have = x.shape[2]
    if have == heads:
        return x
    if heads % have:
        raise ValueError(f"{heads} value heads are not a multiple of {have} key heads")
    return x.repeat_interleave(heads // have, dim=2)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x * rsqrt(sum(x^2) + eps) over the last dim (``model/model.py:217-218``)."""
    return x * torch.rsqrt((x * x).sum(dim=-1, keepdim=True) + eps)


def _prepare(q, k, v, g, beta):
    heads = v.shape[2]
    q, k = expand_heads(q, heads), expand_heads(k, heads)
    dk = k.shape[-1]
    qn = l2norm(q.float()) * dk ** -0.5
    kn = l2norm(k.float())
    return qn, kn, v.float(), g.float(), beta.float()


def recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None, output_final_state=False):
    """Token-by-token gated delta rule (``model/model.py:221-239``).

    Per token: S <- exp(g) S; delta = beta (v - k^T S); S <- S + k delta^T; o = q^T S.
    Returns ``(o in q.dtype, final state or None)``.
    """
    out_dtype = q.dtype
    qn, kn, vf, gf, bf = _prepare(q, k, v, g, beta)
    B, T, HV, Dk = kn.shape
    Dv = vf.shape[-1]
    if initial_state is None:
        S = torch.zeros(B, HV, Dk, Dv, dtype=torch.float32)
    else:
        S = initial_state.to(torch.float32).clone()
    outs = []
    for t in range(T):
        S = S * torch.exp(gf[:, t])[:, :, None, None]
        kt = kn[:, t]
        recalled = torch.einsum("bhk,bhkv->bhv", kt, S)
        delta = bf[:, t, :, None] * (vf[:, t] - recalled)
        S = S + kt[..., :, None] * delta[..., None, :]
        outs.append(torch.einsum("bhk,bhkv->bhv", qn[:, t], S))
    o = torch.stack(outs, dim=1) if outs else torch.zeros(B, 0, HV, Dv)
    return o.to(out_dtype), (S if output_final_state else None)


def chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=64, initial_state=None, output_final_state=False):
    """Chunked (WY / UT) gated delta rule, chunk 64 (``model/model.py:242-286``).

    The sequence is zero-padded to a multiple of the chunk (``:249-252``). Inside chunk
    c with cumulative log decay gc: decay_ij = exp(gc_i - gc_j) for j <= i;
    L = I + strict_lower(diag(beta) K K^T * decay); u = L^-1 diag(beta) V;
    w = L^-1 diag(beta exp(gc)) K (``:260-270``). Across chunks (``:275-283``):
    v_new = u - w S; o = (Q K^T * decay) v_new + diag(exp(gc)) Q S;
    S <- exp(gc_last) S + (diag(exp(gc_last - gc)) K)^T v_new.
    """
    out_dtype = q.dtype
    qn, kn, vf, gf, bf = _prepare(q, k, v, g, beta)
    B, T, HV, Dk = kn.shape
    Dv = vf.shape[-1]
    C = chunk_size
    padded = -(-T // C) * C
    extra = padded - T
    if extra:
        qn, kn, vf = (F.pad(x, (0, 0, 0, 0, 0, extra)) for x in (qn, kn, vf))
        gf, bf = (F.pad(x, (0, 0, 0, extra)) for x in (gf, bf))
    n_chunks = padded // C

    def heads_first(x):  # [B, Tp, HV, ...] -> [B, HV, n_chunks, C, ...]
        x = x.transpose(1, 2)
        return x.reshape(B, HV, n_chunks, C, *x.shape[3:])

    Qc, Kc, Vc, Gc, Bc = (heads_first(x) for x in (qn, kn, vf, gf, bf))
    gc = Gc.cumsum(dim=-1)
    rows = torch.arange(C)
    incl = rows[:, None] >= rows[None, :]
    strict = rows[:, None] > rows[None, :]
    gap = (gc[..., :, None] - gc[..., None, :]).masked_fill(~incl, 0.0)
    decay = torch.exp(gap).masked_fill(~incl, 0.0)

    kk = (Kc * Bc[..., None]) @ Kc.transpose(-1, -2)
    Lmat = (kk * decay).masked_fill(~strict, 0.0) + torch.eye(C)
    u = torch.linalg.solve_triangular(Lmat, Vc * Bc[..., None], upper=False, unitriangular=True)
    w = torch.linalg.solve_triangular(Lmat, Kc * (Bc * torch.exp(gc))[..., None], upper=False, unitriangular=True)

    if initial_state is None:
        S = torch.zeros(B, HV, Dk, Dv, dtype=torch.float32)
    else:
        S = initial_state.to(torch.float32).clone()
    o = torch.empty(B, HV, n_chunks, C, Dv)
    for c in range(n_chunks):
        qc, kc, gcc = Qc[:, :, c], Kc[:, :, c], gc[:, :, c]
        v_new = u[:, :, c] - w[:, :, c] @ S
        local = (qc @ kc.transpose(-1, -2) * decay[:, :, c]) @ v_new
        carried = (qc * torch.exp(gcc)[..., None]) @ S
        o[:, :, c] = local + carried
        last = gcc[..., -1]
        k_tail = kc * torch.exp(last[..., None] - gcc)[..., None]
        S = S * torch.exp(last)[..., None, None] + k_tail.transpose(-1, -2) @ v_new
    o = o.reshape(B, HV, padded, Dv)[:, :, :T].transpose(1, 2)
    return o.to(out_dtype), (S if output_final_state else None)


def chunk_gated_delta_rule_varlen(q, k, v, g, beta, cu_seqlens, initial_state=None, output_final_state=False):
    """Packed varlen prefill: sequence i is tokens ``cu_seqlens[i]:cu_seqlens[i+1]`` of a B=1 batch.

    The reference has no varlen path (it pads and zeroes the gates instead,
    ``inference/engine.py:378``); the oracle is one call of ``chunk_gated_delta_rule``
    per sequence with that sequence's initial state, which the packed call must equal.
    """
    if q.shape[0] != 1:
        raise ValueError("varlen inputs are packed into a batch of 1")
    cu = [int(x) for x in cu_seqlens.tolist()]
    n = len(cu) - 1
    outs, finals = [], []
    for i in range(n):
        s, e = cu[i], cu[i + 1]
        h0 = None if initial_state is None else initial_state[i:i + 1]
        o, S = chunk_gated_delta_rule(q[:, s:e], k[:, s:e], v[:, s:e], g[:, s:e], beta[:, s:e],
                                      initial_state=h0, output_final_state=True)
        outs.append(o)
        finals.append(S)
    o = torch.cat(outs, dim=1) if outs else torch.zeros(1, 0, v.shape[2], v.shape[3], dtype=q.dtype)
    return o, (torch.cat(finals, dim=0) if output_final_state else None)


def advance_gated_delta_rule(k, v, g, beta, state, steps):
    """New state after the first ``clamp(steps[b], 0, T)`` tokens of row b, no outputs.

    Restates the eager fallback of ``gated_delta_rule_advance_inplace``
    (``model/model.py:305-311``): tokens at or past ``steps[b]`` get g = 0 and beta = 0,
    which leaves the state unchanged. Returns the new state (the caller copies it in place).
    """
    T = k.shape[1]
    keep = (torch.arange(T)[None, :] < steps.reshape(-1, 1).to(torch.int64)).to(torch.float32)[..., None]
    _, S = recurrent_gated_delta_rule(torch.zeros_like(k), k, v, g.float() * keep, beta * keep.to(beta.dtype),
                                      initial_state=state, output_final_state=True)
    return S


def verify_with_snapshots(q, k, v, g, beta, initial_state):
    """Outputs of T drafted tokens plus the state after each token, ``[B, T, HV, Dk, Dv]``.

    The per-token states are the rollback points of block-K speculative verify: the
    state after ``j`` accepted tokens equals snapshot ``j - 1``, the same state that
    ``gated_delta_rule_advance_inplace`` recomputes (``inference/engine.py:250-258``).
    """
    T = q.shape[1]
    snaps = []
    outs = []
    S = initial_state.float()
    for t in range(T):
        o, S = recurrent_gated_delta_rule(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], g[:, t:t + 1], beta[:, t:t + 1],
                                          initial_state=S, output_final_state=True)
        outs.append(o)
        snaps.append(S)
    return torch.cat(outs, dim=1), torch.stack(snaps, dim=1)


def exact_recurrence_f64(q, k, v, g, beta, state=None):
    """float64 recurrence used to grade accuracy (``model/metal_test.py:25-35``)."""
    heads = v.shape[2]
    q, k = expand_heads(q, heads).double(), expand_heads(k, heads).double()
    v, g, beta = v.double(), g.double(), beta.double()
    B, T, HV, Dk = k.shape
    S = torch.zeros(B, HV, Dk, v.shape[-1], dtype=torch.float64) if state is None else state.double().clone()
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * Dk ** -0.5
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    outs = []
    for t in range(T):
        S = S * g[:, t].exp()[..., None, None]
        delta = beta[:, t, :, None] * (v[:, t] - torch.einsum("bhk,bhkv->bhv", k[:, t], S))
        S = S + k[:, t][..., :, None] * delta[..., None, :]
        outs.append(torch.einsum("bhk,bhkv->bhv", q[:, t], S))
    return torch.stack(outs, 1), S
