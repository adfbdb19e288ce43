"""fp32 CPU restatement of the ops that wrap the gated delta rule (test infrastructure only).

Rounding follows the reference's eager path on bf16 tensors, which was checked on the CPU:
``F.conv1d`` equals an fp32 sum in tap order rounded once to bf16, ``F.silu`` on bf16
equals ``x / (1 + exp(-x))`` in fp32 rounded to bf16, and the decode step multiplies
in bf16 (each product rounded) before an fp32 sum.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def _silu_bf16(x_f32: torch.Tensor) -> torch.Tensor:
    x = x_f32.to(torch.bfloat16).float()
    return (x / (1.0 + torch.exp(-x))).to(torch.bfloat16)


def causal_conv1d(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Depthwise causal conv (kernel = ``weight.shape[-1]``) then SiLU (``model/model.py:199-204``).

    x ``[B, T, C]`` bf16, weight ``[C, K]``; returns ``[B, T, C]`` in x's dtype. Output t of
    channel c is silu(sum_i w[c, i] * x[t - K + 1 + i, c]) with zeros before the start.
    """
    B, T, C = x.shape
    K = weight.shape[-1]
    xp = F.pad(x.float().transpose(1, 2), (K - 1, 0))
    acc = torch.zeros(B, C, T)
    for i in range(K):
        acc = acc + weight[:, i].float()[None, :, None] * xp[..., i:i + T]
    return _silu_bf16(acc).to(x.dtype).transpose(1, 2)


def causal_conv1d_step(x: torch.Tensor, state: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """One decode token (``model/model.py:207-214``); updates ``state`` ``[B, C, K]`` in place.

    The window is the last K entries of state ++ x; the state becomes that window. The
    taps are multiplied in the state's dtype (bf16 products), summed, then SiLU.
    """
    K = weight.shape[-1]
    window = torch.cat((state, x.to(state.dtype)[..., None]), dim=-1)[..., -K:]
    state.copy_(window)
    prod = (window * weight.unsqueeze(0)).float()
    acc = prod[..., 0]
    for i in range(1, K):
        acc = acc + prod[..., i]
    y = acc.to(state.dtype).float()
    return (y / (1.0 + torch.exp(-y))).to(state.dtype).to(x.dtype)


def conv_step(state, qkv, weight, key_dim: int, value_dim: int, head_k_dim: int, head_v_dim: int):
    """Conv over the state window plus T new tokens (``model/model.py:324-339``).

    state ``[B, C, taps]``, qkv ``[B, T, C]``, weight ``[C, 1, 4]``. ext = state ++ qkv^T
    ``[B, C, taps + T]``; output t = silu(sum_i w_i ext[t + taps - 3 + i]). Returns
    ``(ext, q, k, v)`` with q, k repeat-interleaved to the value heads.
    """
    B, T, C = qkv.shape
    taps = state.shape[-1]
    w = weight.reshape(C, -1)
    K = w.shape[-1]
    ext = torch.cat((state, qkv.transpose(1, 2).to(state.dtype)), dim=-1)
    acc = torch.zeros(B, C, T)
    first = taps + 1 - K  # column of ext feeding tap 0 of output 0
    for i in range(K):
        acc = acc + w[:, i].float()[None, :, None] * ext[..., first + i:first + i + T].float()
    conv = _silu_bf16(acc).transpose(1, 2)
    q, k, v = conv.split([key_dim, key_dim, value_dim], dim=-1)
    k_heads, v_heads = key_dim // head_k_dim, value_dim // head_v_dim
    q = q.reshape(B, T, k_heads, head_k_dim).repeat_interleave(v_heads // k_heads, dim=2)
    k = k.reshape(B, T, k_heads, head_k_dim).repeat_interleave(v_heads // k_heads, dim=2)
    return ext, q.contiguous(), k.contiguous(), v.reshape(B, T, v_heads, head_v_dim).contiguous()


def gated_rms_norm(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Output-gated RMSNorm (``model/model.py:150-158``): bf16(w * bf16(x rsqrt(mean x^2 + eps))) * silu(z)."""
    xf = x.float()
    normed = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    y = weight * normed
    zf = z.float()
    return (y.float() * (zf / (1.0 + torch.exp(-zf)))).to(x.dtype)


def delta_gates(b, a, dt_bias, log_decay_rate, valid=None):
    """beta = sigmoid(b) in b's dtype; g = log_decay_rate * softplus(a + dt_bias) in fp32 (``model/model.py:314-321``).

    ``log_decay_rate`` is ``-exp(A_log)`` (``inference/engine.py:170``). Rows with ``valid``
    False get beta = 0 and g = 0.
    """
    beta = b.sigmoid()
    g = log_decay_rate.float() * F.softplus(a.float() + dt_bias)
    if valid is None:
        return beta, g
    kept = valid[..., None]
    return beta * kept.to(beta.dtype), g * kept.float()


def apply_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotary embedding on bf16 with per-row cos / sin ``[B, T, F]`` (``model/model.py:188-196``,
    ``_rotate_half`` ``:177-179``): cos and sin rounded to x's dtype, every product and the sum
    rounded to x's dtype, the elements past 2F copied."""
    cos, sin = cos.to(x.dtype), sin.to(x.dtype)
    rd = 2 * cos.shape[-1]
    cos = torch.cat((cos, cos), dim=-1).unsqueeze(-2)
    sin = torch.cat((sin, sin), dim=-1).unsqueeze(-2)
    x_rot, x_pass = x[..., :rd], x[..., rd:]
    x1, x2 = x_rot.chunk(2, dim=-1)
    turned = torch.cat((-x2, x1), dim=-1)
    return torch.cat((x_rot * cos + turned * sin, x_pass), dim=-1)


def rotate_into_cache(k, v, qm, km, vm, cos_c, sin_c, cos_m, sin_m, k_cache, v_cache, rows, positions, tail_start):
    """The drafter's cache writes (``model/model.py:342-351``), in place on the caches; returns
    the rotated mask-row queries."""
    k_cache[rows, positions] = apply_rotary(k, cos_c, sin_c)
    v_cache[rows, positions] = v
    B, M = qm.shape[:2]
    q = apply_rotary(qm, cos_m, sin_m)
    k_cache[:B, tail_start:tail_start + M] = apply_rotary(km, cos_m, sin_m)
    v_cache[:B, tail_start:tail_start + M] = vm
    return q


def decode_attention_f32(q, k_cache, v_cache, mask, scale):
    """Attention of q ``[B, R, H, D]`` over the first ``L`` keys of the caches ``[rows, slots, Hkv, D]``
    with the additive mask ``[B, 1, R, L]``, in fp32 (the float32 reference that
    ``model/triton_kernels_test.py:122-126`` holds ``decode_attention``, ``model/model.py:354-361``,
    to). Key head ``h // (H // Hkv)``; a row with every key masked gets zeros."""
    B, R, H, D = q.shape
    L = mask.shape[-1]
    G = H // k_cache.shape[2]
    keys, values = (t[:B, :L].float().repeat_interleave(G, dim=2) for t in (k_cache, v_cache))
    scores = torch.einsum("brhd,blhd->bhrl", q.float(), keys) * scale + mask.float()
    probs = torch.softmax(scores, dim=-1).nan_to_num(0.0)
    return torch.einsum("bhrl,blhd->brhd", probs, values)
