"""Generate the golden vectors in this folder from the reference's own eager functions.

Run in a checkout that has the reference (PostHog/jeeves) available:

    python tests/golden/make_golden.py --reference /path/to/jeeves

It imports ``model.model`` from the reference, runs the reference's eager (CPU, fp32)
functions on seeded inputs, and writes one ``.pt`` file per case next to this script.
The files pin the CPU oracle in ``oracle/`` (``tests/test_oracle.py``) and the CUDA
kernels (``tests/test_gpu_*.py``); neither test needs the reference at run time.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def seeded(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def gdn_inputs(gen, B, T, H, HV, D, dtype, normalise=True):
    """Inputs distributed as the benchmark configs describe them."""
    q = torch.randn(B, T, H, D, generator=gen)
    k = torch.randn(B, T, H, D, generator=gen)
    if normalise:
        q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6)
        k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    v = torch.randn(B, T, HV, D, generator=gen)
    g = -torch.exp(torch.randn(B, T, HV, generator=gen) * 0.5 - 3.0)
    beta = torch.sigmoid(torch.randn(B, T, HV, generator=gen))
    return q.to(dtype), k.to(dtype), v.to(dtype), g, beta.to(dtype)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("JEEVES_REFERENCE"),
                    help="the reference checkout to import model.model from (or set JEEVES_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or JEEVES_REFERENCE")
    sys.path.insert(0, args.reference)
    import model.model as ref  # the reference's own module

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = {}

    # Config 0: one layer, fp32, B=1, T=256, 4 key / 8 value heads, zero initial state.
    q, k, v, g, beta = gdn_inputs(seeded(0), 1, 256, 4, 8, 128, torch.float32)
    qe, ke = q.repeat_interleave(2, dim=2), k.repeat_interleave(2, dim=2)
    o, S = ref.torch_chunk_gated_delta_rule(qe, ke, v, g, beta, output_final_state=True)
    out["chunk_cfg0"] = dict(q=q, k=k, v=v, g=g, beta=beta, o=o, S=S)

    # bf16, ragged length (not a multiple of 64), GQA 2:1, random initial state.
    gen = seeded(11)
    q, k, v, g, beta = gdn_inputs(gen, 2, 100, 2, 4, 128, torch.bfloat16)
    h0 = torch.randn(2, 4, 128, 128, generator=gen) * 0.02
    qe, ke = q.repeat_interleave(2, dim=2), k.repeat_interleave(2, dim=2)
    o, S = ref.torch_chunk_gated_delta_rule(qe, ke, v, g, beta, initial_state=h0, output_final_state=True)
    out["chunk_bf16_ragged"] = dict(q=q, k=k, v=v, g=g, beta=beta, h0=h0, o=o, S=S)

    # Recurrent form over 5 tokens (block-4 verify shape) with an initial state.
    gen = seeded(12)
    q, k, v, g, beta = gdn_inputs(gen, 2, 5, 2, 4, 128, torch.bfloat16, normalise=False)
    h0 = torch.randn(2, 4, 128, 128, generator=gen) * 0.02
    qe, ke = q.repeat_interleave(2, dim=2), k.repeat_interleave(2, dim=2)
    o, S = ref.torch_recurrent_gated_delta_rule(qe, ke, v, g, beta, initial_state=h0, output_final_state=True)
    out["recurrent_bf16"] = dict(q=q, k=k, v=v, g=g, beta=beta, h0=h0, o=o, S=S)

    # Rollback / commit: advance by steps that include the clamped cases.
    gen = seeded(13)
    _, k, v, g, beta = gdn_inputs(gen, 4, 5, 2, 2, 128, torch.bfloat16, normalise=False)
    g = -torch.rand(4, 5, 2, generator=gen)
    h0 = torch.randn(4, 2, 128, 128, generator=gen)
    steps = torch.tensor([-5, 0, 3, 5 + 9])
    state = h0.clone()
    ref.gated_delta_rule_advance_inplace(k, v, g, beta, state, steps)
    out["advance"] = dict(k=k, v=v, g=g, beta=beta, h0=h0, steps=steps, S=state)

    # Prefill conv + SiLU.
    gen = seeded(14)
    x = (torch.randn(2, 37, 96, generator=gen) * 2).to(torch.bfloat16)
    w = (torch.randn(96, 4, generator=gen) * 0.5).to(torch.bfloat16)
    out["conv1d"] = dict(x=x, w=w, y=ref.causal_conv1d(x, w))

    # Decode conv step (state updated in place).
    gen = seeded(15)
    x = (torch.randn(3, 96, generator=gen) * 2).to(torch.bfloat16)
    st = torch.randn(3, 96, 4, generator=gen).to(torch.bfloat16)
    w = (torch.randn(96, 4, generator=gen) * 0.5).to(torch.bfloat16)
    st_after = st.clone()
    y = ref.causal_conv1d_step(x, st_after, w)
    out["conv1d_step"] = dict(x=x, state=st, w=w, y=y, state_after=st_after)

    # Verify conv over the window + T new tokens, split into repeat-interleaved q, k and v.
    gen = seeded(16)
    key_dim, value_dim, hd = 32, 64, 16
    C = 2 * key_dim + value_dim
    st = torch.randn(2, C, 4, generator=gen).to(torch.bfloat16)
    qkv = (torch.randn(2, 4, C, generator=gen) * 2).to(torch.bfloat16)
    w = (torch.randn(C, 1, 4, generator=gen) * 0.5).to(torch.bfloat16)
    ext, cq, ck, cv = ref.conv_step(st, qkv, w, key_dim, value_dim, hd, hd)
    out["conv_step"] = dict(state=st, qkv=qkv, w=w, key_dim=key_dim, value_dim=value_dim, head_dim=hd,
                            ext=ext, q=cq, k=ck, v=cv)

    # Output-gated RMSNorm.
    gen = seeded(17)
    norm = ref.GatedRMSNorm(128).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(128, generator=gen) + 0.5)
    x = (torch.randn(64, 128, generator=gen) * 2).to(torch.bfloat16)
    z = (torch.randn(64, 128, generator=gen) * 3).to(torch.bfloat16)
    with torch.no_grad():
        y = norm(x, z)
    out["gated_norm"] = dict(x=x, z=z, w=norm.weight.detach().clone(), y=y)

    # Delta gates with a validity mask.
    gen = seeded(18)
    b = (torch.randn(3, 5, 8, generator=gen) * 4).to(torch.bfloat16)
    a = (torch.randn(3, 5, 8, generator=gen) * 4).to(torch.bfloat16)
    dt_bias = torch.randn(8, generator=gen)
    rate = -torch.exp(torch.rand(8, generator=gen) * 2)
    valid = torch.rand(3, 5, generator=gen) < 0.7
    beta, gg = ref.delta_gates(b, a, dt_bias, rate, valid)
    out["delta_gates"] = dict(b=b, a=a, dt_bias=dt_bias, rate=rate, valid=valid, beta=beta, g=gg)

    # Rotary with per-row positions (3-D cos / sin), one NaN to propagate.
    gen = seeded(19)
    x = torch.randn(2, 5, 4, 128, generator=gen).to(torch.bfloat16)
    x[0, 1, 2, 7] = float("nan")
    pos = (torch.arange(5)[None] + torch.randint(0, 8000, (2, 1), generator=gen)).float()[..., None]
    freqs = pos * torch.logspace(0, -7, 32)
    cos, sin = freqs.cos(), freqs.sin()
    out["rotary"] = dict(x=x, cos=cos, sin=sin, y=ref.apply_rotary(x, cos, sin))

    # The drafter's cache writes: K candidate rows to shuffled cache rows, M mask rows to the tail.
    gen = seeded(20)
    B, K, M, H, D, nf, tail = 2, 3, 6, 4, 128, 32, 40
    k = torch.randn(B, K, H, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, K, H, D, generator=gen).to(torch.bfloat16)
    merged = torch.randn(B, M, 3 * H * D + 8, generator=gen).to(torch.bfloat16)
    qm, km, vm = (merged[..., i * H * D:(i + 1) * H * D].view(B, M, H, D) for i in range(3))
    f = torch.rand(B, K + M, 1, generator=gen) * 4000 * torch.logspace(0, -7, nf)
    cos, sin = f.cos(), f.sin()
    rows = torch.tensor([[2], [0]]).expand(B, K)
    positions = torch.randint(0, tail - K, (B, 1), generator=gen) + torch.arange(K)[None]
    k_cache = torch.randn(4, 64, H, D, generator=gen).to(torch.bfloat16)
    v_cache = torch.randn(4, 64, H, D, generator=gen).to(torch.bfloat16)
    kc, vc = k_cache.clone(), v_cache.clone()
    q_out = ref.rotate_into_cache(k, v, qm, km, vm, cos[:, :K], sin[:, :K], cos[:, K:], sin[:, K:], kc, vc, rows,
                                  positions, tail)
    out["rotate_into_cache"] = dict(k=k, v=v, merged=merged, cos=cos, sin=sin, rows=rows.contiguous(),
                                    positions=positions, k_cache=k_cache, v_cache=v_cache, tail=tail, K=K, M=M,
                                    q_out=q_out, k_cache_after=kc, v_cache_after=vc)

    # Decode attention (grouped heads, masked slices, one fully masked row) with the fp32
    # reference of model/triton_kernels_test.py:122-126 stored beside it.
    gen = seeded(21)
    B, R, H, Hkv, D, L = 2, 6, 8, 2, 128, 280
    q = torch.randn(B, R, H, D, generator=gen).to(torch.bfloat16)
    k_cache = torch.randn(3, 300, Hkv, D, generator=gen).to(torch.bfloat16)
    v_cache = torch.randn(3, 300, Hkv, D, generator=gen).to(torch.bfloat16)
    allowed = torch.rand(B, 1, R, L, generator=gen) < 0.6
    allowed[0, 0, 2] = False
    mask = torch.full((B, 1, R, L + 8), float("-inf"), dtype=torch.bfloat16)[..., :L].masked_fill_(allowed, 0.0)
    keys, values = (t[:B, :L].float().repeat_interleave(H // Hkv, dim=2) for t in (k_cache, v_cache))
    scores = torch.einsum("brhd,blhd->bhrl", q.float(), keys) * D ** -0.5 + mask.float()
    f32 = torch.einsum("bhrl,blhd->brhd", scores.softmax(-1).nan_to_num(0.0), values)
    out["decode_attention"] = dict(q=q, k_cache=k_cache, v_cache=v_cache, mask=mask, scale=D ** -0.5, o_f32=f32)

    for name, case in out.items():
        torch.save(case, os.path.join(HERE, f"{name}.pt"))
        print(name, {k: tuple(v.shape) if torch.is_tensor(v) else v for k, v in case.items()})


if __name__ == "__main__":
    main()
