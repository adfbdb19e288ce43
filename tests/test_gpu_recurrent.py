"""GPU parity of the recurrent-form kernel (decode, verify + snapshots, rollback, fp32 mode)
against the CPU oracle and the reference's golden vectors."""

import pytest
import torch

import jeeves_b200 as gdn
import oracle
from tests.helpers import cuda, gdn_inputs, maxabs, rel, same_bits

pytestmark = pytest.mark.gpu

# Tolerances: outputs in bf16 within the north-star max-abs 2e-2; the state is fp32 math on
# CUDA cores, so it must match the fp32 oracle to 1e-5 relative (the fp32-mode bound).
O_TOL, S_TOL = 2e-2, 1e-5


def test_golden_recurrent_bf16(golden):
    c = golden("recurrent_bf16")
    q, k, v, g, beta, h0 = cuda(c["q"], c["k"], c["v"], c["g"], c["beta"], c["h0"])
    o, S = gdn.gated_delta_rule_step(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    assert maxabs(o, c["o"]) < O_TOL and rel(S, c["S"]) < S_TOL
    # bf16 outputs: nearly all elements round identically to the fp32 reference
    assert (o.cpu() != c["o"]).float().mean().item() < 0.02


def test_golden_config0_fp32_mode(golden):
    c = golden("chunk_cfg0")
    q, k, v, g, beta = cuda(c["q"], c["k"], c["v"], c["g"], c["beta"])
    o, S = gdn.gated_delta_rule_chunk(q, k, v, g, beta, output_final_state=True)
    assert o.dtype == torch.float32
    assert maxabs(o, c["o"]) < 1e-5 and rel(S, c["S"]) < 1e-5


@pytest.mark.parametrize("B,T,H,HV", [(1, 1, 2, 4), (4, 1, 16, 32), (3, 5, 4, 8), (2, 7, 2, 2), (64, 1, 16, 32)])
def test_step_matches_oracle(B, T, H, HV):
    q, k, v, g, beta, h0 = gdn_inputs(B * 100 + T, B, T, H, HV, normalise=False)
    o_ref, S_ref = oracle.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    o, S = gdn.gated_delta_rule_step(*cuda(q, k, v, g, beta), initial_state=h0.cuda(), output_final_state=True)
    assert maxabs(o, o_ref) < O_TOL and rel(S, S_ref) < S_TOL


def test_step_inplace_matches_oracle():
    q, k, v, g, beta, h0 = gdn_inputs(7, 8, 1, 16, 32, normalise=False)
    o_ref, S_ref = oracle.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    state = h0.cuda()
    o = gdn.fla_inplace.gated_delta_rule_step_inplace(*cuda(q, k, v, g, beta), state)
    assert maxabs(o, o_ref) < O_TOL and rel(state, S_ref) < S_TOL


def test_fp32_inputs_and_beta_dtypes():
    q, k, v, g, beta, h0 = gdn_inputs(8, 2, 9, 2, 4, dtype=torch.float32)
    o_ref, S_ref = oracle.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    o, S = gdn.gated_delta_rule_step(*cuda(q, k, v, g, beta), initial_state=h0.cuda())
    assert maxabs(o, o_ref) < 1e-5 and rel(S, S_ref) < 1e-5


def test_strided_inputs():
    q, k, v, g, beta, h0 = gdn_inputs(9, 2, 6, 4, 8, normalise=False)
    packed = torch.cat([q, k], dim=2).cuda()  # [B, T, 2H, D]: q and k are strided views
    qv, kv = packed[:, :, :4], packed[:, :, 4:]
    assert not qv.is_contiguous()
    o_ref, S_ref = oracle.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    o, S = gdn.gated_delta_rule_step(qv, kv, *cuda(v, g, beta), initial_state=h0.cuda())
    assert maxabs(o, o_ref) < O_TOL and rel(S, S_ref) < S_TOL


def test_golden_advance(golden):
    c = golden("advance")
    k, v, g, beta, h0, steps = cuda(c["k"], c["v"], c["g"], c["beta"], c["h0"], c["steps"])
    state = h0.clone()
    gdn.gated_delta_rule_advance_inplace(k, v, g, beta, state, steps)
    assert rel(state, c["S"]) < S_TOL
    for b, s in enumerate(c["steps"].tolist()):
        if s <= 0:
            assert same_bits(state[b], h0[b])


def test_advance_clamps_and_equals_prefix_run():
    B, T = 4, 5
    _, k, v, g, beta, h0 = gdn_inputs(10, B, T, 16, 32, normalise=False)
    k, v, g, beta, h0 = cuda(k, v, g, beta, h0)
    clamped, exact = h0.clone(), h0.clone()
    gdn.gated_delta_rule_advance_inplace(k, v, g, beta, clamped, torch.tensor([-5, T + 9, 0, 3], device="cuda"))
    gdn.gated_delta_rule_advance_inplace(k, v, g, beta, exact, torch.tensor([0, T, 0, 3], device="cuda", dtype=torch.int32))
    assert same_bits(clamped, exact)
    assert same_bits(clamped[0], h0[0]) and same_bits(clamped[2], h0[2])
    # advancing j tokens equals running the first j tokens (same kernel, same arithmetic)
    prefix, _ = None, None
    _, S3 = gdn.gated_delta_rule_step(torch.zeros_like(k[3:4, :3]), k[3:4, :3], v[3:4, :3], g[3:4, :3], beta[3:4, :3],
                                       initial_state=h0[3:4])
    assert rel(clamped[3:4], S3) < 1e-6


def test_advance_g_beta_zero_is_identity():
    _, k, v, g, beta, h0 = gdn_inputs(11, 3, 7, 2, 4, normalise=False)
    k, v, h0 = cuda(k, v, h0)
    state = h0.clone()
    gdn.gated_delta_rule_advance_inplace(k, v, torch.zeros(3, 7, 4, device="cuda"),
                                         torch.zeros(3, 7, 4, device="cuda", dtype=torch.bfloat16), state,
                                         torch.full((3,), 7, device="cuda"))
    assert same_bits(state, h0)


def test_verify_snapshots_and_rollback():
    B, T, H, HV = 6, 5, 16, 32
    q, k, v, g, beta, h0 = gdn_inputs(12, B, T, H, HV, normalise=False)
    o_ref, snaps_ref = oracle.verify_with_snapshots(q, k, v, g, beta, h0)
    qc, kc, vc, gc, bc, hc = cuda(q, k, v, g, beta, h0)
    o, snaps = gdn.gated_delta_rule_verify(qc, kc, vc, gc, bc, hc)
    assert maxabs(o, o_ref) < O_TOL and rel(snaps, snaps_ref) < S_TOL
    assert same_bits(hc, h0.cuda())  # verify reads the state, never writes it
    accepted = torch.tensor([1, 2, 3, 4, 5, 0], device="cuda")
    rolled, advanced = hc.clone(), hc.clone()
    gdn.gated_delta_rule_rollback(rolled, snaps, accepted)
    gdn.gated_delta_rule_advance_inplace(kc, vc, gc, bc, advanced, accepted)
    assert same_bits(rolled, advanced)
    # verify outputs equal the plain recurrent outputs
    o2, _ = gdn.gated_delta_rule_step(qc, kc, vc, gc, bc, initial_state=hc, output_final_state=False)
    assert same_bits(o, o2)


def test_resumed_equals_uninterrupted():
    B, T = 2, 9
    q, k, v, g, beta, h0 = cuda(*gdn_inputs(13, B, T, 2, 4, normalise=False))
    o_full, S_full = gdn.gated_delta_rule_step(q, k, v, g, beta, initial_state=h0)
    o_a, S_a = gdn.gated_delta_rule_step(q[:, :4], k[:, :4], v[:, :4], g[:, :4], beta[:, :4], initial_state=h0)
    o_b, S_b = gdn.gated_delta_rule_step(q[:, 4:], k[:, 4:], v[:, 4:], g[:, 4:], beta[:, 4:], initial_state=S_a)
    assert same_bits(torch.cat([o_a, o_b], 1), o_full) and same_bits(S_b, S_full)


@pytest.mark.parametrize("T", [2, 3, 5])
def test_final_state_equals_advance_by_all_tokens_and_snapshots(T):
    """The final state of a recurrent call, the advance by all T tokens and the last per-token
    snapshot are the same bits, and advancing by j equals snapshot j - 1 (the property the
    reference pins between its advance kernel and fla's recurrent one)."""
    B = 6
    q, k, v, g, beta, h0 = cuda(*gdn_inputs(90 + T, B, T, 16, 32, normalise=False))
    _, final = gdn.gated_delta_rule_step(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    adv = h0.clone()
    gdn.gated_delta_rule_advance_inplace(k, v, g, beta, adv, torch.full((B,), T, device="cuda"))
    _, snaps = gdn.gated_delta_rule_verify(q, k, v, g, beta, h0)
    assert same_bits(final, adv) and same_bits(final, snaps[:, T - 1])
    steps = torch.arange(B, device="cuda") % (T + 1)
    part = h0.clone()
    gdn.gated_delta_rule_advance_inplace(k, v, g, beta, part, steps)
    for b in range(B):
        j = int(steps[b])
        assert same_bits(part[b], h0[b] if j == 0 else snaps[b, j - 1]), b


def test_varlen_recurrent_equals_per_sequence():
    lens = [3, 0, 11, 6]
    T = sum(lens)
    q, k, v, g, beta, _ = gdn_inputs(14, 1, T, 2, 4, normalise=False)
    h0 = torch.randn(len(lens), 4, 128, 128) * 0.02
    cu = torch.tensor([0, 3, 3, 14, 20], dtype=torch.int32)
    o, S = gdn.gated_delta_rule_step(*cuda(q, k, v, g, beta), initial_state=h0.cuda(), cu_seqlens=cu.cuda())
    for i in range(len(lens)):
        s, e = int(cu[i]), int(cu[i + 1])
        o_r, S_r = oracle.recurrent_gated_delta_rule(q[:, s:e], k[:, s:e], v[:, s:e], g[:, s:e], beta[:, s:e],
                                                     initial_state=h0[i:i + 1], output_final_state=True)
        if e > s:
            assert maxabs(o[:, s:e], o_r) < O_TOL
        assert rel(S[i:i + 1], S_r) < S_TOL


def test_errors_follow_reference_convention():
    q, k, v, g, beta, h0 = cuda(*gdn_inputs(15, 2, 3, 2, 4))
    with pytest.raises(ValueError):
        gdn.gated_delta_rule_step(q.half(), k.half(), v.half(), g, beta)
    with pytest.raises(ValueError, match="state"):
        gdn.gated_delta_rule_advance_inplace(k, v, g, beta, h0.transpose(2, 3), torch.ones(2, device="cuda"))
    with pytest.raises(ValueError, match="steps"):
        gdn.gated_delta_rule_advance_inplace(k, v, g, beta, h0.clone(), torch.ones(2, device="cuda"))


@pytest.mark.parametrize("T", [2, 5, 8])
@pytest.mark.parametrize("H,HV", [(2, 4), (16, 32)])
def test_outputs_only_call_against_float64_and_the_state_writing_call(T, H, HV):
    """Outputs of a short block without a state write: within the output bound of the float64
    recurrence, the same bits as the call that also writes the final state, state untouched."""
    B = 3
    q, k, v, g, beta, h0 = gdn_inputs(40 + T + HV, B, T, H, HV, normalise=False)
    o64, _ = oracle.exact_recurrence_f64(q, k, v, g, beta, h0)
    qc, kc, vc, gc, bc, hc = cuda(q, k, v, g, beta, h0)
    o, none = gdn.gated_delta_rule_step(qc, kc, vc, gc, bc, initial_state=hc, output_final_state=False)
    o_seq, _ = gdn.gated_delta_rule_step(qc, kc, vc, gc, bc, initial_state=hc, output_final_state=True)
    assert none is None and same_bits(hc, h0.cuda())
    assert maxabs(o, o64) < O_TOL and same_bits(o, o_seq)


def test_outputs_only_call_with_gates_equals_gates_then_call():
    """The gate-fused form of an outputs-only call equals delta_gates followed by the plain call."""
    gen = torch.Generator().manual_seed(77)
    B, T, H, HV = 4, 5, 16, 32
    q, k, v, _, _, h0 = cuda(*gdn_inputs(78, B, T, H, HV, normalise=False))
    b = torch.randn(B, T, HV, generator=gen).to(torch.bfloat16).cuda()
    a = torch.randn(B, T, HV, generator=gen).to(torch.bfloat16).cuda()
    dt = torch.rand(HV, generator=gen).cuda()
    rate = (-torch.rand(HV, generator=gen) * 4).cuda()
    beta, g = gdn.delta_gates(b, a, dt, rate)
    o_ref, _ = gdn.gated_delta_rule_step(q, k, v, g, beta, initial_state=h0, output_final_state=False)
    o, _ = gdn.gated_delta_rule_step_gates(q, k, v, b, a, dt, rate, initial_state=h0, output_final_state=False)
    assert same_bits(o, o_ref)


@pytest.mark.parametrize("T", [1, 5, 8])
@pytest.mark.parametrize("snapshots", [False, True])
@pytest.mark.parametrize("B", [16, 64])
def test_batched_rows_equal_the_same_rows_packed_bitwise(T, snapshots, B):
    """A batch of rows and the same rows packed with cu_seqlens give the same outputs, final states
    and snapshots, bit for bit. With T = 1 the batched call runs the one-token tile (8 state rows a
    thread) and the packed call the multi-token tile (16 rows a thread), below and at the 2048
    (row, head) pairs where the column slices widen."""
    H, HV = 16, 32
    q, k, v, g, beta, h0 = cuda(*gdn_inputs(300 + T, B, T, H, HV, normalise=False))
    if snapshots:
        o, snaps = gdn.gated_delta_rule_verify(q, k, v, g, beta, h0)
    else:
        o, S = gdn.gated_delta_rule_step(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    cu = torch.arange(0, B * T + 1, T, dtype=torch.int32, device="cuda")
    pack = lambda t: t.reshape(1, B * T, *t.shape[2:])
    o_p, S_p = gdn.gated_delta_rule_step(pack(q), pack(k), pack(v), pack(g), pack(beta), initial_state=h0,
                                         output_final_state=True, cu_seqlens=cu)
    assert same_bits(o, o_p.view(B, T, HV, 128))
    if snapshots:
        assert same_bits(snaps[:, T - 1], S_p)
    else:
        assert same_bits(S, S_p)


def _f64_verify(q, k, v, g, beta, h0, scale=128 ** -0.5):
    """Outputs, update vectors and per-token states of the token recurrence in float64 (the
    oracle's recurrence, model/model.py:221-239, with the update vector kept)."""
    q, k, v, g, beta, S = (x.detach().double().cpu() for x in (q, k, v, g, beta, h0))
    B, T, H, _ = q.shape
    HV = v.shape[2]
    q = q.repeat_interleave(HV // H, dim=2)
    k = k.repeat_interleave(HV // H, dim=2)
    q = q / torch.sqrt((q * q).sum(-1, keepdim=True) + 1e-6) * scale
    k = k / torch.sqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    o, d, states = [], [], []
    for t in range(T):
        S = S * torch.exp(g[:, t])[..., None, None]
        dt = beta[:, t, :, None] * (v[:, t] - torch.einsum("bhk,bhkv->bhv", k[:, t], S))
        S = S + torch.einsum("bhk,bhv->bhkv", k[:, t], dt)
        o.append(torch.einsum("bhk,bhkv->bhv", q[:, t], S))
        d.append(dt)
        states.append(S)
    return torch.stack(o, 1), torch.stack(d, 1), torch.stack(states, 1)


@pytest.mark.parametrize("T", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("B,H,HV", [(6, 16, 32), (3, 2, 4), (37, 4, 4)])
def test_verify_deltas_block_against_float64(T, B, H, HV):
    """bf16 rows and T <= 8: the tensor-core block (the state as two bf16 parts, the recurrence
    unrolled over the Gram products). Outputs within the bf16 bound, update vectors and the
    committed state within the fp32 state bound of the float64 recurrence."""
    q, k, v, g, beta, h0 = gdn_inputs(500 + 10 * T + B, B, T, H, HV, normalise=False)
    o_ref, d_ref, st_ref = _f64_verify(q, k, v, g, beta, h0)
    qc, kc, vc, gc, bc, hc = cuda(q, k, v, g, beta, h0)
    o, deltas = gdn.gated_delta_rule_verify_deltas(qc, kc, vc, gc, bc, hc)
    assert same_bits(hc, h0.cuda())  # read, not written
    assert maxabs(o, o_ref) < O_TOL
    assert rel(deltas, d_ref) < S_TOL
    accepted = torch.arange(B) % (T + 2) - 1  # -1 .. T + 1: clamped to 0 .. T
    state = hc.clone()
    gdn.gated_delta_rule_delta_commit(kc, gc, deltas, state, accepted.cuda())
    j = accepted.clamp(0, T)
    want = torch.stack([h0[b].double() if j[b] == 0 else st_ref[b, j[b] - 1] for b in range(B)])
    assert rel(state, want) < S_TOL
    keep = (j == 0).cuda()
    assert same_bits(state[keep], hc[keep])


@pytest.mark.parametrize("B", [6, 64])
def test_verify_deltas_fallback_and_delta_commit_equal_the_step_and_the_advance(B):
    """fp32 rows (or T > 8, or no initial state) run the recurrent kernel: its outputs are the
    plain step's, and the delta commit leaves the advance's state, bit for bit, for every
    accepted count (clamped to [0, T])."""
    T, H, HV = 5, 16, 32
    q, k, v, g, beta, h0 = cuda(*gdn_inputs(400 + B, B, T, H, HV, dtype=torch.float32, normalise=False))
    o_ref, _ = gdn.gated_delta_rule_step(q, k, v, g, beta, initial_state=h0, output_final_state=False)
    o, deltas = gdn.gated_delta_rule_verify_deltas(q, k, v, g, beta, h0)
    assert same_bits(o, o_ref) and deltas.shape == (B, T, HV, 128)
    accepted = torch.tensor([(-1, 0, 1, 2, 3, 4, 5, 9)[i % 8] for i in range(B)], device="cuda")
    adv, com = h0.clone(), h0.clone()
    gdn.gated_delta_rule_advance_inplace(k, v, g, beta, adv, accepted)
    gdn.gated_delta_rule_delta_commit(k, g, deltas, com, accepted)
    assert same_bits(com, adv)


@pytest.mark.parametrize("B", [6, 64])
def test_verify_deltas_block_equals_the_step_to_rounding(B):
    """The block's outputs and the delta commit's state against the recurrent kernel's step and
    advance on the same bf16 inputs."""
    T, H, HV = 5, 16, 32
    q, k, v, g, beta, h0 = cuda(*gdn_inputs(410 + B, B, T, H, HV, normalise=False))
    o_ref, _ = gdn.gated_delta_rule_step(q, k, v, g, beta, initial_state=h0, output_final_state=False)
    o, deltas = gdn.gated_delta_rule_verify_deltas(q, k, v, g, beta, h0)
    assert maxabs(o, o_ref) < 1e-2
    accepted = torch.tensor([(0, 1, 2, 3, 4, 5)[i % 6] for i in range(B)], device="cuda")
    adv, com = h0.clone(), h0.clone()
    gdn.gated_delta_rule_advance_inplace(k, v, g, beta, adv, accepted)
    gdn.gated_delta_rule_delta_commit(k, g, deltas, com, accepted)
    assert rel(com, adv) < 2e-6


def test_delta_commit_checks_its_arguments():
    B, T, H, HV = 2, 3, 2, 4
    q, k, v, g, beta, h0 = cuda(*gdn_inputs(450, B, T, H, HV, normalise=False))
    _, deltas = gdn.gated_delta_rule_verify_deltas(q, k, v, g, beta, h0)
    acc = torch.tensor([1, 2], device="cuda")
    with pytest.raises(ValueError):
        gdn.gated_delta_rule_delta_commit(k, g, deltas[:, :2], h0.clone(), acc)
    with pytest.raises(ValueError):
        gdn.gated_delta_rule_delta_commit(k, g, deltas, h0[:1].clone(), acc)
    with pytest.raises(ValueError):
        gdn.gated_delta_rule_delta_commit(k, g, deltas, h0.clone(), acc.float())


@pytest.mark.parametrize("L,B", [(3, 5), (70, 1)])
def test_delta_commit_layers_equals_the_one_layer_commits(L, B):
    """The commit of many layers in one launch (70 layers: two launches of at most 64) leaves every
    layer's state as the one-layer commit does, bit for bit; overlapping states are refused."""
    T, H, HV = 5, 2, 4
    ks, gs, ds, states, want = [], [], [], [], []
    accepted = torch.tensor([(0, 1, 3, 5, 9)[i % 5] for i in range(B)], device="cuda")
    for l in range(L):
        q, k, v, g, beta, h0 = cuda(*gdn_inputs(700 + l, B, T, H, HV, normalise=False))
        _, deltas = gdn.gated_delta_rule_verify_deltas(q, k, v, g, beta, h0)
        one = h0.clone()
        gdn.gated_delta_rule_delta_commit(k, g, deltas, one, accepted)
        ks.append(k); gs.append(g); ds.append(deltas); states.append(h0); want.append(one)
    gdn.gated_delta_rule_delta_commit_layers(ks, gs, ds, states, accepted)
    for st, one in zip(states, want):
        assert same_bits(st, one)
    with pytest.raises(ValueError):
        gdn.gated_delta_rule_delta_commit_layers(ks[:2], gs[:2], ds[:2], [states[0], states[0]], accepted)


@pytest.mark.parametrize("T,B", [(1, 6), (5, 37), (8, 64)])
def test_block_verify_with_fused_gated_norm_equals_the_two_calls(T, B):
    """The gated norm in the block verify's drain gives the standalone norm of the block's outputs
    bit for bit, update vectors included."""
    H, HV = 4, 8
    q, k, v, g, beta, h0 = cuda(*gdn_inputs(600 + T, B, T, H, HV, normalise=False))
    gen = torch.Generator().manual_seed(601)
    z = (torch.randn(B, T, HV, 128, generator=gen) * 3).to(torch.bfloat16)
    z.view(-1)[::97] = 0
    z.view(-1)[5::101] = -120.0
    z = z.cuda()
    nw = (torch.rand(128, generator=gen) + 0.5).to(torch.bfloat16).cuda()
    o, d_ref = gdn.gated_delta_rule_verify_deltas(q, k, v, g, beta, h0)
    y_ref = gdn.gated_rms_norm(o.view(-1, 128), z.view(-1, 128), nw).view(o.shape)
    y, d = gdn.gated_delta_rule_verify_deltas_gated_norm(q, k, v, g, beta, h0, z, nw)
    assert same_bits(y, y_ref) and same_bits(d, d_ref)
