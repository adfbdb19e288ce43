"""GPU parity of the verify branch of a delta layer (config 4): the layer step against the
composition of the oracle's ops (conv over the conv-state window, recurrent outputs from the state,
gated norm), the commit by recompute and by snapshot against the oracle's advance, and the
conv-state commit against the engine's gather (inference/engine.py:473-474)."""

import pytest
import torch

import jeeves_b200 as gdn
import oracle
from tests.helpers import maxabs, rel, same_bits

pytestmark = pytest.mark.gpu


def verify_inputs(seed, B, T, H, HV, taps):
    gen = torch.Generator().manual_seed(seed)
    C = 2 * H * 128 + HV * 128
    qkv = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
    cs = torch.randn(B, C, taps, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C, 4, generator=gen) * 0.5).to(torch.bfloat16)
    g = -torch.exp(torch.randn(B, T, HV, generator=gen) * 0.5 - 3.0)
    beta = torch.sigmoid(torch.randn(B, T, HV, generator=gen)).to(torch.bfloat16)
    state = torch.randn(B, HV, 128, 128, generator=gen) * 0.02
    z = torch.randn(B, T, HV, 128, generator=gen).to(torch.bfloat16)
    nw = (torch.rand(128, generator=gen) + 0.5).to(torch.bfloat16)
    accepted = torch.randint(0, T + 1, (B,), generator=gen)
    return qkv, cs, w, g, beta, state, z, nw, accepted


@pytest.mark.parametrize("B,T,H,HV,taps", [(4, 5, 16, 32, 3), (3, 5, 2, 4, 4), (2, 2, 2, 4, 3)])
@pytest.mark.parametrize("design", ["recompute", "snapshots", "deltas"])
def test_verify_layer_matches_oracle_composition(B, T, H, HV, taps, design):
    qkv, cs, w, g, beta, state, z, nw, accepted = verify_inputs(B * 100 + T * 10 + taps, B, T, H, HV, taps)
    C = qkv.shape[-1]
    # oracle: conv over the window, outputs from the state, gated norm; commit = advance by the
    # accepted tokens and the conv window after them
    ext_ref, q, k, v = oracle.conv_step(cs, qkv, w, H * 128, HV * 128, 128, 128)
    o_ref, _ = oracle.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=state)
    y_ref = oracle.gated_rms_norm(o_ref.reshape(-1, 128), z.reshape(-1, 128), nw).reshape(B, T, HV, 128)
    S_ref = oracle.advance_gated_delta_rule(k, v, g, beta, state, accepted)
    cols = accepted.clamp(0, T)[:, None, None] + torch.arange(taps)[None, None]
    cs_ref = torch.gather(ext_ref, 2, cols.expand(B, C, taps))

    d = dict(qkv=qkv.cuda(), cs=cs.cuda(), w=w.cuda(), g=g.cuda(), beta=beta.cuda(), state=state.cuda(), z=z.cuda(),
             nw=nw.cuda())
    ext = torch.empty(B, C, taps + T, dtype=torch.bfloat16, device="cuda")
    snaps = torch.empty(B, T, HV, 128, 128, device="cuda") if design == "snapshots" else None
    deltas = torch.empty(B, T, HV, 128, device="cuda") if design == "deltas" else None
    y, pending = gdn.verify_layer_step(d["qkv"], d["cs"], d["w"], d["g"], d["beta"], d["state"], d["z"], d["nw"], H,
                                       ext_out=ext, snapshots=snaps, deltas=deltas)
    assert same_bits(ext, ext_ref)
    assert same_bits(d["state"], state)  # the verify reads the state only
    assert maxabs(y, y_ref) < 2e-2
    assert (y.cpu() != y_ref).float().mean().item() < 0.02
    gdn.verify_layer_commit(pending, d["state"], accepted.cuda(), ext=ext, conv_state=d["cs"])
    assert rel(d["state"], S_ref) < 1e-5
    unchanged = accepted == 0
    assert same_bits(d["state"].cpu()[unchanged], state[unchanged])
    assert same_bits(d["cs"], cs_ref)


def test_commit_designs_agree():
    """The snapshot rollback and the recompute advance leave the same state bit for bit and their
    verifies give the same outputs; the kept-update-vector design (the tensor-core block for these
    bf16 rows) agrees with them to fp32 rounding."""
    B, T, H, HV, taps = 6, 5, 2, 4, 3
    qkv, cs, w, g, beta, state, z, nw, _ = verify_inputs(7, B, T, H, HV, taps)
    accepted = torch.tensor([1, 2, 3, 4, 5, 0]).cuda()
    results, ys = [], []
    designs = ({}, {"snapshots": torch.empty(B, T, HV, 128, 128, device="cuda")},
               {"deltas": torch.empty(B, T, HV, 128, device="cuda")})
    for extra in designs:
        st = state.cuda()
        y, pending = gdn.verify_layer_step(qkv.cuda(), cs.cuda(), w.cuda(), g.cuda(), beta.cuda(), st, z.cuda(),
                                           nw.cuda(), H, **extra)
        gdn.verify_layer_commit(pending, st, accepted)
        results.append(st)
        ys.append(y)
    assert same_bits(results[0], results[1]) and same_bits(ys[0], ys[1])
    assert rel(results[2], results[0]) < 2e-6 and maxabs(ys[2], ys[0]) < 2e-2


@pytest.mark.parametrize("B,T,taps,qkv_pad", [(16, 5, 3, 0), (72, 5, 3, 0), (5, 8, 4, 0), (3, 1, 3, 0), (4, 5, 3, 1)])
def test_verify_layer_one_call_equals_the_separate_calls(B, T, taps, qkv_pad):
    """The kept-update-vector verify layer as one library call (the conv step with the block verify
    as its programmatic dependent; the gated norm in the block's drain below 2,048 states, after it
    from there: B = 72 with 32 value heads) gives the conv step followed by the block verify and the
    standalone norm bit for bit. qkv_pad = 1 gives the rows an odd stride, so the conv runs its
    per-channel form, which does not release the block early."""
    H, HV = 16, 32
    qkv, cs, w, g, beta, state, z, nw, _ = verify_inputs(800 + B + T, B, T, H, HV, taps)
    C = qkv.shape[-1]
    padded = torch.zeros(B, T, C + qkv_pad, dtype=torch.bfloat16)
    padded[..., :C] = qkv
    d = dict(qkv=padded.cuda()[..., :C], cs=cs.cuda(), w=w.cuda(), g=g.cuda(), beta=beta.cuda(), state=state.cuda(),
             z=z.cuda(), nw=nw.cuda())
    ext_ref, q, k, v = gdn.conv_step(d["cs"], d["qkv"], d["w"], H * 128, HV * 128, 128, 128)
    o, d_ref = gdn.gated_delta_rule_verify_deltas(q, k, v, d["g"], d["beta"], d["state"])
    y_ref = gdn.gated_rms_norm(o.view(-1, 128), d["z"].view(-1, 128), d["nw"]).view(o.shape)
    ext = torch.empty_like(ext_ref)
    deltas = torch.empty(B, T, HV, 128, device="cuda")
    y, pending = gdn.verify_layer_step(d["qkv"], d["cs"], d["w"], d["g"], d["beta"], d["state"], d["z"], d["nw"], H,
                                       ext_out=ext, deltas=deltas)
    assert same_bits(ext, ext_ref) and same_bits(y, y_ref) and same_bits(deltas, d_ref)
    assert same_bits(pending[0], k) and same_bits(pending[1], v) and pending[5] is deltas
    assert same_bits(d["state"], state)  # read, not written


def test_verify_layers_commit_equals_the_layer_commits():
    """One launch committing every layer's kept update vectors leaves each state as the one-layer
    commit does, bit for bit; layers of other designs in the same list are committed one by one."""
    B, T, H, HV, taps, L = 6, 5, 2, 4, 3, 3
    accepted = torch.tensor([1, 2, 3, 4, 5, 0]).cuda()
    pendings, states, want = [], [], []
    for l in range(L):
        qkv, cs, w, g, beta, state, z, nw, _ = verify_inputs(900 + l, B, T, H, HV, taps)
        extra = {"snapshots": torch.empty(B, T, HV, 128, 128, device="cuda")} if l == 1 else \
            {"deltas": torch.empty(B, T, HV, 128, device="cuda")}
        st = state.cuda()
        _, p = gdn.verify_layer_step(qkv.cuda(), cs.cuda(), w.cuda(), g.cuda(), beta.cuda(), st, z.cuda(), nw.cuda(),
                                     H, **extra)
        one = st.clone()
        gdn.verify_layer_commit(p, one, accepted)
        pendings.append(p)
        states.append(st)
        want.append(one)
    gdn.verify_layers_commit(pendings, states, accepted)
    for st, one in zip(states, want):
        assert same_bits(st, one)


def test_conv_state_commit_over_stacked_layers_matches_gather():
    """One launch over the engine's stacked [layers, max_rows, C, taps] conv states, on the
    leading B rows (strided slices), equals torch.gather of the ext windows."""
    layers, R, B, C, taps, T = 3, 5, 4, 256, 4, 5
    gen = torch.Generator().manual_seed(11)
    ext = torch.randn(layers, R, C, taps + T, generator=gen).to(torch.bfloat16).cuda()
    states = torch.randn(layers, R, C, taps, generator=gen).to(torch.bfloat16).cuda()
    accepted = torch.tensor([0, 5, 2, 9])  # 9 clamps to T
    before = states.clone()
    gdn.conv_state_commit(ext[:, :B], states[:, :B], accepted.cuda())
    cols = (accepted.clamp(0, T)[:, None] + torch.arange(taps)[None])[None, :, None, :].expand(layers, B, C, taps)
    want = torch.gather(ext[:, :B].cpu(), 3, cols)
    assert same_bits(states[:, :B], want)
    assert same_bits(states[:, B:], before[:, B:])  # rows past B untouched


@pytest.mark.parametrize("taps,T", [(3, 5), (4, 4)])
def test_conv_state_commit_16_byte_form_matches_gather(taps, T):
    """The engine's shape (taps + T = 8 values a channel, one 16-byte vector): every clamped
    acceptance, over strided layer and row slices of the stacked states, equals torch.gather."""
    layers, R, B, C = 3, 9, 7, 8192
    gen = torch.Generator().manual_seed(12 + taps)
    ext = torch.randn(layers, R, C, taps + T, generator=gen).to(torch.bfloat16).cuda()
    states = torch.randn(layers + 1, R, C, taps, generator=gen).to(torch.bfloat16).cuda()
    accepted = torch.tensor([-2, 0, 1, 2, 3, T, T + 7])
    before = states.clone()
    gdn.conv_state_commit(ext[:, :B], states[1:, :B], accepted.cuda())
    cols = (accepted.clamp(0, T)[:, None] + torch.arange(taps)[None])[None, :, None, :].expand(layers, B, C, taps)
    want = torch.gather(ext[:, :B].cpu(), 3, cols)
    assert same_bits(states[1:, :B], want)
    assert same_bits(states[0], before[0]) and same_bits(states[1:, B:], before[1:, B:])


def test_conv_state_commit_rejects_mismatched_shapes():
    ext = torch.zeros(2, 64, 7, dtype=torch.bfloat16, device="cuda")
    st = torch.zeros(2, 64, 3, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        gdn.conv_state_commit(ext, st, torch.zeros(3, dtype=torch.int64, device="cuda"))
    with pytest.raises(ValueError):
        gdn.conv_state_commit(ext.float(), st, torch.zeros(2, dtype=torch.int64, device="cuda"))
