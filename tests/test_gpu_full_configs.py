"""Parity at the full sizes of the benchmark configurations 2-4 (config 1's shape is covered in
test_gpu_chunk.py): the packed varlen prefill of 32 sequences, the decode step at 256 rows and the
block-4 verify at 128 rows, each with 32 value heads. Where a CPU oracle run of the whole case
would be slow the check is a size-independent property of the GPU path (packed == one call per
sequence, rollback by snapshot == recompute advance, bit for bit) plus the oracle on a part."""

import pytest
import torch

import jeeves_b200 as gdn
import oracle
from tests.helpers import cuda, gdn_inputs, maxabs, rel, same_bits

pytestmark = pytest.mark.gpu

H, HV = 16, 32
O_TOL = 2e-2          # bf16 outputs, max-abs
S_TOL_CHUNK = 1e-3    # fp32 state of the tensor-core prefill, relative
S_TOL_RECURRENT = 1e-5  # fp32 state of the CUDA-core recurrent kernel, relative


def test_config2_packed_varlen_full_size():
    """32 sequences of U{128..2048} tokens (seed 2, as the benchmark draws them) with random
    initial states: the packed call equals one call per sequence bit for bit, and the shortest
    and the longest sequence match the oracle."""
    lens = torch.randint(128, 2049, (32,), generator=torch.Generator().manual_seed(2)).tolist()
    T = sum(lens)
    q, k, v, g, beta, _ = gdn_inputs(41, 1, T, H, HV, state=False)
    h0 = torch.randn(len(lens), HV, 128, 128, generator=torch.Generator().manual_seed(42)) * 0.02
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    qc, kc, vc, gc, bc = cuda(q, k, v, g, beta)
    o, S = gdn.gated_delta_rule_chunk(qc, kc, vc, gc, bc, initial_state=h0.cuda(), output_final_state=True,
                                      cu_seqlens=cu.cuda())
    for n, (a, b) in enumerate(zip(cu[:-1].tolist(), cu[1:].tolist())):
        o1, S1 = gdn.gated_delta_rule_chunk(qc[:, a:b], kc[:, a:b], vc[:, a:b], gc[:, a:b], bc[:, a:b],
                                            initial_state=h0[n:n + 1].cuda(), output_final_state=True)
        assert same_bits(o[:, a:b], o1) and same_bits(S[n:n + 1], S1), n
    for n in (min(range(len(lens)), key=lambda i: lens[i]), max(range(len(lens)), key=lambda i: lens[i])):
        a, b = cu[n].item(), cu[n + 1].item()
        o_ref, S_ref = oracle.chunk_gated_delta_rule(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b],
                                                     initial_state=h0[n:n + 1], output_final_state=True)
        assert maxabs(o[:, a:b], o_ref) < O_TOL, n
        assert rel(S[n:n + 1], S_ref) < S_TOL_CHUNK, n


def test_config3_decode_step_full_size():
    """One decode token at 256 rows, the state updated in place, against the oracle."""
    B = 256
    q, k, v, g, beta, h0 = gdn_inputs(43, B, 1, H, HV, normalise=False)
    o_ref, S_ref = oracle.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=True)
    state = h0.cuda()
    o = gdn.fla_inplace.gated_delta_rule_step_inplace(*cuda(q, k, v, g, beta), state)
    assert maxabs(o, o_ref) < O_TOL
    assert rel(state, S_ref) < S_TOL_RECURRENT


def test_config4_verify_and_rollback_full_size():
    """Block-4 verify at 128 rows (5 tokens, 5 per-token state snapshots) against the oracle; the
    rollback to accepted lengths drawn from {1..5} equals the recompute advance bit for bit."""
    B, T = 128, 5
    q, k, v, g, beta, h0 = gdn_inputs(44, B, T, H, HV, normalise=False)
    o_ref, snaps_ref = oracle.verify_with_snapshots(q, k, v, g, beta, h0)
    qc, kc, vc, gc, bc, hc = cuda(q, k, v, g, beta, h0)
    o, snaps = gdn.gated_delta_rule_verify(qc, kc, vc, gc, bc, hc)
    assert maxabs(o, o_ref) < O_TOL
    for t in range(T):  # one token's snapshots at a time keeps the host copies small
        assert rel(snaps[:, t], snaps_ref[:, t]) < S_TOL_RECURRENT, t
    del snaps_ref
    accepted = torch.randint(1, T + 1, (B,), generator=torch.Generator().manual_seed(45)).cuda()
    rolled, advanced = hc.clone(), hc.clone()
    gdn.gated_delta_rule_rollback(rolled, snaps, accepted)
    gdn.gated_delta_rule_advance_inplace(kc, vc, gc, bc, advanced, accepted)
    assert same_bits(rolled, advanced)
