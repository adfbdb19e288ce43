"""The benchmark's algorithmic work counts, recomputed here from the shapes (CPU only).

The roofline fractions that `bench.py` prints divide these counts by measured times, so each is
derived again below from first principles: every input read once, every output written once,
q and k at the key heads (never repeated to the value heads), states in fp32.
"""

import bench

D, H, HV = 128, 16, 32
C = 2 * H * D + HV * D          # conv channels of the 9B-shaped layer (q | k | v)
STATE = HV * D * D * 4          # one sequence's recurrent state, fp32


def test_prefill_bytes_config1():
    # per token: q and k (bf16, key heads), v and o (bf16, value heads), g (fp32) and beta (bf16)
    per_token = 2 * H * D * 2 + 2 * HV * D * 2 + HV * (4 + 2)
    assert per_token == 24_768
    # config 1 writes the final state only; config 2 also reads each sequence's initial state
    assert bench.prefill_core_bytes(4096) == 4096 * per_token + STATE == 103_546_880
    assert bench.prefill_core_bytes(1000, n_seq=3, with_h0=True) == 1000 * per_token + 3 * 2 * STATE


def test_prefill_flops_per_token_and_head():
    # per chunk of 64 tokens and value head: K K^T and Q K^T (64 x 64 x 128 each), W = X K and
    # U = X V (64 x 64 x 128), P' VN (64 x 64 x 128), W S and Q S (64 x 128 x 128), K^T VN
    # (128 x 64 x 128); two flops per multiply-add
    mac = 5 * 64 * 64 * 128 + 3 * 64 * 128 * 128
    assert 2 * mac // 64 == 180_224
    assert bench.prefill_flops(4096) == 4096 * HV * 180_224


def test_verify_unit_bytes_per_design():
    T, taps = 5, 3
    conv = C * taps * 2 * 3 + C * (taps + T) * 2      # conv state read and rolled forward, ext window
    io = T * C * 2 + T * HV * 6 + 2 * T * HV * D * 2  # qkv, g / beta, z in and y out
    kept_kv = 2 * T * (H * D + HV * D) * 2            # k and v written by the verify, read by the commit
    kept_deltas = 2 * T * H * D * 2 + 2 * T * HV * D * 4
    assert bench.verify_unit_bytes("recompute") == 3 * STATE + conv + io + kept_kv == 6_857_664
    assert bench.verify_unit_bytes("deltas") == 3 * STATE + conv + io + kept_deltas == 6_939_584
    # snapshots: the state read once and T per-token states written; the rollback copy is not counted
    assert bench.verify_unit_bytes("snapshots") == (1 + T) * STATE + conv + io == 13_026_240


def test_decode_and_projection_counts_quoted_in_the_bench_line():
    # decode, per (sequence, layer, token): state read and written, conv state read and written,
    # qkv in, g / beta, z in and y out
    decode = 2 * STATE + 2 * C * 3 * 2 + C * 2 + HV * 6 + 2 * HV * D * 2
    assert decode == 4_325_568
    # merged projection of the 9B shape: 4096 tokens x 4096 -> 12,352 output channels
    assert bench.IN_PROJ_N == C + HV * D + 2 * HV == 12_352
    assert 2 * 4096 * 4096 * bench.IN_PROJ_N == 414_464_344_064
