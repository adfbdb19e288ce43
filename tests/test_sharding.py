"""CPU tests of the multi-GPU split: shard bookkeeping, and a 2-rank gloo run whose sharded
results (computed per rank with the CPU oracle) equal the single-process results."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from jeeves_b200 import sharding
from tests.helpers import gdn_inputs


def test_row_shard_covers_every_row_once():
    for n in (0, 1, 7, 256, 257):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                start, count = sharding.row_shard(n, r, world)
                seen.extend(range(start, start + count))
            assert seen == list(range(n))


def test_balance_sequences_is_a_partition_and_balanced():
    lengths = torch.randint(128, 2049, (32,), generator=torch.Generator().manual_seed(2)).tolist()
    for world in (1, 2, 4, 8):
        parts = sharding.balance_sequences(lengths, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(32))
        loads = [sum(lengths[i] for i in p) for p in parts]
        # LPT is within max(length) of perfect balance
        assert max(loads) - min(loads) <= max(lengths)
        for p in parts:
            assert p == sorted(p)


def test_gather_packed_and_local_cu_seqlens():
    lengths = [3, 0, 5, 2]
    cu = sharding.cu_seqlens_of(lengths)
    x = torch.arange(10).view(1, 10)
    assert sharding.gather_packed(x, cu, [2, 0]).tolist() == [[3, 4, 5, 6, 7, 0, 1, 2]]
    idx, local, lcu = sharding.local_varlen(lengths, 0, 2)
    assert lcu.tolist()[-1] == sum(local)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lengths = [70, 5, 130, 64, 1, 99]
        q, k, v, g, beta, _ = gdn_inputs(3, 1, sum(lengths), 2, 4)
        h0 = torch.randn(len(lengths), 4, 128, 128, generator=torch.Generator().manual_seed(4)) * 0.02
        cu = sharding.cu_seqlens_of(lengths)
        idx, local, lcu = sharding.local_varlen(lengths, rank, world)
        pick = lambda t: sharding.gather_packed(t, cu, idx)
        o, S = oracle.chunk_gated_delta_rule_varlen(pick(q), pick(k), pick(v), pick(g), pick(beta), lcu,
                                                    initial_state=h0[idx], output_final_state=True)
        gathered = [None] * world
        dist.all_gather_object(gathered, (idx, local, o, S))  # results only; the data path has no collective
        if rank == 0:
            full_o, full_S = oracle.chunk_gated_delta_rule_varlen(q, k, v, g, beta, cu, initial_state=h0,
                                                                  output_final_state=True)
            ok = True
            cuv = cu.tolist()
            for ids, lens, o_r, S_r in gathered:
                off = 0
                for j, i in enumerate(ids):
                    ok &= torch.equal(o_r[:, off:off + lens[j]], full_o[:, cuv[i]:cuv[i + 1]])
                    ok &= torch.equal(S_r[j], full_S[i])
                    off += lens[j]
            torch.save(bool(ok), result_path)
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_varlen_shards_equal_one_process(tmp_path):
    path = str(tmp_path / "ok.pt")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    assert torch.load(path) is True
