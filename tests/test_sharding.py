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


def _guard_worker(rank, world, port, mode, result_dir):
    """Four steps; rank 1 fails in step 2 (raises, or exits without a word). Rank 0 must learn of it
    at its next step boundary, before launching step 3, and record what it saw."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    guard = sharding.StepGuard(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=3.0)
    seen = "no failure seen"
    try:
        for step in range(4):
            def work():
                if rank == 1 and step == 2:
                    if mode == "exit":
                        os._exit(3)  # leaves between steps, nothing in flight, no message
                    raise RuntimeError("planted failure on rank 1")
                return step
            guard.run(step, work)
    except sharding.PeerFailure as e:
        seen = f"PeerFailure: {e}"
    except RuntimeError as e:
        seen = f"own error: {e}"
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as fh:
        fh.write(seen)


@pytest.mark.parametrize("mode", ["raise", "exit"])
def test_step_guard_reports_a_failed_peer_without_hanging(tmp_path, mode):
    """Two gloo ranks as separate processes (as torchrun starts them). The surviving rank raises
    PeerFailure at the next step boundary (the failed rank's message, or the deadline when it exits
    without one), and every process ends within the time limit."""
    import subprocess
    import sys
    import time

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    port = _free_port()
    code = ("import sys; sys.path.insert(0, {root!r}); from tests.test_sharding import _guard_worker; "
            "_guard_worker({rank}, 2, {port}, {mode!r}, {out!r})")
    t0 = time.monotonic()
    procs = [subprocess.Popen([sys.executable, "-c", code.format(root=root, rank=r, port=port, mode=mode,
                                                                out=str(tmp_path))],
                              stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL) for r in range(2)]
    try:
        codes = [p.wait(timeout=120) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert time.monotonic() - t0 < 100
    seen0 = (tmp_path / "rank0.txt").read_text()
    assert seen0.startswith("PeerFailure"), seen0
    if mode == "raise":
        assert "planted failure" in seen0
        assert (tmp_path / "rank1.txt").read_text().startswith("own error")
    else:
        assert "did not reach step 3" in seen0
        assert codes[1] == 3 and not (tmp_path / "rank1.txt").exists()
