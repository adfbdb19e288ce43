"""Splitting the gated-delta hot path across GPUs (one process per GPU, no collective).

Sequences are independent in every workload of the path, so each rank owns a subset of them
and runs the kernels on its own GPU; nothing is exchanged on the data path. Batched decode and
verify split rows contiguously; a packed varlen prefill balances its sequences by token count
(longest first onto the least-loaded rank) and repacks each rank's sequences with their own
``cu_seqlens``. A single long sequence does not split: each GPU then serves its own sequences
(replicas).
"""

from __future__ import annotations

import heapq

import torch


def row_shard(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous ``(start, count)`` of ``n`` rows for ``rank``; the first ``n % world`` ranks get one more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def balance_sequences(lengths: list[int], world: int) -> list[list[int]]:
    """Longest-processing-time partition of sequence indices across ``world`` ranks.

    Sequences are taken longest first and each goes to the rank with the fewest tokens so far
    (ties to the lower rank); each rank's list keeps the original order of its sequences.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    heap = [(0, r) for r in range(world)]
    owner = [0] * len(lengths)
    for i in sorted(range(len(lengths)), key=lambda i: (-lengths[i], i)):
        load, r = heapq.heappop(heap)
        owner[i] = r
        heapq.heappush(heap, (load + lengths[i], r))
    return [[i for i in range(len(lengths)) if owner[i] == r] for r in range(world)]


def cu_seqlens_of(lengths: list[int]) -> torch.Tensor:
    out = [0]
    for n in lengths:
        out.append(out[-1] + n)
    return torch.tensor(out, dtype=torch.int32)


def gather_packed(x: torch.Tensor, cu_seqlens: torch.Tensor, indices: list[int]) -> torch.Tensor:
    """Tokens of the chosen sequences from a packed ``[1, T, ...]`` tensor, repacked in that order."""
    cu = cu_seqlens.tolist()
    parts = [x[:, cu[i]:cu[i + 1]] for i in indices]
    return torch.cat(parts, dim=1) if parts else x[:, :0]


def local_varlen(lengths: list[int], rank: int, world: int):
    """Sequence indices, lengths and local ``cu_seqlens`` owned by ``rank``."""
    indices = balance_sequences(lengths, world)[rank]
    local = [lengths[i] for i in indices]
    return indices, local, cu_seqlens_of(local)


class PeerFailure(RuntimeError):
    """A peer rank failed or stopped answering between steps."""


class StepGuard:
    """Failure detection between steps, on the host, over the process group's key-value store.

    Every rank calls ``enter(step)`` before the first launch of a step: it publishes the step it
    has reached and waits until every peer has reached it too. A rank that fails between steps
    calls ``fail(reason)`` (``guard.run`` does it for an exception) and stops; its peers then raise
    ``PeerFailure`` at their next ``enter`` instead of launching work that would wait on it. A peer
    that exits without a word is caught by the deadline: ``PeerFailure`` after ``timeout_s``
    seconds without progress. Nothing here touches a GPU; ranks only ever leave between steps,
    with none of their kernels or collectives in flight.
    """

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "gdn_guard"):
        if world <= 0 or not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside a world of {world}")
        self.store, self.rank, self.world, self.timeout_s, self.prefix = store, rank, world, timeout_s, prefix

    def _step_key(self, r: int) -> str:
        return f"{self.prefix}/step/{r}"

    def _fail_key(self, r: int) -> str:
        return f"{self.prefix}/failed/{r}"

    def fail(self, reason: str) -> None:
        self.store.set(self._fail_key(self.rank), reason)

    def enter(self, step: int) -> None:
        import time

        self.store.set(self._step_key(self.rank), str(step))
        deadline = time.monotonic() + self.timeout_s
        waiting = [r for r in range(self.world) if r != self.rank]
        while waiting:
            for r in list(waiting):
                if self.store.check([self._fail_key(r)]):
                    raise PeerFailure(f"rank {r} failed before step {step}: {self.store.get(self._fail_key(r)).decode()}")
                if self.store.check([self._step_key(r)]) and int(self.store.get(self._step_key(r))) >= step:
                    waiting.remove(r)
            if waiting and time.monotonic() > deadline:
                raise PeerFailure(f"ranks {waiting} did not reach step {step} within {self.timeout_s} s")
            if waiting:
                time.sleep(0.01)

    def run(self, step: int, fn):
        """``enter(step)``, then ``fn()``; an exception in ``fn`` is published to the peers first."""
        self.enter(step)
        try:
            return fn()
        except BaseException as e:
            self.fail(f"{type(e).__name__}: {e}")
            raise
