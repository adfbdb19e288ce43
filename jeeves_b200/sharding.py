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
