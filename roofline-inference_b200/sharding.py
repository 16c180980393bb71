"""Host-side partitioning of the attention path over N GPUs of one node.

KV-head sharding (one sequence, strong scaling): rank r of N owns KV heads
[r*nkv/N, (r+1)*nkv/N) and their query heads 2h, 2h+1.  Softmax never crosses
heads, so the only exchange is an all-gather of the per-rank head outputs.
The reference has no multi-device code (its scope is a single stream,
README.md "Single stream ... GPU only"); this partitioning follows from the
GQA structure of its attention (agent-test/v2/attention.py:3-5: query heads
2g and 2g+1 read KV head g).

Sequence sharding (ragged batch): whole sequences go to ranks, balanced by
total context (longest-processing-time-first), and the per-rank outputs are
gathered into fixed-size slots so the collective has equal counts.
"""
from __future__ import annotations

import torch

HEAD_DIM = 128


def head_range(rank: int, world: int, nkv: int = 8) -> tuple[int, int]:
    """KV heads [h0, h1) owned by `rank`."""
    if world < 1 or nkv % world:
        raise ValueError(f"world size {world} must divide the {nkv} KV heads")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    per = nkv // world
    return rank * per, (rank + 1) * per


def shard_qkv(qkv: torch.Tensor, rank: int, world: int, nkv: int = 8) -> torch.Tensor:
    """Slice of the projection rows [..., (2nkv + 2nkv) * 128] this rank needs:
    its query heads, then its K heads, then its V heads -- the layout the
    fused norm/RoPE kernel expects for nq = 2 * local heads (kernels.py:117)."""
    h0, h1 = head_range(rank, world, nkv)
    nq = 2 * nkv
    lead = qkv.shape[:-1]
    x = qkv.reshape(*lead, nq + 2 * nkv, HEAD_DIM)
    q = x[..., 2 * h0:2 * h1, :]
    k = x[..., nq + h0:nq + h1, :]
    v = x[..., nq + nkv + h0:nq + nkv + h1, :]
    return torch.cat([q, k, v], dim=-2).reshape(*lead, -1).contiguous()


def assemble_heads(gathered: torch.Tensor) -> torch.Tensor:
    """[world, ..., nq_local, 128] from an all-gather -> [..., nq, 128] in
    global head order (rank r holds query heads [r*nq_local, (r+1)*nq_local))."""
    world = gathered.shape[0]
    moved = gathered.movedim(0, -3)  # [..., world, nq_local, 128]
    return moved.reshape(*moved.shape[:-3], world * moved.shape[-2], moved.shape[-1])


def balance_sequences(lens: list[int], world: int) -> list[list[int]]:
    """Sequence indices per rank, longest first onto the least loaded rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lens)), key=lambda i: (-lens[i], i))
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        out[r].append(i)
        load[r] += lens[i]
    return [sorted(x) for x in out]


def slots_per_rank(assignment: list[list[int]]) -> int:
    """Equal slot count for the gather (the largest rank's share)."""
    return max((len(a) for a in assignment), default=0)


def scatter_back(gathered: torch.Tensor, assignment: list[list[int]], batch: int) -> torch.Tensor:
    """[world, slots, ...] gathered slot outputs -> [batch, ...] in sequence order."""
    out = torch.empty((batch,) + tuple(gathered.shape[2:]), dtype=gathered.dtype,
                      device=gathered.device)
    for r, seqs in enumerate(assignment):
        for s, i in enumerate(seqs):
            out[i] = gathered[r, s]
    return out
