"""Multi-GPU placement of the packed decode path (one process per GPU).

The path shards with no exchange inside the kernels:

* **by sequence** -- every rank holds whole sequences (all layers, all KV
  heads) and decodes them alone; nothing is communicated;
* **by KV head** -- every rank holds ``n_kv / world`` KV heads of every
  sequence together with their ``n_q / world`` query heads (the GQA groups of
  ``repeat_kv``, reference.py:10-15, stay on one rank), runs K1/K2/K3 on
  them, and the ``[B, n_q / world, D]`` attention outputs of one layer are
  gathered over NCCL (``all_gather_into_tensor``) so every rank holds the
  layer's full output.

This module holds the host-side rules of the KV-head split; the gather is a
plain NCCL collective on the caller's stream (no library kernel reads a peer's
memory).
"""
from __future__ import annotations

import torch


def kv_head_range(n_kv: int, n_q: int, world: int, rank: int) -> tuple[int, int, int, int]:
    """(first KV head, end KV head, first q-head, end q-head) of ``rank``.
    KV heads are split evenly and contiguously; q-head h * gq + j belongs to
    KV head h, so each rank's q-heads are contiguous too."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if n_kv % world:
        raise ValueError(f"{n_kv} KV heads do not split over {world} ranks")
    if n_q % n_kv:
        raise ValueError("query heads must divide into KV heads")
    per = n_kv // world
    gq = n_q // n_kv
    h0 = rank * per
    return h0, h0 + per, h0 * gq, (h0 + per) * gq


def shard_levels(levels, n_kv: int, world: int, rank: int):
    """The rank's rows of per-layer ``[n_kv, head_dim]`` tier maps (a list, one
    map or None per layer, as ``PackedKVCache`` takes them)."""
    h0, h1, _, _ = kv_head_range(n_kv, n_kv, world, rank)
    return [None if lv is None else torch.as_tensor(lv)[h0:h1] for lv in levels]


def gather_heads(local: torch.Tensor, gathered: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather one layer's head-sharded output.  ``local`` ``[B, n_q/world,
    D]`` (contiguous) -> ``gathered`` ``[world, B, n_q/world, D]``, rank r's
    block at index r, on the current stream.  Returns ``gathered``."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if gathered.shape != (world,) + tuple(local.shape) or not local.is_contiguous():
        raise ValueError(f"gather buffer {tuple(gathered.shape)} does not hold {world} x {tuple(local.shape)}")
    if world == 1:
        gathered[0].copy_(local)
        return gathered
    # the concatenated form [world * B, ...] (both NCCL and gloo take it)
    dist.all_gather_into_tensor(gathered.view((world * local.shape[0],) + tuple(local.shape[1:])), local, group=group)
    return gathered


def assemble_heads(gathered: torch.Tensor) -> torch.Tensor:
    """``[world, B, n_q/world, D]`` -> ``[B, n_q, D]`` in q-head order."""
    world, B, hq, D = gathered.shape
    return gathered.permute(1, 0, 2, 3).reshape(B, world * hq, D)
