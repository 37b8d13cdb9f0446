"""Partitioning of the decode step over the GPUs of one box (one process per GPU).

The attention heads of a decode step and the ciphertexts of a key-switch batch are independent: each rank takes a
contiguous share and keeps a replica of the keys, with no collective on the data path. The one exchange is after the
step, when the out-projection needs every head: `gather_heads` collects the per-head results (ciphertext residues
or decrypted slots) from all ranks in head order.

The reference runs a session on one GPU (`crates/pc-gpu/src/executor.rs`); spreading heads and batches over the
GPUs of a box is this library's addition, at the seams where no data moves between them.
"""
from __future__ import annotations

import torch


def share(n: int, world: int, rank: int) -> range:
    """Rank `rank`'s contiguous share of n independent units: the first n % world ranks take one more."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad partition: n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (1 if rank < extra else 0))


def head_range(n_heads: int, world: int, rank: int) -> range:
    """The attention heads rank `rank` decodes."""
    return share(n_heads, world, rank)


def batch_range(n_cts: int, world: int, rank: int) -> range:
    """The ciphertexts of a batch rank `rank` key-switches."""
    return share(n_cts, world, rank)


def gather_heads(local: torch.Tensor, n_heads: int, group=None) -> torch.Tensor:
    """All ranks' per-head results, in head order, on every rank.

    `local` is [len(head_range(n_heads, world, rank)), ...] on this rank (any dtype; CUDA tensors with NCCL, CPU
    tensors with gloo). Shares differ by at most one head, so each rank pads to the largest share, one all_gather
    moves the padded blocks, and the padding is dropped.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    mine = head_range(n_heads, world, rank)
    if local.shape[0] != len(mine):
        raise ValueError(f"rank {rank} holds {local.shape[0]} heads, its share is {len(mine)}")
    width = len(head_range(n_heads, world, 0))
    pad = local.new_zeros((width,) + tuple(local.shape[1:]))
    pad[:len(mine)] = local
    blocks = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(blocks, pad, group=group)
    return torch.cat([blocks[r][:len(head_range(n_heads, world, r))] for r in range(world)])
