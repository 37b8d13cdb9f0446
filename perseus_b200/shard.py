"""Partitioning of the decode step over the GPUs of one box (one process per GPU).

The attention heads of a decode step and the ciphertexts of a key-switch batch are independent: each rank takes a
contiguous share and keeps a replica of the keys, with no collective on the data path. The one exchange is after the
step, when the out-projection needs every head: `gather_heads` collects the per-head results (ciphertext residues
or decrypted slots) from all ranks in head order.

The attention block in the lane layout (perseus_b200/block.py) splits its cache blocks instead: each rank attends
over its share of the blocks, and `gather_sum` adds the ranks' partial outputs — one all_gather of the ciphertexts'
residues (the collective moves bytes; NCCL's own sum would not reduce mod p), then one modular sum on every rank, so
every rank holds the same words.

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


def gather_sum(ops, ct, group=None):
    """The sum over all ranks of ct (this rank's partial result: a session Ct on the device, or an oracle ciphertext
    or batch on the host), on every rank: one all_gather of the residues (the whole ciphertext layout, so every rank
    sends the same shape), then the session's one-pass modular sum (an oracle batch: member by member). Exact: every
    rank gets the same words as summing all the partials on one GPU, in any order."""
    import numpy as np
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if torch.is_tensor(getattr(ct, "data", None)):  # a session ciphertext batch on the device (NCCL)
        from . import fhe

        bufs = [torch.empty_like(ct.data) for _ in range(world)]
        dist.all_gather(bufs, ct.data.contiguous(), group=group)
        return ops.sum([fhe.Ct(b, ct.top, ct.scale, ct.slots) for b in bufs])
    members = ct.cts if hasattr(ct, "cts") else [ct]  # oracle ciphertexts on the host (gloo)
    local = torch.from_numpy(np.ascontiguousarray(np.stack([m.data for m in members])).view(np.int64))
    bufs = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(bufs, local, group=group)
    parts = []
    for b in bufs:
        arr = b.numpy().view(np.uint64)
        got = [type(m)(arr[i].copy(), m.top, m.scale, m.slots) for i, m in enumerate(members)]
        parts.append(got[0] if not hasattr(ct, "cts") else ops.stack(got))
    return ops.sum(parts)
