"""Head and batch sharding over ranks (host logic of the multi-GPU path), with gloo ranks on the CPU: every head
decoded exactly once, results gathered in head order, the gathered decode equal to fp64 attention."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from perseus_b200 import attention as A
from perseus_b200 import fhe
from perseus_b200 import shard


@pytest.mark.parametrize("n,world", [(12, 1), (12, 2), (12, 5), (12, 8), (3, 2), (64, 3), (2, 4), (0, 2)])
def test_share_partitions(n, world):
    parts = [shard.share(n, world, r) for r in range(world)]
    assert [u for p in parts for u in p] == list(range(n))
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)


def test_share_refuses_bad_ranks():
    for args in [(12, 0, 0), (12, 2, 2), (12, 2, -1), (-1, 2, 0)]:
        with pytest.raises(ValueError):
            shard.share(*args)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n_heads, tokens, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from tests import _oracle as O
        from tests._oracle_ops import OracleOps

        O.lib().orc_set_threads(2)
        ch = fhe.Chain(12, tuple(fhe.ntt_primes(50, 12, 8)), tuple(fhe.ntt_primes(60, 12, 1)), 8)
        lay = A.Layout(head_dim=64, tokens=tokens, slots=ch.n // 2)
        gal = [1] + sorted({fhe.rotation_galois(s, ch.log_n) for s in lay.rot_steps()} - {1})
        o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
        o.keygen(0, 192, 3.2, gal)
        ops = OracleOps(o)
        coeffs = A.softmax_poly(tokens)
        top = len(ch.q) - 1
        # every rank draws the whole problem from one seed and decodes its own heads
        rng = np.random.default_rng(7)
        q = rng.normal(0, 1, (n_heads, 64)) / 8
        K = rng.normal(0, 1, (n_heads, tokens, 64)) / 8
        V = rng.normal(0, 1, (n_heads, tokens, 64)) / 8
        mine = shard.head_range(n_heads, world, rank)
        got, ids = [], []
        for h in mine:
            cache = A.KVCache(ops, lay, top)
            cache.load(K[h], V[h])
            out = A.attend(ops, A.encrypt_query(ops, q[h], lay, top, ch.q[top]), cache, coeffs, ch.q)
            got.append(ops.decrypt_slots(out).real[:64])
            ids.append(h)
        local = torch.tensor(np.array(got).reshape(len(mine), 64), dtype=torch.float64)
        full = shard.gather_heads(local, n_heads)
        heads = shard.gather_heads(torch.tensor(ids, dtype=torch.int64).reshape(-1, 1), n_heads)
        assert heads.flatten().tolist() == list(range(n_heads))
        want = np.stack([A.plain_attention(q[h], K[h], V[h], coeffs) for h in range(n_heads)])
        err = np.abs(full.numpy() - want).max()
        assert err < 1e-3, err
        # integer payloads (ciphertext residues) travel exactly
        words = torch.tensor([[(h << 40) + 12345 + j for j in range(4)] for h in mine], dtype=torch.int64)
        back = shard.gather_heads(words.reshape(len(mine), 4), n_heads)
        assert back.tolist() == [[(h << 40) + 12345 + j for j in range(4)] for h in range(n_heads)]
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # the parent reports it
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world,n_heads", [(2, 3)])
def test_sharded_decode_gloo(world, n_heads):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n_heads, 16, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs)


def test_gather_refuses_wrong_share():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    p = ctx.Process(target=_wrong_share, args=(_free_port(), errq))
    p.start()
    p.join(timeout=120)
    assert p.exitcode == 0
    assert errq.get() == "ValueError"


def _wrong_share(port, errq):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        shard.gather_heads(torch.zeros(3, 4), 12)  # a single rank holds all 12 heads
        errq.put("no error")
    except ValueError:
        errq.put("ValueError")
    dist.destroy_process_group()
