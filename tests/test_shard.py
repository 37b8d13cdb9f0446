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


def _block_rank_main(rank, world, port, errq):
    """The lane-layout attention block with its cache blocks split over the ranks (perseus_b200.block.LaneCache
    shard=...), against the unsharded step on the same session randomness: every rank's output equals the
    unsharded output word for word, and its blocks equal the matching unsharded blocks, over two tokens."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from perseus_b200 import block as B
        from tests import _oracle as O
        from tests._oracle_ops import OracleOps

        O.lib().orc_set_threads(2)
        logn = 10
        lay = B.layout(1 << (logn - 1), 32, heads=4, head_dim=8, tokens=32, radix_bits=3)  # 2 blocks of 16
        q = O.ntt_primes(50, logn, 12)
        p = O.ntt_primes(50, logn, 3, skip=12)
        gal = [1] + [O.lib().orc_rotation_galois(s, logn) for s in lay.rot_steps()]
        rng = np.random.default_rng(9)
        n, pre = 32, 15  # tokens 15 (block 0, lane 15) and 16 (block 1, lane 0) are pushed
        w = B.Weights(*[rng.normal(0, 0.1, (n, n)) if i % 2 == 0 else rng.normal(0, 0.02, n) for i in range(8)])
        K, V = rng.normal(0, 1, (pre, n)) / 8, rng.normal(0, 1, (pre, n)) / 8
        xs = [rng.normal(0, 1, n) / 2 for _ in range(2)]
        coeffs = A.softmax_poly(lay.tokens)
        runs = []
        for sh in (None, (world, rank)):
            c = O.Ctx(logn, q, p, 4)
            c.keygen(seed=0, h=64, sigma=3.2, galois=gal)
            ops = OracleOps(c)
            top = c.nq - 1
            cache = B.LaneCache(ops, lay, top - 2, shard=sh)
            cache.load(K, V)
            ys = []
            for x in xs:
                xc = ops.encrypt(B.LIN.input_vector(x, lay.geo), top, 2.0**40, lay.slots)
                ys.append(B.decode(ops, xc, w, cache, coeffs, c.q))
            runs.append((ys, cache))
        (ys, full), (zs, part) = runs
        one = lambda c: c.cts[0] if hasattr(c, "cts") else c  # noqa: E731
        for y, z in zip(ys, zs):
            y, z = one(y), one(z)
            assert z.top == y.top and (z.data[:, : y.top + 1] == y.data[:, : y.top + 1]).all()
        assert part.mine == list(shard.share(lay.blocks, world, rank))
        blocks = lambda b: b.cts if hasattr(b, "cts") else [b]  # noqa: E731
        for li, b in enumerate(part.mine):
            for mine_b, all_b in ((blocks(part.k)[li], blocks(full.k)[b]), (blocks(part.v)[li], blocks(full.v)[b])):
                assert (mine_b.data[:, : part.top + 1] == all_b.data[:, : part.top + 1]).all(), b
        if part.idle:
            assert not blocks(part.k)[0].data.any()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # the parent reports it
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world", [2, 3, 4])
def test_sharded_block_gloo(world):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_block_rank_main, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs)


def _model_rank_main(rank, world, port, errq):
    """The multi-layer decode (perseus_b200.model.Decoder) with every layer's cache blocks split over the ranks,
    refreshes and MLP on every rank, against the unsharded decode on the same session randomness: every rank's
    output equals the unsharded output word for word, and its blocks equal the matching unsharded blocks."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from perseus_b200 import bootstrap as BS
        from perseus_b200 import fhe
        from perseus_b200 import linear as LIN
        from perseus_b200 import model as M
        from tests import _oracle as O
        from tests._oracle_ops import OracleOps

        O.lib().orc_set_threads(2)
        logn = 10
        n_ring = 1 << logn
        cfg = M.ModelCfg(layers=1, d=24, width=32, heads=3, head_dim=8, mlp=64, tokens=32, radix_bits=2)
        prm = BS.Params(n_ring, K=24, r=3, per_group=5)
        q = O.ntt_primes(50, logn, 25)
        p = O.ntt_primes(50, logn, 6, skip=25)
        lay = M.B.layout(n_ring // 2, cfg.width, cfg.heads, cfg.head_dim, cfg.tokens, cfg.radix_bits)
        steps = sorted(set(BS.rot_steps(prm)) | set(lay.rot_steps()))
        gal = list(dict.fromkeys([1] + [fhe.rotation_galois(s, logn) for s in steps] + [BS.conj_galois(n_ring)]))
        rng = np.random.default_rng(52)
        weights = [M.random_layer(rng, d=cfg.d, mlp=cfg.mlp, std=0.1)]
        pre = 15  # token 15 lands in block 0, lane 15
        Ks, Vs = [rng.normal(0, 1, (pre, cfg.d)) / 8], [rng.normal(0, 1, (pre, cfg.d)) / 8]
        x = rng.normal(0, 1, cfg.d)
        runs = []
        for sh in (None, (world, rank)):
            c = O.Ctx(logn, q, p, 5)
            c.keygen(seed=0, h=64, sigma=3.2, galois=gal)
            ops = OracleOps(c)
            dec = M.Decoder(ops, cfg, weights, c.q, BS.Bootstrapper(ops, prm, c.q, c.q[0]), shard=sh)
            dec.load(Ks, Vs)
            y = dec.decode(ops.encrypt(LIN.input_vector(x, dec.lay.geo), 0, 2.0**40, dec.lay.slots))
            runs.append((y, dec.caches[0]))
        (y, full), (z, part) = runs
        one = lambda c: c.cts[0] if hasattr(c, "cts") else c  # noqa: E731
        y, z = one(y), one(z)
        assert z.top == y.top and (z.data[:, : y.top + 1] == y.data[:, : y.top + 1]).all()
        blocks = lambda b: b.cts if hasattr(b, "cts") else [b]  # noqa: E731
        for li, b in enumerate(part.mine):
            for mine_b, all_b in ((blocks(part.k)[li], blocks(full.k)[b]), (blocks(part.v)[li], blocks(full.v)[b])):
                assert (mine_b.data[:, : part.top + 1] == all_b.data[:, : part.top + 1]).all(), b
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # the parent reports it
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_model_gloo(world):
    """world 3: the two cache blocks over three ranks leave one rank idle in every layer's attention"""
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_model_rank_main, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs)
