"""Word-for-word parity at the sizes the benchmark's numbers are quoted on (every residue of every output equal to the
oracle's on the same seeded keys, encryption randomness and inputs):

- the one-head-per-ciphertext attention core of config 3 on the 24 + 8 limb chain at N = 2^16 (dnum 3), 128 cached
  tokens, two heads batched, radix-3 ladders, eager and replayed as a CUDA graph;
- config 3's attention block in the lane layout at the same ring: LayerNorm, Q/K/V projections at GPT-2's padded
  width, the token pushed into the 4-block 128-token cache, attention, output projection, residual — the output and
  both caches after the push;
- the config-2 benchmark step at batch 8: the NTT / INTT pass over the batch's rows, the relinearized product, the 16
  hoisted rotations 2^0 .. 2^15 (inner products in groups of four keys) and the one-pass sum of the 17 outputs.

The oracle does the same op sequence on the host with every core (about a minute per test on 16 cores).
"""
import os

import numpy as np
import pytest
import torch

from perseus_b200 import attention as A
from perseus_b200 import block as B
from perseus_b200 import fhe
from tests import _oracle as O
from tests._oracle_ops import OracleOps

pytestmark = pytest.mark.gpu

SEED, H, SIGMA = 0, 192, 3.2


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


def oracle_for(s):
    O.lib().orc_set_threads(os.cpu_count() or 1)
    o = O.Ctx(s.log_n, s.chain.q, s.chain.p, s.chain.dnum)
    o.keygen(SEED, H, SIGMA, s.galois)
    return o


def test_attention_core_config3_two_heads():
    ch = fhe.config2_chain()
    lay = A.Layout(64, 128, ch.n // 2, radix_bits=3)
    heads = 2
    s = fhe.Session(ch, rot_steps=lay.rot_steps(), k_max=heads, seed=SEED, h=H, sigma=SIGMA)
    oo = OracleOps(oracle_for(s))
    top = len(ch.q) - 1
    rng = np.random.default_rng(300)
    data = [(rng.normal(0, 1, 64) / 8, rng.normal(0, 1, (128, 64)) / 8, rng.normal(0, 1, (128, 64)) / 8)
            for _ in range(heads)]
    coeffs = A.softmax_poly(lay.tokens)
    res = []
    for ops in (s, oo):  # the same encryptions in the same order on both sides (the same nonces)
        caches, qs = [], []
        for qv, K, V in data:
            c = A.KVCache(ops, lay, top)
            c.load(K, V)
            caches.append(c)
        for qv, K, V in data:
            qs.append(A.encrypt_query(ops, qv, lay, top, ch.q[top]))
        cache, q = A.HeadBatch(ops, caches), ops.stack(qs)
        res.append((A.attend(ops, q, cache, coeffs, ch.q), cache, q))
    (y, cache, q), (oy, _, _) = res
    torch.cuda.synchronize()
    assert y.top == oy.top
    for h in range(heads):
        assert (host(y.data[h])[:, : y.top + 1] == oy.cts[h].data[:, : y.top + 1]).all(), f"head {h}"
    graph = A.DecodeGraph(s, cache, coeffs, ch.q, q)
    g = graph(q)
    assert torch.equal(g.data[:, :, : y.top + 1], y.data[:, :, : y.top + 1]), "graph replay"
    for h, (qv, K, V) in enumerate(data):
        got = s.decrypt_slots(g, h).real[:64]
        assert np.abs(got - A.plain_attention(qv, K, V, coeffs)).max() < 1e-3


def test_block_config3_norm_residual():
    ch = fhe.config2_chain()
    lay = B.layout(ch.n // 2, 1024, heads=12, head_dim=64, tokens=128, radix_bits=3)
    s = fhe.Session(ch, rot_steps=lay.rot_steps(), k_max=max(lay.blocks, 3), seed=SEED, h=H, sigma=SIGMA)
    oops = OracleOps(oracle_for(s))
    rng = np.random.default_rng(301)
    n, pre = 768, 101  # the new token lands in block 3, lane 5
    w = B.Weights(*[rng.normal(0, 0.02, (n, n)) if i % 2 == 0 else rng.normal(0, 0.02, n) for i in range(8)])
    gamma, beta = 1 + rng.normal(0, 0.02, n), rng.normal(0, 0.02, n)
    K, V = rng.normal(0, 1, (pre, n)) / 8, rng.normal(0, 1, (pre, n)) / 8
    x = rng.normal(0, 1, n)
    norm, top = B.NormCfg(), len(ch.q) - 1
    coeffs = A.softmax_poly(lay.tokens)
    outs = []
    for ops in (s, oops):
        cache = B.LaneCache(ops, lay, top - 10)
        cache.load(K, V)
        xc = ops.encrypt(B.LIN.input_vector(x, lay.geo), top=top, scale=2.0**40, slots=lay.slots)
        outs.append((B.decode(ops, xc, B.fold_norm(w, gamma, beta), cache, coeffs, ch.q, norm=norm, residual=True),
                     cache))
    (y, cache), (oy, ocache) = outs
    torch.cuda.synchronize()
    oy = oy.cts[0] if hasattr(oy, "cts") else oy
    assert y.top == oy.top
    assert (host(y.data[0])[:, : y.top + 1] == oy.data[:, : y.top + 1]).all(), "block output"
    for blk in range(lay.blocks):
        for dev, orc in ((cache.k, ocache.k), (cache.v, ocache.v)):
            assert (host(dev.data[blk])[:, : cache.top + 1] == orc.cts[blk].data[:, : cache.top + 1]).all(), blk
    got = B.LIN.output_values(s.decrypt_slots(y).real, lay.geo, n)
    want = B.plain_decode(norm.plain(x) * gamma + beta, w, K, V, coeffs, 12, 64) + x
    assert np.abs(got - want).max() < 1e-3


def test_config2_bench_step_batch8():
    ch = fhe.config2_chain()
    steps = [1 << k for k in range(16)]  # the benchmark's rotations; 2^15 is the identity at N = 2^16
    batch = 8
    s = fhe.Session(ch, rot_steps=steps, k_max=batch, seed=SEED, h=H, sigma=SIGMA)
    o = oracle_for(s)
    n, nq, rows = ch.n, len(ch.q), ch.rows
    rng = np.random.default_rng(302)
    x = np.zeros((batch, 2, rows, n), np.uint64)  # residues uniform mod each prime (the benchmark's inputs)
    for r in range(nq):
        x[:, :, r] = rng.integers(0, ch.q[r], (batch, 2, n), dtype=np.uint64)
    ct = fhe.Ct(torch.from_numpy(x.view(np.int64)).cuda(), nq - 1, 2.0**40, n // 2)
    top = nq - 1
    # the NTT / INTT pass over the batch's Q rows
    nbuf = ct.data[:, :, :nq].contiguous().view(-1, n)
    s.ntt_batch(nbuf, batch * 2 * nq)
    want = np.ascontiguousarray(x[:, :, :nq]).reshape(-1, n).copy()
    O.lib().orc_ntt_batch(o.h, want, batch * 2 * nq, 0)
    assert (host(nbuf) == want).all(), "forward NTT batch"
    s.ntt_batch(nbuf, batch * 2 * nq, inverse=True)
    assert (host(nbuf) == x[:, :, :nq].reshape(-1, n)).all(), "inverse NTT batch"
    # relinearization + 16 hoisted rotations + the one-pass sum
    outs = [s.mult(ct, ct)]
    outs += s.rotate_hoisted(ct, steps)
    total = s.sum(outs)
    torch.cuda.synchronize()
    for c in range(batch):
        oc = x[c]
        om = o.mult(oc, oc, top)
        assert (host(outs[0].data[c])[:, : top + 1] == om[:, : top + 1]).all(), f"relin ct {c}"
        acc = om
        for st, r in zip(steps, outs[1:]):
            orot = o.rotate(oc, st, top)
            assert (host(r.data[c])[:, : top + 1] == orot[:, : top + 1]).all(), f"rotation {st} ct {c}"
            acc = o.add(acc, orot, top)
        assert (host(total.data[c])[:, : top + 1] == acc[:, : top + 1]).all(), f"sum ct {c}"
