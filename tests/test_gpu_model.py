"""The multi-layer encrypted decode (perseus_b200/model.py) on the GPU:

- two layers at N = 2^14 (27 + 10 limbs: a refresh leaves top 10; 3 heads x 64 in a 256-wide layout, MLP 768 in
  three full blocks, a 64-token cache per layer): every residue of the output and of every layer's caches after the push equals the oracle's
  running the same op sequence on the same keys and encryptions, and the decryption is within 1e-3 of fp64;
- config 5 at its size: GPT-2 small's 12 layers (768 wide, 12 heads x 64, MLP 3072, weights N(0, 0.02)) with a
  256-token encrypted cache per layer resident in HBM, N = 2^16 on config 4's chain (a refresh leaves 12 levels), two
  tokens decoded one after the other; decrypted within 1e-2 of the fp64 decode with the same polynomials (48 refreshes
  per token).
"""
import os

import numpy as np
import pytest
import torch

from perseus_b200 import bootstrap as BS
from perseus_b200 import fhe
from perseus_b200 import linear as LIN
from perseus_b200 import model as M
from tests import _oracle as O
from tests._oracle_ops import OracleOps

pytestmark = pytest.mark.gpu


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


def session(ch, prm, lay, k_max, h):
    steps = sorted(set(BS.rot_steps(prm)) | set(lay.rot_steps()))
    return fhe.Session(ch, rot_steps=steps, k_max=k_max, seed=0, h=h, sigma=3.2, galois_extra=(BS.conj_galois(ch.n),))


def test_two_layers_bit_exact_with_the_oracle():
    logn = 14
    cfg = M.ModelCfg(layers=2, d=192, width=256, heads=3, head_dim=64, mlp=768, tokens=64, radix_bits=3)
    prm = BS.Params(1 << logn, K=24, r=3, per_group=5)
    ch = fhe.Chain(logn, tuple(fhe.ntt_primes(50, logn, 27)), tuple(fhe.ntt_primes(50, logn, 10, skip=27)), 3)
    lay = M.B.layout(ch.n // 2, cfg.width, cfg.heads, cfg.head_dim, cfg.tokens, cfg.radix_bits)
    s = session(ch, prm, lay, 4, 64)
    O.lib().orc_set_threads(os.cpu_count() or 1)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(0, 64, 3.2, s.galois)
    oo = OracleOps(o)
    rng = np.random.default_rng(60)
    weights = [M.random_layer(rng, d=cfg.d, mlp=cfg.mlp, std=0.05) for _ in range(cfg.layers)]
    pre = 40
    Ks = [rng.normal(0, 1, (pre, cfg.d)) / 8 for _ in range(cfg.layers)]
    Vs = [rng.normal(0, 1, (pre, cfg.d)) / 8 for _ in range(cfg.layers)]
    x = rng.normal(0, 1, cfg.d)
    outs = []
    for ops in (s, oo):  # the same encryptions in the same order on both sides
        dec = M.Decoder(ops, cfg, weights, ch.q, BS.Bootstrapper(ops, prm, ch.q, ch.q[0]))
        assert dec.out_top == 10
        dec.load(Ks, Vs)
        xc = ops.encrypt(LIN.input_vector(x, dec.lay.geo), 0, 2.0**40, dec.lay.slots)
        outs.append((dec, dec.decode(xc)))
    (dec, y), (odec, oy) = outs
    torch.cuda.synchronize()
    oy = oy.cts[0] if hasattr(oy, "cts") else oy
    assert y.top == oy.top
    assert (host(y.data[0])[:, : y.top + 1] == oy.data[:, : y.top + 1]).all(), "decoder output"
    for l, (c, oc) in enumerate(zip(dec.caches, odec.caches)):
        for blk in range(dec.lay.blocks):
            for dv, ov in ((c.k, oc.k), (c.v, oc.v)):
                assert (host(dv.data[blk])[:, : c.top + 1] == ov.cts[blk].data[:, : c.top + 1]).all(), (l, blk)
    want = M.plain_decode(x, weights, [[K.copy(), V.copy()] for K, V in zip(Ks, Vs)], cfg, dec.coeffs)
    got = LIN.output_values(s.decrypt_slots(y).real, dec.lay.geo, cfg.d)
    assert np.abs(got - want).max() < 1e-3


def test_config5_twelve_layers():
    cfg = M.ModelCfg()
    ch = fhe.config4_chain()
    prm = BS.Params(ch.n, K=24, r=3, per_group=5)
    lay = M.B.layout(ch.n // 2, cfg.width, cfg.heads, cfg.head_dim, cfg.tokens, cfg.radix_bits)
    s = session(ch, prm, lay, lay.blocks, 192)
    rng = np.random.default_rng(61)
    weights = [M.random_layer(rng) for _ in range(cfg.layers)]
    pre = cfg.tokens - 2
    Ks = [rng.normal(0, 1, (pre, cfg.d)) / 8 for _ in range(cfg.layers)]
    Vs = [rng.normal(0, 1, (pre, cfg.d)) / 8 for _ in range(cfg.layers)]
    dec = M.Decoder(s, cfg, weights, ch.q, BS.Bootstrapper(s, prm, ch.q, ch.q[0]))
    assert (dec.out_top, dec.cache_top) == (12, 10)
    dec.load(Ks, Vs)
    plain = [[K.copy(), V.copy()] for K, V in zip(Ks, Vs)]
    for tok in range(2):
        x = rng.normal(0, 1, cfg.d)
        xc = s.encrypt(LIN.input_vector(x, dec.lay.geo), top=0, scale=2.0**40, slots=dec.lay.slots)
        y = dec.decode(xc)
        want = M.plain_decode(x, weights, plain, cfg, dec.coeffs)
        got = LIN.output_values(s.decrypt_slots(y).real, dec.lay.geo, cfg.d)
        assert np.abs(got - want).max() < 1e-2, (tok, float(np.abs(got - want).max()))
    assert all(c.count == cfg.tokens for c in dec.caches)
