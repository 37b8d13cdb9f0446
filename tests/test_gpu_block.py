"""The attention block's decode step on the GPU against the same op sequence on the oracle, word for word: Q/K/V
projections, the token pushed into the lane cache, attention over two token blocks, the output projection (FP64
chain at N = 2^14 with 12 limbs); decrypted against the fp64 step."""
import numpy as np
import pytest

from perseus_b200 import attention as A
from perseus_b200 import block as B
from perseus_b200 import fhe
from tests import _oracle as O
from tests._oracle_ops import OracleOps

pytestmark = pytest.mark.gpu


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


@pytest.mark.parametrize("radix", [3])
def test_block_decode_bit_exact(radix):
    ch = fhe.Chain(14, tuple(fhe.ntt_primes(50, 14, 12)), tuple(fhe.ntt_primes(50, 14, 3, skip=12)), 4)
    lay = B.layout(ch.n // 2, 256, heads=4, head_dim=64, tokens=64, radix_bits=radix)
    s = fhe.Session(ch, rot_steps=lay.rot_steps(), k_max=3, seed=0)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(0, 192, 3.2, s.galois)
    oops = OracleOps(o)
    rng = np.random.default_rng(12)
    n, pre = 256, 37  # the new token: block 1, lane 5
    w = B.Weights(*[rng.normal(0, 0.05, (n, n)) if i % 2 == 0 else rng.normal(0, 0.02, n) for i in range(8)])
    K, V = rng.normal(0, 1, (pre, n)) / 8, rng.normal(0, 1, (pre, n)) / 8
    x = rng.normal(0, 1, n) / 2
    top = s.top()
    coeffs = A.softmax_poly(lay.tokens)
    outs = []
    for ops in (s, oops):
        cache = B.LaneCache(ops, lay, top - 2)
        cache.load(K, V)
        xc = ops.encrypt(B.LIN.input_vector(x, lay.geo), top=top, scale=2.0**40, slots=lay.slots)
        outs.append((B.decode(ops, xc, w, cache, coeffs, ch.q), cache))
    (y, cache), (oy, ocache) = outs
    assert y.top == oy.top == top - 10
    assert (host(y.data[0])[:, : y.top + 1] == oy.data[:, : y.top + 1]).all()
    for blk in range(lay.blocks):
        for dev, orc in ((cache.k, ocache.k), (cache.v, ocache.v)):
            assert (host(dev.data[blk])[:, : cache.top + 1] == orc.cts[blk].data[:, : cache.top + 1]).all(), blk
    got = B.LIN.output_values(s.decrypt_slots(y).real, lay.geo, n)
    want = B.plain_decode(x, w, K, V, coeffs, 4, 64)
    assert np.abs(got - want).max() < 1e-3


def test_block_with_norm_bit_exact():
    """LayerNorm (gamma, beta folded into Q/K/V), the block over one token block, the residual: GPU = oracle word for
    word (21-limb FP64 chain at N = 2^14)."""
    ch = fhe.Chain(14, tuple(fhe.ntt_primes(50, 14, 21)), tuple(fhe.ntt_primes(50, 14, 3, skip=21)), 7)
    lay = B.layout(ch.n // 2, 256, heads=4, head_dim=64, tokens=32, radix_bits=2)
    s = fhe.Session(ch, rot_steps=lay.rot_steps(), k_max=3, seed=0)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(0, 192, 3.2, s.galois)
    oops = OracleOps(o)
    rng = np.random.default_rng(13)
    n, pre = 256, 9
    w = B.Weights(*[rng.normal(0, 0.05, (n, n)) if i % 2 == 0 else rng.normal(0, 0.02, n) for i in range(8)])
    gamma, beta = 1 + rng.normal(0, 0.1, n), rng.normal(0, 0.1, n)
    K, V = rng.normal(0, 1, (pre, n)) / 8, rng.normal(0, 1, (pre, n)) / 8
    x = rng.normal(0, 1, n)
    norm = B.NormCfg()
    top = s.top()
    coeffs = A.softmax_poly(lay.tokens)
    outs = []
    for ops in (s, oops):
        cache = B.LaneCache(ops, lay, top - 10)
        cache.load(K, V)
        xc = ops.encrypt(B.LIN.input_vector(x, lay.geo), top=top, scale=2.0**40, slots=lay.slots)
        outs.append(B.decode(ops, xc, B.fold_norm(w, gamma, beta), cache, coeffs, ch.q, norm=norm, residual=True))
    y, oy = outs
    oy = oy.cts[0] if hasattr(oy, "cts") else oy  # one cache block: the oracle's batch of one
    assert y.top == oy.top == top - 18
    assert (host(y.data[0])[:, : y.top + 1] == oy.data[:, : y.top + 1]).all()
    got = B.LIN.output_values(s.decrypt_slots(y).real, lay.geo, n)
    xn = norm.plain(x) * gamma + beta
    want = B.plain_decode(xn, w, K, V, coeffs, 4, 64) + x
    assert np.abs(got - want).max() < 1e-3


def test_block_two_sequences_bit_exact():
    """Two sequences decoded in one batched step (their caches one batch of 2 x 2 blocks): GPU = oracle word for word,
    each output against its own fp64 step."""
    ch = fhe.Chain(14, tuple(fhe.ntt_primes(50, 14, 12)), tuple(fhe.ntt_primes(50, 14, 3, skip=12)), 4)
    lay = B.layout(ch.n // 2, 256, heads=4, head_dim=64, tokens=64, radix_bits=3)
    S = 2
    s = fhe.Session(ch, rot_steps=lay.rot_steps(), k_max=3 * S, seed=0)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(0, 192, 3.2, s.galois)
    oops = OracleOps(o)
    rng = np.random.default_rng(14)
    n, pre = 256, 40
    w = B.Weights(*[rng.normal(0, 0.05, (n, n)) if i % 2 == 0 else rng.normal(0, 0.02, n) for i in range(8)])
    Ks = [rng.normal(0, 1, (pre, n)) / 8 for _ in range(S)]
    Vs = [rng.normal(0, 1, (pre, n)) / 8 for _ in range(S)]
    xs = [rng.normal(0, 1, n) / 2 for _ in range(S)]
    top = s.top()
    coeffs = A.softmax_poly(lay.tokens)
    outs = []
    for ops in (s, oops):
        cache = B.LaneCache(ops, lay, top - 2, seqs=S)
        cache.load(Ks, Vs)
        xc = ops.stack([ops.encrypt(B.LIN.input_vector(x, lay.geo), top=top, scale=2.0**40, slots=lay.slots)
                        for x in xs])
        outs.append(B.decode(ops, xc, w, cache, coeffs, ch.q))
    y, oy = outs
    for q in range(S):
        assert (host(y.data[q])[:, : y.top + 1] == oy.cts[q].data[:, : y.top + 1]).all(), q
        got = B.LIN.output_values(s.decrypt_slots(y, q).real, lay.geo, n)
        assert np.abs(got - B.plain_decode(xs[q], w, Ks[q], Vs[q], coeffs, 4, 64)).max() < 1e-3
