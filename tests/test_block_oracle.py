"""The attention block's decode step (projections, cache push, attention in lanes, output projection) on the oracle:
decrypted against the fp64 step with the same polynomial softmax (small ring; the GPU parity test runs the same
sequence on both sides word for word)."""
import numpy as np
import pytest

from perseus_b200 import attention as A
from perseus_b200 import block as B
from tests import _oracle as O
from tests._oracle_ops import OracleOps

LOGN = 10


def _weights(rng, n, s=0.1):
    return B.Weights(*[rng.normal(0, s, (n, n)) if i % 2 == 0 else rng.normal(0, 0.02, n) for i in range(8)])


@pytest.mark.parametrize("radix", [1, 3])
def test_block_decode_on_the_oracle(radix):
    lay = B.layout(1 << (LOGN - 1), 32, heads=4, head_dim=8, tokens=32, radix_bits=radix)
    assert (lay.t, lay.blocks) == (16, 2)
    q = O.ntt_primes(50, LOGN, 12)
    p = O.ntt_primes(50, LOGN, 3, skip=12)  # the special primes cover a digit (3 limbs)
    c = O.Ctx(LOGN, q, p, 4)
    c.keygen(seed=0, h=64, sigma=3.2, galois=[1] + [O.lib().orc_rotation_galois(s, LOGN) for s in lay.rot_steps()])
    ops = OracleOps(c)
    rng = np.random.default_rng(9)
    n, pre = 32, 21  # the new token lands in block 1, lane 5
    w = _weights(rng, n)
    K, V = rng.normal(0, 1, (pre, n)) / 8, rng.normal(0, 1, (pre, n)) / 8
    x = rng.normal(0, 1, n) / 2
    top = c.nq - 1
    cache = B.LaneCache(ops, lay, top - 2)
    cache.load(K, V)
    coeffs = A.softmax_poly(lay.tokens)
    xc = ops.encrypt(B.LIN.input_vector(x, lay.geo), top, 2.0**40, lay.slots)
    y = B.decode(ops, xc, w, cache, coeffs, c.q)
    assert cache.count == pre + 1 and y.top == top - 10
    got = B.LIN.output_values(ops.decrypt_slots(y).real, lay.geo, n)
    want = B.plain_decode(x, w, K, V, coeffs, 4, 8)
    assert np.abs(got - want).max() < 1e-3, np.abs(got - want).max()


def test_block_with_norm_and_residual_on_the_oracle():
    """LayerNorm (polynomial inverse square root, gamma and beta folded into Q/K/V), the block, the residual."""
    lay = B.layout(1 << (LOGN - 1), 32, heads=4, head_dim=8, tokens=16, radix_bits=2)
    q = O.ntt_primes(50, LOGN, 21)
    p = O.ntt_primes(50, LOGN, 3, skip=21)
    c = O.Ctx(LOGN, q, p, 7)
    c.keygen(seed=0, h=64, sigma=3.2, galois=[1] + [O.lib().orc_rotation_galois(s, LOGN) for s in lay.rot_steps()])
    ops = OracleOps(c)
    rng = np.random.default_rng(10)
    n, pre = 32, 3
    w = _weights(rng, n)
    gamma, beta = 1 + rng.normal(0, 0.1, n), rng.normal(0, 0.1, n)
    wf = B.fold_norm(w, gamma, beta)
    K, V = rng.normal(0, 1, (pre, n)) / 8, rng.normal(0, 1, (pre, n)) / 8
    x = rng.normal(0, 1, n)
    norm = B.NormCfg(lo=0.25, hi=4.0)
    u = ((x - x.mean()) ** 2).mean()
    assert norm.lo < u < norm.hi
    top = c.nq - 1
    cache = B.LaneCache(ops, lay, top - 10)
    cache.load(K, V)
    coeffs = A.softmax_poly(lay.tokens)
    xc = ops.encrypt(B.LIN.input_vector(x, lay.geo), top, 2.0**40, lay.slots)
    y = B.decode(ops, xc, wf, cache, coeffs, c.q, norm=norm, residual=True)
    assert y.top == top - 18
    got = B.LIN.output_values(ops.decrypt_slots(y).real, lay.geo, n)
    # the reference applies gamma and beta after the polynomial norm, the encrypted path inside the linears
    want = B.plain_decode(x, B.Weights(w.wq, w.bq, w.wk, w.bk, w.wv, w.bv, w.wo, w.bo), K, V, coeffs, 4, 8,
                          norm=_Affine(norm, gamma, beta), residual=True)
    assert np.abs(got - want).max() < 1e-3, np.abs(got - want).max()


class _Affine:
    def __init__(self, norm, gamma, beta):
        self.norm, self.gamma, self.beta = norm, gamma, beta

    def plain(self, x):
        return self.norm.plain(x) * self.gamma + self.beta


@pytest.mark.parametrize("radix", [1, 2, 3])
def test_lane_layout_invariants(radix):
    """GPT-2's lane layout: every lane reachable by rotations whose keys the layout generates; the score mask on lane
    tau of each head's first element block; lane 0 of the real elements; the ladders' spans."""
    lay = B.layout(1 << 15, 1024, heads=12, head_dim=64, tokens=128, radix_bits=radix)
    assert (lay.t, lay.blocks, lay.width) == (32, 4, 768)
    keys = {s % lay.slots for s in lay.rot_steps()}
    for lane in range(lay.t):
        steps = lay.push_steps(lane)
        assert -sum(steps) == lane and all(s % lay.slots in keys for s in steps)
        assert len(steps) <= (2 if radix == 3 else 5)
    m = lay.mask()
    assert m.sum() == 12 * 32 and all(m[h * 64 * 32 + tau] == 1 for h in range(12) for tau in range(32))
    l0 = lay.lane0(0.5)
    assert (np.flatnonzero(l0) == np.arange(768) * 32).all() and l0.max() == 0.5
    assert lay.score_ladder() == (32, 2048) and lay.replicate_ladder() == (-32, 2048)
    assert lay.sum_ladder() == (1, 32) and lay.norm_ladder() == (32, 32 * 1024)
    with pytest.raises(ValueError):
        B.layout(1 << 15, 1024, heads=12, head_dim=64, tokens=100)


def test_block_two_sequences_on_the_oracle():
    """Two independent sequences decoded in one batched step: each output equals its own fp64 step."""
    lay = B.layout(1 << (LOGN - 1), 32, heads=4, head_dim=8, tokens=32, radix_bits=3)
    q = O.ntt_primes(50, LOGN, 12)
    p = O.ntt_primes(50, LOGN, 3, skip=12)
    c = O.Ctx(LOGN, q, p, 4)
    c.keygen(seed=0, h=64, sigma=3.2, galois=[1] + [O.lib().orc_rotation_galois(s, LOGN) for s in lay.rot_steps()])
    ops = OracleOps(c)
    rng = np.random.default_rng(31)
    n, pre, S = 32, 19, 2
    w = _weights(rng, n)
    Ks = [rng.normal(0, 1, (pre, n)) / 8 for _ in range(S)]
    Vs = [rng.normal(0, 1, (pre, n)) / 8 for _ in range(S)]
    xs = [rng.normal(0, 1, n) / 2 for _ in range(S)]
    top = c.nq - 1
    cache = B.LaneCache(ops, lay, top - 2, seqs=S)
    cache.load(Ks, Vs)
    coeffs = A.softmax_poly(lay.tokens)
    xc = ops.stack([ops.encrypt(B.LIN.input_vector(x, lay.geo), top, 2.0**40, lay.slots) for x in xs])
    y = B.decode(ops, xc, w, cache, coeffs, c.q)
    for s_ in range(S):
        got = B.LIN.output_values(ops.decrypt_slots(y, s_).real, lay.geo, n)
        want = B.plain_decode(xs[s_], w, Ks[s_], Vs[s_], coeffs, 4, 8)
        assert np.abs(got - want).max() < 1e-3, (s_, np.abs(got - want).max())
