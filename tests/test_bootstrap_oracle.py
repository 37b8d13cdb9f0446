"""CKKS bootstrapping (perseus_b200/bootstrap.py) on the oracle: the CoeffToSlot / SlotToCoeff stage diagonals against
the oracle's encoder (crates/pc-core/src/encode.rs restated), and a full refresh of a level-0 ciphertext at a small
ring (BASELINE config 4's steps: ModRaise, CoeffToSlot, EvalMod by a degree-63 Chebyshev interpolant with double
angles, SlotToCoeff) decrypting to its slots."""
import math

import numpy as np
import pytest

from perseus_b200 import bootstrap as BS
from perseus_b200 import fhe
from tests import _oracle as O
from tests._oracle_ops import OracleOps

LOGN = 10
N = 1 << LOGN
S = N // 2


def _apply(groups, x):
    for _, d in groups:
        y = np.zeros(len(x), np.complex128)
        for o, dd in d.items():
            y += dd * np.roll(x, -o)
        x = y
    return x


def _bitrev(v):
    bits = int(math.log2(len(v)))
    return v[[int(format(i, f"0{bits}b")[::-1], 2) for i in range(len(v))]]


@pytest.fixture(scope="module")
def ctx():
    q = O.ntt_primes(50, LOGN, 20)
    p = O.ntt_primes(50, LOGN, 6, skip=20)  # P one prime larger than a digit of 5
    steps = sorted(set(BS.rot_steps(BS.Params(N, per_group=3))) | set(BS.rot_steps(BS.Params(N, per_group=5))))
    gal = list(dict.fromkeys([1] + [fhe.rotation_galois(s, LOGN) for s in steps] + [BS.conj_galois(N)]))
    c = O.Ctx(LOGN, q, p, 4)
    c.keygen(seed=0, h=64, sigma=3.2, galois=gal)
    return c


@pytest.mark.parametrize("per", [2, 3, 4])
def test_stage_groups_are_the_encoders_fft(ctx, per):
    """Slots = F(bitrev(w)) for w_i = (c_i + i c_(i+S)) / scale of the oracle's own encoding; G = S F^-1."""
    c = ctx
    rng = np.random.default_rng(per)
    z = rng.uniform(-1, 1, S) + 1j * rng.uniform(-1, 1, S)
    scale = 2.0**40
    rows = c.encode(z, S, scale, 0)
    coef = rows[0].astype(np.int64)
    coef = np.where(coef > c.q[0] // 2, coef - np.int64(c.q[0]), coef).astype(np.float64)
    w = (coef[:S] + 1j * coef[S:]) / scale
    F, G = BS.groups(N, False, per), BS.groups(N, True, per)
    assert np.abs(_apply(F, _bitrev(w)) - z).max() < 1e-9
    assert np.abs(_apply(G, z) / S - _bitrev(w)).max() < 1e-9
    assert len(F) == len(G) == -(-int(math.log2(S)) // per)


@pytest.mark.parametrize("per", [3, 5])
def test_bootstrap_refreshes_a_level0_ciphertext(ctx, per):
    """per 5 at this ring: a group of 63 offsets over 32 distinct rotations, folded mod S."""
    c = ctx
    prm = BS.Params(N, K=24, r=3, per_group=per)
    ops = OracleOps(c)
    rng = np.random.default_rng(5)
    z = rng.uniform(-1, 1, S)
    ct = ops.encrypt(z, 0, 2.0**40, S)
    bt = BS.Bootstrapper(ops, prm, c.q, c.q[0])
    out = bt(ct, len(c.q) - 1)
    ng = len(BS.groups(N, True, per))  # CoeffToSlot and SlotToCoeff: one level per group; EvalMod 7 + r
    assert out.top == len(c.q) - 1 - (ng + 7 + prm.r + ng)
    got = ops.decrypt_slots(out)
    assert np.abs(got.real - z).max() < 1e-4 and np.abs(got.imag).max() < 1e-4
    # the refreshed ciphertext computes: one more product at its level
    sq = ops.rescale_one(ops.mult(out, out))
    assert np.abs(ops.decrypt_slots(sq).real - z * z).max() < 1e-4
