"""The projection layout without encryption (rotations as numpy rolls), then encrypted on the oracle: y = x W + b
read back from the output slots. The geometry of GPT-2's padded 1024-wide layer at 2^15 slots is the reference's
(python/perseus/impl/layout.py:77-98 cm_params: t 32, 32 plaintexts, 8 baby and 4 giant steps)."""
import numpy as np
import pytest

from perseus_b200 import linear as LIN
from tests import _oracle as O
from tests._oracle_ops import OracleOps


def rot(v, k):
    return np.roll(v, -k)


def ladder(v, start, stop):
    g = start
    while g < stop:
        v = v + rot(v, g)
        g *= 2
    return v


def test_gpt2_geometry():
    g = LIN.geometry(1 << 15, 1024, ext=False)  # the reference's split
    assert (g.t, g.npts, g.bstep, g.gstep, g.stride) == (32, 32, 8, 4, 1024)
    assert sorted(g.rot_steps()) == sorted([31, 62, 124, 248, 496] + [1024 * b for b in range(1, 8)] +
                                           [8192, 16384, 24576] + [1, 2, 4, 8, 16])
    g = LIN.geometry(1 << 15, 1024)  # the double-hoisted product's
    assert (g.t, g.npts, g.bstep, g.gstep, g.stride, g.ext) == (32, 32, 16, 2, 1024, True)
    assert sorted(g.rot_steps()) == sorted([31, 62, 124, 248, 496] + [1024 * b for b in range(1, 16)] +
                                           [16384] + [1, 2, 4, 8, 16])
    with pytest.raises(ValueError):
        LIN.geometry(1 << 15, 96)


@pytest.mark.parametrize("slots,d,n", [(1 << 15, 1024, 768), (512, 64, 50), (8192, 256, 256), (512, 32, 32)])
def test_layout_in_the_clear(slots, d, n):
    geo = LIN.geometry(slots, d)
    rng = np.random.default_rng(d)
    x, W, b = rng.normal(0, 1, n), rng.normal(0, 0.02, (n, n)), rng.normal(0, 0.1, n)
    X = ladder(LIN.input_vector(x, geo), *geo.prep_ladder())
    w = LIN.weight_vectors(W, geo)
    # BSGS with the giant pre-rotation, as the evaluator runs it
    pts = [np.roll(w[j], (j // geo.bstep) * geo.bstep * geo.stride) for j in range(geo.npts)]
    Y = np.zeros(slots)
    for g in range(geo.gstep):
        acc = sum(rot(X, b * geo.stride) * pts[g * geo.bstep + b] for b in range(geo.bstep))
        Y += rot(acc, g * geo.bstep * geo.stride)
    Y = ladder(Y, *geo.fold_ladder()) + LIN.bias_vector(b, geo)
    assert np.abs(LIN.output_values(Y, geo, n) - (x @ W + b)).max() < 1e-12


LOGN = 10


def test_linear_on_the_oracle():
    geo = LIN.geometry(1 << (LOGN - 1), 64)
    q = O.ntt_primes(50, LOGN, 5)
    p = O.ntt_primes(50, LOGN, 2, skip=5)
    c = O.Ctx(LOGN, q, p, 3)
    c.keygen(seed=0, h=192, sigma=3.2, galois=[1] + [O.lib().orc_rotation_galois(s, LOGN) for s in geo.rot_steps()])
    ops = OracleOps(c)
    rng = np.random.default_rng(3)
    n = 48
    x, W, b = rng.normal(0, 1, n), rng.normal(0, 0.02, (n, n)), rng.normal(0, 0.1, n)
    top = c.nq - 1
    ct = ops.encrypt(LIN.input_vector(x, geo), top, 2.0**40, geo.slots)
    lin = LIN.encode(ops, W, geo, top, ct.scale, bias=b)
    y = LIN.linear(ops, ct, lin)
    assert y.top == top - 1
    got = LIN.output_values(ops.decrypt_slots(y).real, geo, n)
    assert np.abs(got - (x @ W + b)).max() < 1e-5
