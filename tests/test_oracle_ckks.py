"""The oracle's homomorphic ops decrypt to the plaintext results: decrypt(eval(enc(x))) ~ f(x).

Small rings (N = 2^10) so the pure-CPU suite stays fast; the same code paths run at the BASELINE sizes in the GPU
parity tests. The parameter shape mirrors BASELINE config 1 (50-bit Q primes, one 60-bit special prime, one limb per
digit) and config 2 (several limbs per digit, several special primes).
"""
import numpy as np
import pytest

from tests import _oracle as O

LOGN = 10
N = 1 << LOGN
SLOTS = N // 2
SCALE = 2.0**40


def make_ctx(nq=4, kp=1, dnum=4, pbits=60, steps=(1, 2, 4, -1)):
    q = O.ntt_primes(50, LOGN, nq)
    p = O.ntt_primes(pbits, LOGN, kp, skip=nq if pbits == 50 else 0)
    c = O.Ctx(LOGN, q, p, dnum)
    gal = [1] + [O.lib().orc_rotation_galois(s, LOGN) for s in steps]
    c.keygen(seed=0, h=192, sigma=3.2, galois=gal)
    return c


@pytest.fixture(scope="module")
def ctx():
    return make_ctx()


@pytest.fixture(scope="module")
def ctx3():
    # three limbs per digit (dnum 2 over 6 limbs), two 50-bit special primes: config 2's structure
    return make_ctx(nq=6, kp=3, dnum=2, pbits=50)


def vals(seed, n=SLOTS, scale=1.0):
    r = np.random.default_rng(seed)
    return r.normal(0, 1, n) * scale


def test_encrypt_decrypt(ctx):
    x = vals(1)
    top = ctx.nq - 1
    ct = ctx.encrypt(x, SLOTS, SCALE, top)
    y = ctx.decrypt(ct, top, SLOTS, SCALE)
    assert np.abs(y.real - x).max() < 1e-7


def test_secret_weight(ctx):
    s = ctx.secret()
    assert int((s != 0).sum()) == 192


@pytest.mark.parametrize("which", ["ctx", "ctx3"])
def test_mult_relin_rescale(which, request):
    c = request.getfixturevalue(which)
    top = c.nq - 1
    x, y = vals(2), vals(3)
    a = c.encrypt(x, SLOTS, SCALE, top)
    b = c.encrypt(y, SLOTS, SCALE, top)
    m = c.mult(a, b, top)
    # decode reads the bottom prime only (crates/pc-core/src/encode.rs:236-268): rescale before decrypting
    r = c.rescale(m, top)
    got = c.decrypt(r, top - 1, SLOTS, SCALE * SCALE / c.q[top])
    assert np.abs(got.real - x * y).max() < 1e-4


@pytest.mark.parametrize("which", ["ctx", "ctx3"])
@pytest.mark.parametrize("step", [1, 4, -1])
def test_rotate(which, step, request):
    c = request.getfixturevalue(which)
    top = c.nq - 1
    x = vals(4)
    ct = c.encrypt(x, SLOTS, SCALE, top)
    r = c.rotate(ct, step, top)
    got = c.decrypt(r, top, SLOTS, SCALE)
    assert np.abs(got.real - np.roll(x, -step)).max() < 1e-6


def test_rotate_lower_level(ctx3):
    # key switching below the top: live digits and limbs cut at the level (crates/pc-gpu/src/ks.rs:579-582)
    c = ctx3
    top = 3
    x = vals(5)
    ct = c.encrypt(x, SLOTS, SCALE, top)
    r = c.rotate(ct, 2, top)
    got = c.decrypt(r, top, SLOTS, SCALE)
    assert np.abs(got.real - np.roll(x, -2)).max() < 1e-6


def test_rotate_and_sum(ctx):
    top = ctx.nq - 1
    x = vals(6)
    ct = ctx.encrypt(x, SLOTS, SCALE, top)
    r = ctx.rotate_and_sum(ct, 1, 8, top)
    got = ctx.decrypt(r, top, SLOTS, SCALE)
    want = sum(np.roll(x, -k) for k in range(8))
    assert np.abs(got.real - want).max() < 1e-5


@pytest.fixture(scope="module")
def ctx_r():
    # keys for radix-2 groups of gaps 1, 2 (steps 1, 2, 3) and 4, 8 (steps 4, 8, 12), plus rung steps
    return make_ctx(nq=6, kp=3, dnum=2, pbits=50, steps=(1, 2, 3, 4, 8, 12, 16, -1, -2, -3))


def test_rotate_sum(ctx_r):
    """out = x + sum rot(x, s): the rotations summed in the extended basis, one ModDown (the reference's rotate_sum)."""
    top = ctx_r.nq - 1
    x = vals(16)
    ct = ctx_r.encrypt(x, SLOTS, SCALE, top)
    got = ctx_r.decrypt(ctx_r.rotate_sum(ct, [1, 2, 3], top), top, SLOTS, SCALE).real
    want = x + np.roll(x, -1) + np.roll(x, -2) + np.roll(x, -3)
    assert np.abs(got - want).max() < 1e-5
    # a step of Galois element 1 is refused, as in a reference group
    with pytest.raises(AssertionError):
        ctx_r.rotate_sum(ct, [SLOTS], top)


@pytest.mark.parametrize("start,stop,radix", [(1, 16, 2), (1, 32, 2), (-1, 4, 2), (1, 8, 3)])
def test_rotate_and_sum_radix(ctx_r, start, stop, radix):
    """The radix ladder: groups with keys go through rotate_sum, the rest rung by rung; the same sum as the rungs."""
    top = ctx_r.nq - 1
    x = vals(17)
    ct = ctx_r.encrypt(x, SLOTS, SCALE, top)
    got = ctx_r.decrypt(ctx_r.rotate_and_sum(ct, start, stop, top, radix), top, SLOTS, SCALE).real
    want = sum(np.roll(x, -start * k) for k in range(stop // abs(start)))
    assert np.abs(got - want).max() < 1e-4


def test_mult_pt_and_add_pt(ctx):
    top = ctx.nq - 1
    x, w = vals(7), vals(8)
    ct = ctx.encrypt(x, SLOTS, SCALE, top)
    pt = ctx.encode(w, SLOTS, SCALE, top)
    prod = ctx.rescale(ctx.mult_pt(ct, pt, top), top)
    got = ctx.decrypt(prod, top - 1, SLOTS, SCALE * SCALE / ctx.q[top])
    assert np.abs(got.real - x * w).max() < 1e-4
    got = ctx.decrypt(ctx.add_pt(ct, pt, top), top, SLOTS, SCALE)
    assert np.abs(got.real - (x + w)).max() < 1e-6


def test_determinism(ctx):
    # the same seed reproduces keys and encryptions word for word (the parity tests rely on it)
    c2 = make_ctx()
    for i in range(3):
        b1, a1, s1 = ctx.key(i)
        b2, a2, s2 = c2.key(i)
        assert (b1 == b2).all() and (a1 == a2).all() and (s1 == s2).all()


def bsgs_diagonals(diags, bstep, stride):
    """The plaintext vectors of a BSGS product: diagonal d = bstep j + b pre-rotated by -bstep j stride."""
    return [np.roll(v, (d // bstep) * bstep * stride) for d, v in enumerate(diags)]


def eval_pts(ctx, vecs, scale, top):
    pts = np.zeros((len(vecs), ctx.nq, N), np.uint64)
    for d, v in enumerate(vecs):
        rows = ctx.encode(v, SLOTS, scale, top)
        O.lib().orc_ntt_fwd(rows, top + 1, np.asarray(ctx.q[: top + 1], np.uint64), LOGN)
        pts[d, : top + 1] = rows
    return pts


@pytest.mark.parametrize("npts,bstep", [(8, 4), (7, 4), (3, 4), (6, 2)])
def test_linear_transform(ctx_r, npts, bstep):
    """The BSGS product decrypts to sum_d diag_d * rot(x, d) (the generalized diagonal method), ragged last giant
    steps and a single giant step included."""
    top = ctx_r.nq - 1
    x = vals(18)
    rng = np.random.default_rng(19)
    diags = [rng.normal(0, 1, SLOTS) for _ in range(npts)]
    ct = ctx_r.encrypt(x, SLOTS, SCALE, top)
    pscale = float(ctx_r.q[top])
    pts = eval_pts(ctx_r, bsgs_diagonals(diags, bstep, 1), pscale, top)
    out = ctx_r.rescale(ctx_r.linear_transform(ct, pts, bstep, 1, top), top)
    got = ctx_r.decrypt(out, top - 1, SLOTS, SCALE).real
    want = sum(dg * np.roll(x, -d) for d, dg in enumerate(diags))
    assert np.abs(got - want).max() < 1e-4


def eval_pts_ext(ctx, vecs, scale, top):
    primes = list(ctx.q[: top + 1]) + list(ctx.p)
    pts = np.zeros((len(vecs), len(primes), N), np.uint64)
    for d, v in enumerate(vecs):
        rows = ctx.encode_ext(v, SLOTS, scale, top)
        O.lib().orc_ntt_fwd(rows, len(primes), np.asarray(primes, np.uint64), LOGN)
        pts[d] = rows
    return pts


@pytest.mark.parametrize("npts,bstep,top", [(8, 4, 5), (7, 4, 5), (3, 4, 5), (12, 4, 3), (16, 16, 5)])
def test_linear_transform_ext(ctx_r, npts, bstep, top):
    """The double-hoisted BSGS product (babies in the extended basis, no baby ModDown; plaintexts over the special
    primes too) decrypts to sum_d diag_d * rot(x, d) as the plain product does (within the key-switch noise), at the
    top level and below it; a single giant step and 16 babies included. The two forms round at other points."""
    x = vals(18)
    rng = np.random.default_rng(19)
    diags = [rng.normal(0, 1, SLOTS) for _ in range(npts)]
    ct = ctx_r.encrypt(x, SLOTS, SCALE, top)
    pscale = float(ctx_r.q[top])
    vecs = bsgs_diagonals(diags, bstep, 1)
    want = sum(dg * np.roll(x, -d) for d, dg in enumerate(diags))
    if bstep <= 4:  # the plain form with the same keys
        ref = ctx_r.rescale(ctx_r.linear_transform(ct, eval_pts(ctx_r, vecs, pscale, top), bstep, 1, top), top)
        assert np.abs(ctx_r.decrypt(ref, top - 1, SLOTS, SCALE).real - want).max() < 1e-4
    else:  # keys for every baby step
        ctx_r = make_ctx(nq=6, kp=3, dnum=2, pbits=50, steps=tuple(range(1, bstep)))
        ct = ctx_r.encrypt(x, SLOTS, SCALE, top)
    ext = ctx_r.linear_transform_ext(ct, eval_pts_ext(ctx_r, vecs, pscale, top), bstep, 1, top)
    got = ctx_r.decrypt(ctx_r.rescale(ext, top), top - 1, SLOTS, SCALE).real
    assert np.abs(got - want).max() < 1e-4


@pytest.mark.parametrize("off", [-1, -2])
def test_linear_transform_ext_baby_offset(ctx_r, off):
    """A baby offset folds a rotation of the input into the babies: the product of rot(x, off) without that rotation
    (babies x rotated by b + off, the identity among them as P x)."""
    top, bstep, npts = 5, 4, 8
    x = vals(20)
    rng = np.random.default_rng(21)
    diags = [rng.normal(0, 1, SLOTS) for _ in range(npts)]
    ct = ctx_r.encrypt(x, SLOTS, SCALE, top)
    pts = eval_pts_ext(ctx_r, bsgs_diagonals(diags, bstep, 1), float(ctx_r.q[top]), top)
    out = ctx_r.linear_transform_ext(ct, pts, bstep, 1, top, baby_offset=off)
    got = ctx_r.decrypt(ctx_r.rescale(out, top), top - 1, SLOTS, SCALE).real
    want = sum(dg * np.roll(x, -(d + off)) for d, dg in enumerate(diags))
    assert np.abs(got - want).max() < 1e-4


def test_hoisted_rotations_equal_plain_ones():
    """orc_rotate_hoisted (one ModUp for every step) = orc_rotate step by step, word for word; a step of galois 1
    copies."""
    logn = 10
    q = O.ntt_primes(50, logn, 6)
    p = O.ntt_primes(50, logn, 2, skip=6)
    steps = [1, 3, 5, 1 << (logn - 1)]
    c = O.Ctx(logn, q, p, 3)
    c.keygen(0, 32, 3.2, [1] + [pow(5, s % (1 << (logn - 1)), 2 << logn) for s in steps[:3]])
    rng = np.random.default_rng(7)
    x = c.ct()
    for r in range(len(q)):
        x[:, r] = rng.integers(0, q[r], (2, 1 << logn), dtype=np.uint64)
    for top in (len(q) - 1, 2):
        outs = c.rotate_hoisted(x, steps, top)
        for s, o in zip(steps[:3], outs):
            assert (o[:, : top + 1] == c.rotate(x, s, top)[:, : top + 1]).all(), (top, s)
        assert (outs[3][:, : top + 1] == x[:, : top + 1]).all()
