"""The plaintext-operand table entries (pt_dot, mul_table, mul_add, mul_add_n, add_const) against the oracle, word
for word, through the reference-compatible launcher table (crates/pc-kernels/kernels/args.cuh:184-200, :491-528).

The pt_dot cases follow the reference's own launcher self-test (crates/pc-kernels/src/bin/selftest.rs:678-745:
K = 3 ciphertexts, 3 baby steps, 2 giant steps, 5 diagonals, a row set with special rows read at pt_prow, full and
compact plaintext indices) and widen it to every K bucket, a giant step count that leaves diagonals missing and the
single-giant-step form with res_stride 0. Rows mix 50-bit and 60-bit primes so the 128-bit sums run near their
bound.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from perseus_b200 import _lib as L
from tests import _oracle as O

pytestmark = pytest.mark.gpu

LOGN = 16
N = 1 << LOGN
R = 12  # rows per part in the test layout (prime ids 0..11)


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()


def ptr(x):
    return C.cast(C.pointer(x), C.c_void_p)


@pytest.fixture(scope="module")
def env():
    primes = O.ntt_primes(50, LOGN, 8) + O.ntt_primes(60, LOGN, 4)
    pc = np.zeros((R, 8), np.uint64)
    for i, p in enumerate(primes):
        O.lib().orc_prime_const(p, pc[i])
    return np.array(primes, np.uint64), dev(pc), L.kernel_table()


def rand_cts(rng, primes, K, rows=R):
    """K ciphertexts [K][2][rows][N], row r canonical mod primes[r]."""
    x = np.empty((K, 2, rows, N), np.uint64)
    for r in range(rows):
        x[:, :, r] = rng.integers(0, primes[r], (K, 2, N), dtype=np.uint64)
    return x


def rand_rows(rng, primes, rows=R):
    return np.stack([rng.integers(0, primes[r], N, dtype=np.uint64) for r in range(rows)])


def cref(t, K=None):
    """PolyRef of a [K][2][R][N] buffer."""
    return L.PolyRef(t.data_ptr(), 2 * R * N, R * N)


def test_mul_table(env):
    primes, pc, tab = env
    rng = np.random.default_rng(1)
    K, n = 3, 10
    x, t = rand_cts(rng, primes, K), rand_rows(rng, primes)
    xd, td = dev(x), dev(t)
    out = torch.zeros_like(xd)
    a = L.MulTableArgs(cref(out), cref(xd), td.data_ptr(), pc.data_ptr(), n, K)
    assert tab.mul_table(ptr(a), None) == 0
    want = np.zeros_like(x)
    want[:, :, :n] = O.mul_rows(x[:, :, :n], t[:n], primes[:n])
    assert (host(out) == want).all()
    # in place (out == in)
    a = L.MulTableArgs(cref(xd), cref(xd), td.data_ptr(), pc.data_ptr(), n, K)
    assert tab.mul_table(ptr(a), None) == 0
    want[:, :, n:] = x[:, :, n:]
    assert (host(xd) == want).all()


@pytest.mark.parametrize("sub", [0, 1, 2])
def test_mul_add(env, sub):
    primes, pc, tab = env
    rng = np.random.default_rng(2 + sub)
    K, n = 2, R
    x, y, t = rand_cts(rng, primes, K), rand_cts(rng, primes, K), rand_rows(rng, primes)
    xd, yd, td = dev(x), dev(y), dev(t)
    m = L.MulTableArgs(cref(yd), cref(xd), td.data_ptr(), pc.data_ptr(), n, K)  # out aliases y
    a = L.MulAddArgs(m, cref(yd), sub, 0)
    assert tab.mul_add(ptr(a), None) == 0
    prod = O.mul_rows(x, t, primes)
    want = O.add_rows(y, prod, primes) if sub == 0 else O.sub_rows(y, prod, primes) if sub == 1 else \
        O.sub_rows(prod, y, primes)
    assert (host(yd) == want).all()


@pytest.mark.parametrize("nterm,with_y,lazy", [(1, True, 1), (3, False, 0), (8, True, 1), (8, True, 0)])
def test_mul_add_n(env, nterm, with_y, lazy):
    primes, pc, tab = env
    rng = np.random.default_rng(10 + nterm)
    K, n = 2, 9
    xs = [rand_cts(rng, primes, K) for _ in range(nterm)]
    ts = [rand_rows(rng, primes) for _ in range(nterm)]
    y = rand_cts(rng, primes, K)
    xds, tds, yd = [dev(v) for v in xs], [dev(v) for v in ts], dev(y)
    out = xds[0] if nterm > 1 else torch.zeros_like(yd)  # out may alias a term's operand
    a = L.MulAddNArgs()
    a.out, a.y = cref(out), (cref(yd) if with_y else L.PolyRef())
    for j in range(nterm):
        a.x[j], a.t[j] = cref(xds[j]), tds[j].data_ptr()
    a.pr, a.n, a.K, a.nterm, a.lazy = pc.data_ptr(), n, K, nterm, lazy
    assert tab.mul_add_n(ptr(a), None) == 0
    want = y[:, :, :n].copy() if with_y else np.zeros((K, 2, n, N), np.uint64)
    for j in range(nterm):
        want = O.add_rows(want, O.mul_rows(xs[j][:, :, :n], ts[j][:n], primes[:n]), primes[:n])
    got = host(out)
    assert (got[:, :, :n] == want).all()
    untouched = xs[0] if nterm > 1 else np.zeros_like(y)
    assert (got[:, :, n:] == untouched[:, :, n:]).all()


def test_add_const(env):
    primes, pc, tab = env
    rng = np.random.default_rng(20)
    K, n = 3, 11
    x = rand_cts(rng, primes, K)
    k = np.array([rng.integers(0, p) for p in primes], np.uint64)
    k[1], k[9] = primes[1], primes[9]  # the raw word p (reduced to 0 by the kernel)
    xd, kd = dev(x), dev(k)
    a = L.AddConstArgs(cref(xd), kd.data_ptr(), pc.data_ptr(), n, K)
    assert tab.add_const(ptr(a), None) == 0
    kr = np.where(k >= primes, k - primes, k)
    want = x.copy()
    want[:, 0, :n] = O.add_rows(x[:, 0, :n], np.broadcast_to(kr[:n, None], (n, N)), primes[:n])
    assert (host(xd) == want).all()


def _pt_dot_case(env, K, bstep, gstep, npts, enc, ptw, rs, pt_prow, res_stride0=False, seed=30):
    primes, pc, tab = env
    rng = np.random.default_rng(seed + K)
    nq, np_, qmax = rs
    ids = list(range(nq)) + [qmax + i for i in range(np_)]
    prow = [y if y < nq else pt_prow + (y - nq) for y in range(len(ids))]
    nprow = max(prow) + 1
    # baby rotations: [K][bstep] ciphertexts of the test layout (rot_stride one ciphertext)
    rot = rand_cts(rng, primes, K * bstep).reshape(K, bstep, 2, R, N)
    # plaintext rows: row prow[y] reduced mod the prime of grid row y (rows no grid row reads stay random)
    pts = rng.integers(0, 1 << 49, (npts, nprow, ptw), dtype=np.uint64)
    for y, pid in enumerate(ids):
        pts[:, prow[y]] = rng.integers(0, primes[pid], (npts, ptw), dtype=np.uint64)
    rotd = dev(rot)
    ptds = [dev(pts[d]) for d in range(npts)]
    tabd = dev(np.array([t.data_ptr() for t in ptds], np.uint64))
    ncts = K * (1 if res_stride0 else gstep)
    res = torch.zeros((ncts, 2, R, N), dtype=torch.int64, device="cuda")
    a = L.PtDotArgs()
    a.rot = L.PolyRef(rotd.data_ptr(), bstep * 2 * R * N, R * N)
    a.res = L.PolyRef(res.data_ptr(), (1 if res_stride0 else gstep) * 2 * R * N, R * N)
    a.rot_stride, a.res_stride = 2 * R * N, 0 if res_stride0 else 2 * R * N
    a.pts, a.pr = tabd.data_ptr(), pc.data_ptr()
    a.rs = L.RowSet(nq, np_, qmax, 0)
    a.npts, a.bstep, a.gstep, a.K, a.ptw, a.pt_prow, a.enc = npts, bstep, gstep, K, ptw, pt_prow, enc
    assert tab.pt_dot(ptr(a), None) == 0
    want = O.pt_dot(rot[:, :, :, ids], pts, primes[ids], prow, gstep, enc)
    got = host(res).reshape(K, -1, 2, R, N)
    if res_stride0:
        assert (got[:, 0][:, :, ids] == want[:, 0]).all()
    else:
        assert (got[:, :, :, ids] == want).all()
    others = [r for r in range(R) if r not in ids]
    assert (got[:, :, :, others] == 0).all()


@pytest.mark.parametrize("enc,ptw", [(0xFFFFFFFF, N), (0x7F000001, N // 2), (N // 4 - 1, N // 4)])
def test_pt_dot_selftest_shape(env, enc, ptw):
    # selftest.rs:680: (k, bstep, gstep, npts, pt_prow) = (3, 3, 2, 5, 3); Q rows 0..2 and two special rows
    _pt_dot_case(env, 3, 3, 2, 5, enc, ptw, rs=(3, 2, 8), pt_prow=3)


@pytest.mark.parametrize("K", [1, 2, 4, 5, 8])
def test_pt_dot_batches(env, K):
    _pt_dot_case(env, K, bstep=4, gstep=3, npts=10, enc=0xFFFFFFFF, ptw=N, rs=(6, 2, 10), pt_prow=6)


def test_pt_dot_single_giant_step(env):
    # the form of a per-member dot (crates/pc-gpu/src/bts/spru.rs:570-588): gstep 1, res_stride 0, Q rows only
    _pt_dot_case(env, 1, bstep=8, gstep=1, npts=8, enc=0xFFFFFFFF, ptw=N, rs=(12, 0, 12), pt_prow=0, res_stride0=True)

