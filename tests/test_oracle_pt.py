"""The oracle's plaintext-operand kernels pinned to the reference's own launcher self-test formula
(crates/pc-kernels/src/bin/selftest.rs:678-745: the expected words are exact u128 sums of rotation x diagonal
products reduced mod p, with the compact index i >> 1 for enc 0x7F000001), computed here with Python integers."""
import numpy as np
import pytest

from tests import _oracle as O

LOGN = 5
N = 1 << LOGN


def _primes():
    return O.ntt_primes(50, 10, 3) + O.ntt_primes(60, 10, 2)


@pytest.mark.parametrize("enc,ptw", [(0xFFFFFFFF, N), (0x7F000001, N // 2), (N // 4 - 1, N // 4)])
def test_pt_dot_matches_selftest_formula(enc, ptw):
    # selftest.rs:680: (k, bstep, gstep, npts, pt_prow) = (3, 3, 2, 5, 3) over 3 Q rows and 2 special rows
    K, bstep, gstep, npts, pt_prow = 3, 3, 2, 5, 3
    primes = _primes()
    rng = np.random.default_rng(5)
    rows = len(primes)
    prow = [y if y < 3 else pt_prow + y - 3 for y in range(rows)]
    rot = np.stack([rng.integers(0, p, (K, bstep, 2, N), dtype=np.uint64) for p in primes], 3)
    pts = np.zeros((npts, max(prow) + 1, ptw), np.uint64)
    for y, p in enumerate(primes):
        pts[:, prow[y]] = rng.integers(0, p, (npts, ptw), dtype=np.uint64)
    got = O.pt_dot(rot, pts, primes, prow, gstep, enc)
    for c in range(K):
        for j in range(gstep):
            for y, p in enumerate(primes):
                for part in range(2):
                    for i in range(N):
                        pi = i if enc == 0xFFFFFFFF else (i >> 1 if enc >> 24 == 0x7F else i & enc)
                        s = 0
                        for b in range(bstep):
                            d = bstep * j + b
                            if d >= npts:
                                break
                            s += int(rot[c, b, part, y, i]) * int(pts[d, prow[y], pi])
                        assert int(got[c, j, part, y, i]) == s % p


def test_mul_rows_and_row_adds():
    primes = _primes()
    rng = np.random.default_rng(6)
    x = np.stack([rng.integers(0, p, (2, 2, N), dtype=np.uint64) for p in primes], 2)
    t = np.stack([rng.integers(0, p, N, dtype=np.uint64) for p in primes])
    m = O.mul_rows(x, t, primes)
    a = O.add_rows(x, m, primes)
    s = O.sub_rows(x, m, primes)
    for y, p in enumerate(primes):
        xs, ts = x[:, :, y].astype(object), t[y].astype(object)
        assert (m[:, :, y].astype(object) == xs * ts % p).all()
        assert (a[:, :, y].astype(object) == (xs + xs * ts % p) % p).all()
        assert (s[:, :, y].astype(object) == (xs - xs * ts % p) % p).all()
