"""ctypes binding of the parity oracle (oracle/liboracle.so) — test infrastructure only.

The oracle is a CPU restatement of the reference's u64 hot path; tests compare the CUDA path against it. It is built
from oracle/Makefile on first use.
"""
import ctypes as C
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ODIR = os.path.join(ROOT, "oracle")
LIB = os.path.join(ODIR, "_build", "liboracle.so")

_lib = None

u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")

TAG_KSKA = 0x4B534B41
TAG_ENCA = 0x454E4341


def lib():
    global _lib
    if _lib is not None:
        return _lib
    src = [os.path.join(ODIR, f) for f in ("oracle.cpp", "oracle.h", "Makefile")]
    if not os.path.exists(LIB) or any(os.path.getmtime(s) > os.path.getmtime(LIB) for s in src):
        subprocess.run(["make", "-s", "-C", ODIR], check=True)
    L = C.CDLL(LIB)
    sig = {
        "orc_prime_const": (None, [C.c_uint64, u64p]),
        "orc_reduce128": (C.c_uint64, [C.c_uint64, C.c_uint64, C.c_uint64]),
        "orc_mulmod": (C.c_uint64, [C.c_uint64] * 3),
        "orc_powmod": (C.c_uint64, [C.c_uint64] * 3),
        "orc_invmod": (C.c_uint64, [C.c_uint64] * 2),
        "orc_is_prime": (C.c_int, [C.c_uint64]),
        "orc_first_prime": (C.c_uint64, [C.c_uint32, C.c_uint64]),
        "orc_previous_prime": (C.c_uint64, [C.c_uint64, C.c_uint64]),
        "orc_root_of_unity": (C.c_uint64, [C.c_uint64, C.c_uint64]),
        "orc_ntt_primes": (None, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, u64p]),
        "orc_automorph_slot": (C.c_uint32, [C.c_uint32, C.c_uint32, C.c_uint32]),
        "orc_rotation_galois": (C.c_uint64, [C.c_int64, C.c_uint32]),
        "orc_galois_inverse": (C.c_uint64, [C.c_uint64, C.c_uint32]),
        "orc_chacha_block": (None, [u32p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, u32p]),
        "orc_expand_row_u64": (None, [u32p, C.c_uint32, C.c_uint64, C.c_uint32, C.c_uint32, u64p]),
        "orc_prng_new": (C.c_void_p, [u32p, C.c_uint32]),
        "orc_prng_free": (None, [C.c_void_p]),
        "orc_prng_u32": (C.c_uint32, [C.c_void_p]),
        "orc_prng_u64": (C.c_uint64, [C.c_void_p]),
        "orc_prng_below": (C.c_uint64, [C.c_void_p, C.c_uint64]),
        "orc_prng_f64": (C.c_double, [C.c_void_p]),
        "orc_sample_sparse_ternary": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, i8p]),
        "orc_sample_ternary": (None, [C.c_void_p, C.c_uint32, i8p]),
        "orc_sample_gaussian": (None, [C.c_void_p, C.c_double, C.c_uint32, i64p]),
        "orc_twiddles": (None, [C.c_uint64, C.c_uint64, C.c_uint32, u64p, u64p, u64p, u64p]),
        "orc_ntt_fwd": (None, [u64p, C.c_int, u64p, C.c_uint32]),
        "orc_ntt_inv": (None, [u64p, C.c_int, u64p, C.c_uint32]),
        "orc_ctx_new": (C.c_void_p, [C.c_uint32, C.c_int, u64p, C.c_int, u64p, C.c_int]),
        "orc_ctx_free": (None, [C.c_void_p]),
        "orc_ctx_rows": (C.c_int, [C.c_void_p]),
        "orc_set_threads": (None, [C.c_int]),
        "orc_get_threads": (C.c_int, []),
        "orc_keygen": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint32, C.c_double, C.c_int, u64p]),
        "orc_secret": (None, [C.c_void_p, i8p]),
        "orc_key": (C.c_int, [C.c_void_p, C.c_int, u64p, u64p, u32p]),
        "orc_encode": (C.c_int, [C.c_void_p, f64p, C.c_int, C.c_int, C.c_double, C.c_int, u64p]),
        "orc_encode_ext": (C.c_int, [C.c_void_p, f64p, C.c_int, C.c_int, C.c_double, C.c_int, u64p]),
        "orc_linear_transform_ext": (C.c_int, [C.c_void_p, u64p, u64p, C.c_int, C.c_int, C.c_int64, C.c_int64, u64p,
                                               C.c_int]),
        "orc_decode": (C.c_int, [C.c_void_p, u64p, C.c_int, C.c_double, f64p]),
        "orc_encrypt": (C.c_int, [C.c_void_p, f64p, C.c_int, C.c_int, C.c_double, C.c_int, u64p]),
        "orc_decrypt": (C.c_int, [C.c_void_p, u64p, C.c_int, C.c_int, C.c_double, f64p]),
        "orc_add": (C.c_int, [C.c_void_p, u64p, u64p, u64p, C.c_int]),
        "orc_sub": (C.c_int, [C.c_void_p, u64p, u64p, u64p, C.c_int]),
        "orc_mult": (C.c_int, [C.c_void_p, u64p, u64p, u64p, C.c_int]),
        "orc_tensor": (C.c_int, [C.c_void_p, u64p, u64p, u64p, u64p, C.c_int]),
        "orc_rescale": (C.c_int, [C.c_void_p, u64p, C.c_int]),
        "orc_mod_raise": (C.c_int, [C.c_void_p, u64p, C.c_int]),
        "orc_rotate": (C.c_int, [C.c_void_p, u64p, C.c_int64, u64p, C.c_int]),
        "orc_rotate_and_sum": (C.c_int, [C.c_void_p, u64p, C.c_int64, C.c_int64, u64p, C.c_int]),
        "orc_rotate_sum": (C.c_int, [C.c_void_p, u64p, C.c_void_p, C.c_int, u64p, C.c_int]),
        "orc_rotate_and_sum_radix": (C.c_int, [C.c_void_p, u64p, C.c_int64, C.c_int64, C.c_int, u64p, C.c_int]),
        "orc_mult_pt_rows": (C.c_int, [C.c_void_p, u64p, u64p, u64p, C.c_int]),
        "orc_add_pt_rows": (C.c_int, [C.c_void_p, u64p, u64p, u64p, C.c_int]),
        "orc_keyswitch_ext": (C.c_int, [C.c_void_p, u64p, u64p, C.c_int, C.c_int, C.c_uint32, u64p, C.c_int]),
        "orc_moddown": (C.c_int, [C.c_void_p, u64p, u64p, C.c_int]),
        "orc_ntt_batch": (C.c_int, [C.c_void_p, u64p, C.c_int, C.c_int]),
        "orc_rotate_batch": (C.c_int, [C.c_void_p, u64p, C.c_int, C.c_int64, u64p, C.c_int]),
        "orc_rotate_hoisted": (C.c_int, [C.c_void_p, u64p, C.c_void_p, C.c_int, C.c_void_p, C.c_int]),
        "orc_linear_transform": (C.c_int, [C.c_void_p, u64p, u64p, C.c_int, C.c_int, C.c_int64, u64p, C.c_int]),
        "orc_mul_rows": (C.c_int, [u64p, u64p, u64p, u64p, C.c_int, C.c_int, C.c_int]),
        "orc_pt_dot": (C.c_int, [u64p, u64p, u64p, u64p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                 C.c_int, C.c_int, C.c_int, C.c_uint32]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def ntt_primes(bits, logn, count, skip=0):
    out = np.zeros(count, np.uint64)
    lib().orc_ntt_primes(bits, logn, skip, count, out)
    return [int(x) for x in out]


def expand_row(seed, w13, p, tag, logn):
    out = np.zeros(1 << logn, np.uint64)
    lib().orc_expand_row_u64(np.asarray(seed, np.uint32), w13, p, tag, logn, out)
    return out


def mul_rows(x, t, primes):
    """x [..., nrows, N] times t [nrows, N] row-wise mod primes[row] (the mul_table product)."""
    x = np.ascontiguousarray(x, np.uint64)
    t = np.ascontiguousarray(t, np.uint64)
    nrows, n = t.shape
    out = np.empty_like(x)
    rc = lib().orc_mul_rows(x, t, out, np.asarray(primes, np.uint64), nrows, n.bit_length() - 1, x.size // (nrows * n))
    assert rc == 0
    return out


def pt_dot(rot, pts, primes, prow, gstep, enc=0xFFFFFFFF):
    """rot [K][bstep][2][nrows][N], pts [npts][nprow][ptw] -> res [K][gstep][2][nrows][N] (the BSGS plaintext dot)."""
    rot = np.ascontiguousarray(rot, np.uint64)
    pts = np.ascontiguousarray(pts, np.uint64)
    K, bstep, _, nrows, n = rot.shape
    npts, nprow, ptw = pts.shape
    res = np.zeros((K, gstep, 2, nrows, n), np.uint64)
    pr = np.asarray(prow, np.int32)
    rc = lib().orc_pt_dot(rot, res, pts, np.asarray(primes, np.uint64), pr.ctypes.data, nrows, n.bit_length() - 1, K,
                          bstep, gstep, npts, ptw, nprow, enc)
    assert rc == 0
    return res


def add_rows(a, b, primes):
    """(a + b) mod p row-wise; a, b [..., nrows, N] canonical."""
    p = np.asarray(primes, np.uint64)[:, None]
    s = a + b
    return np.where(s >= p, s - p, s)


def sub_rows(a, b, primes):
    p = np.asarray(primes, np.uint64)[:, None]
    return np.where(a >= b, a - b, a + (p - b))


class Ctx:
    """An oracle CKKS context: Q primes q (bottom first), special primes p, dnum digits."""

    def __init__(self, logn, q, p, dnum):
        self.logn, self.n = logn, 1 << logn
        self.q, self.p, self.dnum = list(q), list(p), dnum
        self.nq, self.kp = len(q), len(p)
        self.rows = self.nq + self.kp
        self.h = lib().orc_ctx_new(logn, self.nq, np.asarray(q, np.uint64), self.kp, np.asarray(p, np.uint64), dnum)
        assert self.h, "orc_ctx_new refused the parameters"
        self.galois = []

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_ctx_free(self.h)
            self.h = None

    def ct(self):
        return np.zeros((2, self.rows, self.n), np.uint64)

    def keygen(self, seed, h, sigma, galois):
        self.galois = [int(g) for g in galois]
        rc = lib().orc_keygen(self.h, seed, h, sigma, len(galois), np.asarray(galois, np.uint64))
        assert rc == 0, rc

    def secret(self):
        s = np.zeros(self.n, np.int8)
        lib().orc_secret(self.h, s)
        return s

    def key(self, idx):
        b = np.zeros((self.dnum, self.rows, self.n), np.uint64)
        a = np.zeros_like(b)
        seed = np.zeros(8, np.uint32)
        assert lib().orc_key(self.h, idx, b, a, seed) == 0
        return b, a, seed

    def _vals(self, values):
        v = np.asarray(values, np.complex128).ravel()
        return np.ascontiguousarray(np.stack([v.real, v.imag], 1).ravel()), len(v)

    def encode(self, values, nslots, scale, top):
        vals, nv = self._vals(values)
        rows = np.zeros((top + 1, self.n), np.uint64)
        assert lib().orc_encode(self.h, vals, nv, nslots, scale, top, rows) == 0
        return rows

    def encode_ext(self, values, nslots, scale, top):
        """the encoding's rows over the Q primes 0..=top, then every special prime"""
        vals, nv = self._vals(values)
        rows = np.zeros((top + 1 + self.kp, self.n), np.uint64)
        assert lib().orc_encode_ext(self.h, vals, nv, nslots, scale, top, rows) == 0
        return rows

    def encrypt(self, values, nslots, scale, top):
        vals, nv = self._vals(values)
        ct = self.ct()
        assert lib().orc_encrypt(self.h, vals, nv, nslots, scale, top, ct) == 0
        return ct

    def decrypt(self, ct, top, nslots, scale):
        out = np.zeros(2 * nslots, np.float64)
        assert lib().orc_decrypt(self.h, np.ascontiguousarray(ct), top, nslots, scale, out) == 0
        return out[0::2] + 1j * out[1::2]

    def _bin(self, f, a, b, top):
        out = self.ct()
        rc = f(self.h, np.ascontiguousarray(a), np.ascontiguousarray(b), out, top)
        assert rc == 0, rc
        return out

    def add(self, a, b, top):
        return self._bin(lib().orc_add, a, b, top)

    def sub(self, a, b, top):
        return self._bin(lib().orc_sub, a, b, top)

    def mult(self, a, b, top):
        return self._bin(lib().orc_mult, a, b, top)

    def mult_pt(self, a, pt_rows, top):
        return self._bin(lib().orc_mult_pt_rows, a, pt_rows, top)

    def add_pt(self, a, pt_rows, top):
        return self._bin(lib().orc_add_pt_rows, a, pt_rows, top)

    def rescale(self, ct, top):
        x = np.ascontiguousarray(ct).copy()
        assert lib().orc_rescale(self.h, x, top) == 0
        return x

    def mod_raise(self, ct, top_out):
        x = np.ascontiguousarray(ct).copy()
        assert lib().orc_mod_raise(self.h, x, top_out) == 0
        return x

    def keyswitch(self, d, c0, c0_mode, kidx, autok, top):
        """ModUp(d), the inner product against key kidx (c0 mode, output at automorph_slot(autok, i)), ModDown."""
        ext = self.ct()
        rc = lib().orc_keyswitch_ext(self.h, np.ascontiguousarray(d), np.ascontiguousarray(c0) if c0 is not None
                                     else np.zeros((self.rows, self.n), np.uint64), c0_mode, kidx, autok, ext, top)
        assert rc == 0, rc
        out = self.ct()
        assert lib().orc_moddown(self.h, ext, out, top) == 0
        return out

    def rotate(self, ct, step, top):
        out = self.ct()
        rc = lib().orc_rotate(self.h, np.ascontiguousarray(ct), step, out, top)
        assert rc == 0, rc
        return out

    def rotate_hoisted(self, ct, steps, top):
        """One ModUp shared by every step (orc_rotate_hoisted): one output per step."""
        outs = [self.ct() for _ in steps]
        st = np.asarray(steps, np.int64)
        ptrs = (C.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
        rc = lib().orc_rotate_hoisted(self.h, np.ascontiguousarray(ct), st.ctypes.data, len(st), ptrs, top)
        assert rc == 0, rc
        return outs

    def rotate_and_sum(self, ct, start, stop, top, radix_bits=1):
        out = self.ct()
        if radix_bits >= 2:
            rc = lib().orc_rotate_and_sum_radix(self.h, np.ascontiguousarray(ct), start, stop, radix_bits, out, top)
        else:
            rc = lib().orc_rotate_and_sum(self.h, np.ascontiguousarray(ct), start, stop, out, top)
        assert rc == 0, rc
        return out

    def linear_transform(self, ct, pts, bstep, stride, top):
        """BSGS plaintext-matrix product; pts [npts][nq][N] evaluation-form plaintexts (diagonals pre-rotated)."""
        out = self.ct()
        pts = np.ascontiguousarray(pts, np.uint64)
        rc = lib().orc_linear_transform(self.h, np.ascontiguousarray(ct), pts, pts.shape[0], bstep, stride, out, top)
        assert rc == 0, rc
        return out

    def linear_transform_ext(self, ct, pts, bstep, stride, top, baby_offset=0):
        """The double-hoisted product; pts [npts][top + 1 + kp][N] evaluation-form plaintexts over the extended rows;
        baby b is ct rotated by (b + baby_offset) stride."""
        out = self.ct()
        pts = np.ascontiguousarray(pts, np.uint64)
        rc = lib().orc_linear_transform_ext(self.h, np.ascontiguousarray(ct), pts, pts.shape[0], bstep, stride,
                                            baby_offset, out, top)
        assert rc == 0, rc
        return out

    def rotate_sum(self, ct, steps, top):
        out = self.ct()
        st = np.asarray(steps, np.int64)
        rc = lib().orc_rotate_sum(self.h, np.ascontiguousarray(ct), st.ctypes.data, len(st), out, top)
        assert rc == 0, rc
        return out
