"""The evaluator API over the CUDA library, mirroring the reference's `Fhe` session (crates/pc-py/src/fhe.rs:770-1640):
encrypt, decrypt_slots, add, sub, mult, square, rescale_one, rotate, rotate_and_sum, mult_pt, add_pt, plus the
batched forms the benchmarks use. Device memory and streams come from torch; every op runs on the CUDA library
through its C ABI (there is no CPU path).

A `Ct` holds K ciphertexts [K][2][nq + kp][N] (uint64 residues viewed as torch.int64), its top limb, its scale and
its slot count. Products leave the rescale pending (scale = product of the scales), as the reference's relin::mult
does (crates/pc-gpu/src/relin.rs:1-4); `rescale_one` pays it.
"""
import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L

# ------------------------------------------------------------------------------------------------ chain helpers


def _is_prime(n):
    if n < 2:
        return False
    small = (2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37)
    for p in small:
        if n % p == 0:
            return n == p
    d, s = n - 1, 0
    while d % 2 == 0:
        d //= 2
        s += 1
    for a in small:
        x = pow(a, d, n)
        if x in (1, n - 1):
            continue
        for _ in range(s - 1):
            x = x * x % n
            if x == n - 1:
                break
        else:
            return False
    return True


def ntt_primes(bits, log_n, count, skip=0):
    """`count` primes p = 1 mod 2N just below 2^bits, largest first, after skipping `skip` of them
    (crates/pc-kernels/src/bin/selftest/host.rs:76-88)."""
    step = 2 << log_n
    c = (1 << bits) + 1
    out, seen = [], 0
    while len(out) < count:
        c -= step
        if _is_prime(c):
            if seen >= skip:
                out.append(c)
            seen += 1
    return out


@dataclass(frozen=True)
class Chain:
    """Explicit prime lists (the reference's Chain, crates/pc-core/src/params.rs:225-258)."""

    log_n: int
    q: tuple
    p: tuple
    dnum: int

    @property
    def n(self):
        return 1 << self.log_n

    @property
    def rows(self):
        return len(self.q) + len(self.p)


def config1_chain():
    """BASELINE config 1 made sound: N = 2^14, 8 x 50-bit Q primes, one 60-bit special prime, dnum 8 (one limb per
    digit, so the single special prime covers every digit)."""
    return Chain(14, tuple(ntt_primes(50, 14, 8)), tuple(ntt_primes(60, 14, 1)), 8)


def config2_chain():
    """N = 2^16, 24 x 50-bit Q primes + 8 x 50-bit special primes, dnum 3 (8 limbs per digit)."""
    return Chain(16, tuple(ntt_primes(50, 16, 24)), tuple(ntt_primes(50, 16, 8, skip=24)), 3)


def config4_chain():
    """BASELINE config 4 (bootstrapping): N = 2^16, 29 x 50-bit Q primes (the refresh spends 16 levels and leaves 12
    usable ones) + 11 x 50-bit special primes, dnum 3 (digits of 10 limbs: P one prime larger than a digit, so the
    key-switch noise stays below the rescale rounding)."""
    return Chain(16, tuple(ntt_primes(50, 16, 29)), tuple(ntt_primes(50, 16, 11, skip=29)), 3)


def rotation_galois(step, log_n):
    """5^(step mod N/2) mod 2N (crates/pc-core/src/galois.rs:38-44)."""
    h = 1 << (log_n - 1)
    return pow(5, step % h, 2 << log_n)


# ------------------------------------------------------------------------------------------------ ciphertexts


@dataclass
class Ct:
    data: torch.Tensor  # [K][2][rows][N] int64 on the device
    top: int
    scale: float
    slots: int

    @property
    def k(self):
        return self.data.shape[0]

    def ptr(self):
        return C.c_void_p(self.data.data_ptr())

    def clone(self):
        return Ct(self.data.clone(), self.top, self.scale, self.slots)


@dataclass
class Diagonals:
    """The plaintexts of a BSGS plaintext-matrix product on the device: pts [npts][nq][N] evaluation rows (diagonal
    d = bstep j + b pre-rotated by -bstep j stride) and the device table of their addresses that pt_dot reads."""

    pts: torch.Tensor
    table: torch.Tensor
    bstep: int
    stride: int
    top: int
    scale: float
    slots: int
    ext: bool = False  # rows over the special primes too (top + 1 + kp rows): the double-hoisted product

    @property
    def npts(self):
        return self.pts.shape[0]

    @property
    def gstep(self):
        return -(-self.npts // self.bstep)

    def steps(self):
        """The rotation steps the product needs keys for: the babies b stride and the giants bstep j stride."""
        return [b * self.stride for b in range(1, self.bstep)] + \
            [j * self.bstep * self.stride for j in range(1, self.gstep)]


# How a session stores its switching keys (the reference's KeySource, crates/pc-gpu/src/ks.rs:57): "dense" keeps b
# and a resident (Cached); "regen" keeps b and the seed of a, which the inner-product kernels regenerate (Regen, half
# the key bytes). Both give the same keys and the same results word for word.
KEY_SOURCES = {"dense": 0, "regen": 1}


class Session:
    """A context over one chain with device-resident keys (relinearization + the given rotation steps)."""

    def __init__(self, chain, rot_steps=(), k_max=1, seed=0, h=192, sigma=3.2, device=None, key_source="dense",
                 galois_extra=(), keygen=True):
        """keygen=False: a server's session, no secret; its key slots (relinearization first, then the galois
        elements of rot_steps and galois_extra) are filled from a client's key bundle (wire.import_keys)."""
        self.chain = chain
        self.device = torch.device(device or "cuda")
        self.n, self.log_n = chain.n, chain.log_n
        self.nq, self.kp, self.rows = len(chain.q), len(chain.p), chain.rows
        self.k_max = k_max
        gal = [1]
        for s in rot_steps:
            g = rotation_galois(s, chain.log_n)
            if g != 1 and g not in gal:
                gal.append(g)
        for g in galois_extra:  # keys for other automorphisms, e.g. conjugation (2N - 1)
            g %= 2 * chain.n
            if g != 1 and g not in gal:
                gal.append(g)
        self.galois = gal
        self._q = (C.c_uint64 * self.nq)(*chain.q)
        self._p = (C.c_uint64 * self.kp)(*chain.p)
        if key_source not in KEY_SOURCES:
            raise ValueError(f"key_source {key_source!r}: one of {sorted(KEY_SOURCES)}")
        self.key_source = key_source
        self.params = L.Params(chain.log_n, self.nq, self.kp, chain.dnum,
                               C.cast(self._q, L.u64p), C.cast(self._p, L.u64p), k_max, KEY_SOURCES[key_source])
        lib = L.lib()
        nbytes = lib.pcb_ctx_bytes(C.byref(self.params), len(gal))
        if nbytes < 0:
            L.check(int(nbytes), "pcb_ctx_bytes")
        with torch.cuda.device(self.device):
            self.arena = torch.empty(int(nbytes), dtype=torch.uint8, device=self.device)
            h_ctx = C.c_void_p()
            L.check(lib.pcb_ctx_create(C.byref(self.params), len(gal), C.c_void_p(self.arena.data_ptr()),
                                       int(nbytes), self._stream(), C.byref(h_ctx)), "pcb_ctx_create")
            self.ctx = h_ctx
            if keygen:
                g = (C.c_uint64 * len(gal))(*gal)
                L.check(lib.pcb_keygen(self.ctx, seed, h, sigma, len(gal), C.cast(g, L.u64p), self._stream()),
                        "pcb_keygen")

    def __del__(self):
        ctx = getattr(self, "ctx", None)
        if not ctx:
            return
        self.ctx = None
        try:
            torch.cuda.synchronize(self.device)
            L.lib().pcb_ctx_destroy(ctx)
        except Exception:
            pass  # interpreter teardown: the process exit releases the host state

    def _stream(self):
        return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    # -------------------------------------------------------------------------------------------- buffers
    def empty(self, k=1):
        return torch.empty((k, 2, self.rows, self.n), dtype=torch.int64, device=self.device)

    def ct_like(self, x):
        return Ct(self.empty(x.k), x.top, x.scale, x.slots)

    def top(self):
        return self.nq - 1

    def stack(self, cts):
        """One K-batched ciphertext from single ones at the same level (heads, independent ciphertexts)."""
        c0 = cts[0]
        if any(c.top != c0.top for c in cts):
            raise ValueError("stack: ciphertexts at different tops")
        return Ct(torch.cat([c.data for c in cts]), c0.top, c0.scale, c0.slots)

    def key(self, idx):
        b, a, g = C.c_void_p(), C.c_void_p(), C.c_uint64()
        L.check(L.lib().pcb_key_ptrs(self.ctx, idx, C.byref(b), C.byref(a), C.byref(g)), "pcb_key_ptrs")
        words = self.chain.dnum * self.rows * self.n
        return b.value, a.value, g.value, words

    def key_tensors(self, idx):
        """Copies of key `idx` (b, a) as [dnum][rows][N] device tensors."""
        shape = (self.chain.dnum, self.rows, self.n)
        b = torch.empty(shape, dtype=torch.int64, device=self.device)
        a = torch.empty(shape, dtype=torch.int64, device=self.device)
        L.check(L.lib().pcb_key_copy(self.ctx, idx, C.c_void_p(b.data_ptr()), C.c_void_p(a.data_ptr()),
                                     self._stream()), "pcb_key_copy")
        return b, a

    def tables(self):
        ptrs = [C.c_void_p() for _ in range(7)]
        L.check(L.lib().pcb_ctx_tables(self.ctx, *[C.byref(p) for p in ptrs]), "pcb_ctx_tables")
        return [p.value for p in ptrs]

    # -------------------------------------------------------------------------------------------- encode / encrypt
    @staticmethod
    def _vals(values):
        v = np.asarray(values, dtype=np.complex128).ravel()
        flat = np.ascontiguousarray(np.stack([v.real, v.imag], 1).ravel())
        return flat, len(v)

    def encode(self, values, slots=None, scale=2.0**40, top=None):
        """Coefficient-form rows 0..=top (host numpy uint64) of the encoding of `values`."""
        top = self.top() if top is None else top
        flat, nv = self._vals(values)
        slots = slots or max(1, 1 << (nv - 1).bit_length())
        rows = np.zeros((top + 1, self.n), np.uint64)
        L.check(L.lib().pcb_encode(self.ctx, flat.ctypes.data_as(C.POINTER(C.c_double)), nv, slots, scale, top,
                                   rows.ctypes.data_as(L.u64p)), "pcb_encode")
        return rows

    def encrypt(self, values, top=None, scale=2.0**40, slots=None):
        top = self.top() if top is None else top
        flat, nv = self._vals(values)
        slots = slots or max(1, 1 << (nv - 1).bit_length())
        out = self.empty(1)
        L.check(L.lib().pcb_encrypt(self.ctx, flat.ctypes.data_as(C.POINTER(C.c_double)), nv, slots, scale, top,
                                    C.c_void_p(out.data_ptr()), self._stream()), "pcb_encrypt")
        return Ct(out, top, scale, slots)

    def decrypt_slots(self, ct, index=0):
        vals = np.zeros(2 * ct.slots, np.float64)
        ptr = ct.data[index].data_ptr()
        L.check(L.lib().pcb_decrypt(self.ctx, C.c_void_p(ptr), ct.top, ct.slots, ct.scale,
                                    vals.ctypes.data_as(C.POINTER(C.c_double)), self._stream()), "pcb_decrypt")
        return vals[0::2] + 1j * vals[1::2]

    def pt(self, values, top, scale, slots):
        """A plaintext in evaluation form on the device ([nq][N]) for mult_pt / add_pt."""
        rows = self.encode(values, slots=slots, scale=scale, top=top)
        dev = torch.zeros((self.nq, self.n), dtype=torch.int64, device=self.device)
        L.check(L.lib().pcb_pt_load(self.ctx, rows.ctypes.data_as(L.u64p), top, C.c_void_p(dev.data_ptr()),
                                    self._stream()), "pcb_pt_load")
        return dev

    # -------------------------------------------------------------------------------------------- ops
    def _same(self, a, b):
        if a.top != b.top or a.k != b.k:
            raise ValueError(f"operands at tops {a.top} / {b.top}, batches {a.k} / {b.k}")

    def add(self, a, b):
        self._same(a, b)
        out = self.ct_like(a)
        L.check(L.lib().pcb_add(self.ctx, a.ptr(), b.ptr(), out.ptr(), a.top, a.k, self._stream()), "pcb_add")
        return out

    def sub(self, a, b):
        self._same(a, b)
        out = self.ct_like(a)
        L.check(L.lib().pcb_sub(self.ctx, a.ptr(), b.ptr(), out.ptr(), a.top, a.k, self._stream()), "pcb_sub")
        return out

    def sum(self, cts, out=None):
        """Sum of up to 32 ciphertext batches of one level in one pass (each input read once)."""
        cts = list(cts)
        for x in cts[1:]:
            self._same(cts[0], x)
        out = out if out is not None else self.ct_like(cts[0])
        ptrs = (C.c_void_p * len(cts))(*[x.data.data_ptr() for x in cts])
        L.check(L.lib().pcb_sum(self.ctx, ptrs, len(cts), out.ptr(), cts[0].top, cts[0].k, self._stream()), "pcb_sum")
        return out

    def inplace_add(self, a, b):
        self._same(a, b)
        L.check(L.lib().pcb_add(self.ctx, a.ptr(), b.ptr(), a.ptr(), a.top, a.k, self._stream()), "pcb_add")
        return a

    def mult(self, a, b):
        """Relinearized product, rescale pending."""
        self._same(a, b)
        out = Ct(self.empty(a.k), a.top, a.scale * b.scale, a.slots)
        L.check(L.lib().pcb_mult(self.ctx, a.ptr(), b.ptr(), out.ptr(), a.top, a.k, self._stream()), "pcb_mult")
        return out

    def square(self, a):
        return self.mult(a, a)

    def rescale_one(self, a):
        """In place: drop the top prime, scale / q_top."""
        L.check(L.lib().pcb_rescale(self.ctx, a.ptr(), a.top, a.k, self._stream()), "pcb_rescale")
        a.scale /= self.chain.q[a.top]
        a.top -= 1
        return a

    def drop_to(self, a, top):
        """The same ciphertext over fewer limbs (residues mod the lower primes are unchanged)."""
        if top > a.top:
            raise ValueError("drop_to raises no level")
        return Ct(a.data, top, a.scale, a.slots)

    def rotate(self, a, step):
        out = self.ct_like(a)
        L.check(L.lib().pcb_rotate(self.ctx, a.ptr(), int(step), out.ptr(), a.top, a.k, self._stream()), "pcb_rotate")
        return out

    def rotate_hoisted(self, a, steps):
        """[rot(a, s) for s in steps] sharing one ModUp (the reference's Fhe.rotate_hoisted)."""
        outs = [self.ct_like(a) for _ in steps]
        st = (C.c_int64 * len(steps))(*[int(x) for x in steps])
        ptrs = (C.c_void_p * len(steps))(*[o.data.data_ptr() for o in outs])
        L.check(L.lib().pcb_rotate_hoisted(self.ctx, a.ptr(), st, len(steps), ptrs, a.top, a.k, self._stream()),
                "pcb_rotate_hoisted")
        return outs

    def rotate_and_sum(self, a, start, stop, radix_bits=1):
        """a + rot(a, s) + rot(a, 2s) + ... below stop: rung by rung, or (radix_bits >= 2) with groups of gaps that
        have keys for all their steps summed by rotate_sum (the reference's radix ladder)."""
        out = self.ct_like(a)
        L.check(L.lib().pcb_rotate_and_sum_radix(self.ctx, a.ptr(), int(start), int(stop), int(radix_bits), out.ptr(),
                                                 a.top, a.k, self._stream()), "pcb_rotate_and_sum_radix")
        return out

    def rotate_sum(self, a, steps):
        """a + sum rot(a, s) over steps, the rotations summed in the extended basis with one ModDown."""
        out = self.ct_like(a)
        st = (C.c_int64 * len(steps))(*[int(x) for x in steps])
        L.check(L.lib().pcb_rotate_sum(self.ctx, a.ptr(), st, len(steps), out.ptr(), a.top, a.k, self._stream()),
                "pcb_rotate_sum")
        return out

    def mult_pt(self, a, pt, pt_scale):
        out = Ct(self.empty(a.k), a.top, a.scale * pt_scale, a.slots)
        L.check(L.lib().pcb_mult_pt(self.ctx, a.ptr(), C.c_void_p(pt.data_ptr()), out.ptr(), a.top, a.k,
                                    self._stream()), "pcb_mult_pt")
        return out

    def mult_pt_add(self, a, pt, pt_scale, y, sub=0, out=None):
        """y + a * pt (sub 1: y - a * pt, 2: a * pt - y) in one pass (the reference's mult_pt_add); the product's
        scale must be y's."""
        if a.top != y.top or a.k != y.k:
            raise ValueError(f"operands at tops {a.top} / {y.top}, batches {a.k} / {y.k}")
        out = out if out is not None else self.ct_like(y)
        L.check(L.lib().pcb_mult_pt_add(self.ctx, a.ptr(), C.c_void_p(pt.data_ptr()), y.ptr(), out.ptr(), int(sub),
                                        a.top, a.k, self._stream()), "pcb_mult_pt_add")
        return out

    def mult_pt_sum(self, terms):
        """sum_j x_j * pt_j for terms (x_j, pt_j, pt_scale_j) at one level and batch, every product at the first
        term's scale, in one pass (pcb_mult_pt_sum; up to 8 terms)."""
        x0, _, s0 = terms[0]
        for x, _, _ in terms[1:]:
            self._same(x0, x)
        out = Ct(self.empty(x0.k), x0.top, x0.scale * s0, x0.slots)
        xs = (C.c_void_p * len(terms))(*[x.data.data_ptr() for x, _, _ in terms])
        ps = (C.c_void_p * len(terms))(*[p.data_ptr() for _, p, _ in terms])
        L.check(L.lib().pcb_mult_pt_sum(self.ctx, xs, ps, len(terms), out.ptr(), x0.top, x0.k, self._stream()),
                "pcb_mult_pt_sum")
        return out

    def diagonals(self, diags, bstep, top=None, scale=None, slots=None, stride=1, ext=False):
        """Encode the generalized diagonals diag_d (d < npts; slot vectors) of a slots x slots matrix M (diag_d[i] =
        M[i, i + d stride]) for linear_transform: y = sum_d diag_d * rot(x, d stride). scale defaults to q_top, so
        one rescale returns the product to x's scale. ext: the rows of the special primes too, for the
        double-hoisted product (pcb_linear_transform_ext)."""
        top = self.top() if top is None else top
        diags = [np.asarray(v) for v in diags]
        slots = slots or len(diags[0])
        scale = float(self.chain.q[top]) if scale is None else scale
        nr = top + 1 + (len(self.chain.p) if ext else 0)
        pts = torch.zeros((len(diags), nr, self.n), dtype=torch.int64, device=self.device)  # the rows read
        enc, load = (L.lib().pcb_encode_ext, L.lib().pcb_pt_load_ext) if ext else (L.lib().pcb_encode, L.lib().pcb_pt_load)
        for d, v in enumerate(diags):
            g = (d // bstep) * bstep * stride
            flat, nv = self._vals(np.roll(v, g))
            rows = np.zeros((nr, self.n), np.uint64)
            L.check(enc(self.ctx, flat.ctypes.data_as(C.POINTER(C.c_double)), nv, slots, scale, top,
                        rows.ctypes.data_as(L.u64p)), "pcb_encode")
            L.check(load(self.ctx, rows.ctypes.data_as(L.u64p), top, C.c_void_p(pts[d].data_ptr()), self._stream()),
                    "pcb_pt_load")
        table = torch.tensor([pts[d].data_ptr() for d in range(len(diags))], dtype=torch.int64, device=self.device)
        return Diagonals(pts, table, int(bstep), int(stride), top, scale, slots, bool(ext))

    def linear_work(self, lt, k=1, nw=1):
        """Scratch for linear_transform(_multi): (bstep + gstep nw) k ciphertexts."""
        return torch.empty(((lt.bstep + lt.gstep * nw) * k, 2, self.rows, self.n), dtype=torch.int64,
                           device=self.device)

    def linear_transform(self, a, lt, out=None, work=None, baby_offset=0):
        """The BSGS plaintext-matrix product sum_d diag_d * rot(a, d stride) of a K-batch (hoisted babies, one
        pt_dot launch, the giant rotations summed in the extended basis with one ModDown). Scale a.scale lt.scale.
        baby_offset (double-hoisted diagonals only): the product of rot(a, baby_offset stride), that rotation folded
        into the babies."""
        if a.top != lt.top:
            raise ValueError(f"ciphertext at top {a.top}, diagonals encoded at top {lt.top}")
        if baby_offset and not lt.ext:
            raise ValueError("a baby offset needs the double-hoisted diagonals (ext=True)")
        out = out if out is not None else Ct(self.empty(a.k), a.top, a.scale * lt.scale, a.slots)
        work = work if work is not None else self.linear_work(lt, a.k)
        if lt.ext:  # the double-hoisted form (babies in the extended basis)
            L.check(L.lib().pcb_linear_transform_ext(self.ctx, a.ptr(), C.c_void_p(lt.table.data_ptr()), 1, lt.npts,
                                                     lt.bstep, lt.stride, int(baby_offset), C.c_void_p(work.data_ptr()),
                                                     out.ptr(), a.top, a.k, self._stream()), "pcb_linear_transform_ext")
        else:
            L.check(L.lib().pcb_linear_transform(self.ctx, a.ptr(), C.c_void_p(lt.table.data_ptr()), lt.npts,
                                                 lt.bstep, lt.stride, C.c_void_p(work.data_ptr()), out.ptr(), a.top,
                                                 a.k, self._stream()), "pcb_linear_transform")
        out.scale = a.scale * lt.scale
        return out

    def linear_transform_multi(self, a, lts, work=None):
        """linear_transform of one input against several diagonal sets of one shape: the babies computed once, the
        giant rotations of all weights run as one batch. Returns one batch: weight w's results are members
        w k .. w k + k - 1 (split() gives them apart)."""
        lt0 = lts[0]
        for lt in lts:
            if (lt.npts, lt.bstep, lt.stride, lt.top, lt.scale) != (lt0.npts, lt0.bstep, lt0.stride, lt0.top, lt0.scale):
                raise ValueError("linear_transform_multi: diagonal sets of different shapes or scales")
        if a.top != lt0.top:
            raise ValueError(f"ciphertext at top {a.top}, diagonals encoded at top {lt0.top}")
        out = Ct(self.empty(len(lts) * a.k), a.top, a.scale * lt0.scale, a.slots)
        work = work if work is not None else self.linear_work(lt0, a.k, len(lts))
        table = torch.cat([lt.table for lt in lts])
        if any(lt.ext != lt0.ext for lt in lts):
            raise ValueError("linear_transform_multi: extended and plain diagonal sets mixed")
        args = (self.ctx, a.ptr(), C.c_void_p(table.data_ptr()), len(lts), lt0.npts, lt0.bstep, lt0.stride)
        rest = (C.c_void_p(work.data_ptr()), out.ptr(), a.top, a.k, self._stream())
        if lt0.ext:
            L.check(L.lib().pcb_linear_transform_ext(*args, 0, *rest), "pcb_linear_transform_ext")
        else:
            L.check(L.lib().pcb_linear_transform_multi(*args, *rest), "pcb_linear_transform_multi")
        return out

    def split(self, a, n):
        """n equal batches of a batch (views, no copies)."""
        k = a.k // n
        return [Ct(a.data[i * k:(i + 1) * k], a.top, a.scale, a.slots) for i in range(n)]

    def add_pt(self, a, pt):
        out = self.ct_like(a)
        L.check(L.lib().pcb_add_pt(self.ctx, a.ptr(), C.c_void_p(pt.data_ptr()), out.ptr(), a.top, a.k,
                                   self._stream()), "pcb_add_pt")
        return out

    def mod_raise(self, a, top):
        """a at level 0 raised to limbs 0..top in a new ciphertext (bootstrapping's ModRaise); decrypts to
        m + q_0 I. pcb_mod_raise works in place on the copy's buffer; `a` is left as it was."""
        if a.top != 0:
            raise ValueError(f"mod_raise takes a level-0 ciphertext, not top {a.top}")
        out = Ct(self.empty(a.k), int(top), a.scale, a.slots)
        out.data[:, :, 0].copy_(a.data[:, :, 0])
        L.check(L.lib().pcb_mod_raise(self.ctx, out.ptr(), int(top), a.k, self._stream()), "pcb_mod_raise")
        return out

    def automorph(self, a, g):
        """The automorphism X -> X^g of a (a key switch with the key of galois element g): g = 2N - 1 conjugates
        every slot; 5^r mod 2N rotates by r."""
        g %= 2 * self.n
        if g not in self.galois:
            raise ValueError(f"no key for galois element {g}")
        out = self.ct_like(a)
        autok = pow(g, (2 * self.n >> 2) - 1, 2 * self.n)  # g^-1 in the group of 5 and -1 (crates/pc-core/src/galois.rs)
        c1 = C.c_void_p(a.data.data_ptr() + self.rows * self.n * 8)
        L.check(L.lib().pcb_keyswitch(self.ctx, c1, a.ptr(), 1, self.galois.index(g), autok, out.ptr(), a.top, a.k, 0,
                                      self._stream()), "pcb_keyswitch")
        return out

    def conjugate(self, a):
        return self.automorph(a, 2 * self.n - 1)

    def monomial(self, power, top, coef=1):
        """coef X^power (coef an integer) as a plaintext of scale 1 ([nq][N] evaluation rows): its slots are all
        coef zeta^(power 5^k); power N / 2 multiplies every slot by i, power 0 by the integer coef.
        mult_pt(a, monomial, 1.0) uses no level."""
        key = ("monomial", int(power) % (2 * self.n), top, int(coef))
        cache = self.__dict__.setdefault("_monomials", {})
        if key not in cache:
            pw = int(power) % (2 * self.n)
            rows = np.zeros((top + 1, self.n), np.uint64)
            for r in range(top + 1):
                q = self.chain.q[r]
                rows[r, pw % self.n] = (int(coef) if pw < self.n else -int(coef)) % q  # X^N = -1
            dev = torch.zeros((self.nq, self.n), dtype=torch.int64, device=self.device)
            L.check(L.lib().pcb_pt_load(self.ctx, rows.ctypes.data_as(L.u64p), top, C.c_void_p(dev.data_ptr()),
                                        self._stream()), "pcb_pt_load")
            cache[key] = dev
        return cache[key]

    def keyswitch(self, d, c0, c0_mode, kidx, autok, out, top, k):
        L.check(L.lib().pcb_keyswitch(self.ctx, C.c_void_p(d), C.c_void_p(c0 or 0), c0_mode, kidx, autok,
                                      C.c_void_p(out), top, k, 0, self._stream()), "pcb_keyswitch")

    def ntt_batch(self, x, nrows, inverse=False):
        L.check(L.lib().pcb_ntt_batch(self.ctx, C.c_void_p(x.data_ptr()), nrows, int(inverse), self._stream()),
                "pcb_ntt_batch")

    def device_sync(self):
        torch.cuda.synchronize(self.device)


Fhe = Session
