"""Test infrastructure: the session op signatures over the oracle context, so the attention, projection and block
drivers can run the same op sequence on the CPU restatement as on the CUDA path. A batch (the session's K-batched
ciphertext) is an OBatch of single ciphertexts; every op maps over its members."""
from dataclasses import dataclass

import numpy as np


@dataclass
class OCt:
    data: np.ndarray  # [2][rows][N] uint64
    top: int
    scale: float
    slots: int


class OBatch:
    """A batch of oracle ciphertexts at one level and scale."""

    def __init__(self, cts):
        self.cts = list(cts)

    @property
    def k(self):
        return len(self.cts)

    @property
    def top(self):
        return self.cts[0].top

    @property
    def scale(self):
        return self.cts[0].scale

    @scale.setter
    def scale(self, v):
        for c in self.cts:
            c.scale = v

    @property
    def slots(self):
        return self.cts[0].slots


@dataclass
class OracleDiagonals:
    pts: np.ndarray
    bstep: int
    stride: int
    top: int
    scale: float
    ext: bool = False


def _batched(f):
    """Apply f member by member when an argument is a batch (other arguments shared)."""

    def g(self, *args, **kw):
        n = next((a.k for a in args if isinstance(a, OBatch)), None)
        if n is None:
            return f(self, *args, **kw)
        return OBatch([f(self, *[a.cts[i] if isinstance(a, OBatch) else a for a in args], **kw) for i in range(n)])

    return g


class OracleOps:
    def __init__(self, ctx):
        self.c = ctx

    def encrypt(self, values, top, scale, slots):
        return OCt(self.c.encrypt(values, slots, scale, top), top, scale, slots)

    @_batched
    def add(self, a, b):
        assert a.top == b.top
        return OCt(self.c.add(a.data, b.data, a.top), a.top, a.scale, a.slots)

    @_batched
    def mult(self, a, b):
        assert a.top == b.top
        return OCt(self.c.mult(a.data, b.data, a.top), a.top, a.scale * b.scale, a.slots)

    @_batched
    def sub(self, a, b):
        assert a.top == b.top
        return OCt(self.c.sub(a.data, b.data, a.top), a.top, a.scale, a.slots)

    @property
    def chain(self):
        """The prime chain (`q`, `p`) as the session's."""
        return self.c

    @_batched
    def mod_raise(self, a, top):
        assert a.top == 0
        return OCt(self.c.mod_raise(a.data, top), top, a.scale, a.slots)

    @_batched
    def automorph(self, a, g):
        """X -> X^g by the key of galois element g (g = 2N - 1: conjugation), as the session's automorph."""
        n2 = 2 * self.c.n
        g %= n2
        autok = pow(g, (n2 >> 2) - 1, n2)
        out = self.c.keyswitch(a.data[1], a.data[0], 1, self.c.galois.index(g), autok, a.top)
        return OCt(out, a.top, a.scale, a.slots)

    def conjugate(self, a):
        return self.automorph(a, 2 * self.c.n - 1)

    def monomial(self, power, top, coef=1):
        """coef X^power in coefficient form (rows 0..top) for mult_pt with scale 1."""
        n = self.c.n
        pw = int(power) % (2 * n)
        rows = np.zeros((top + 1, n), np.uint64)
        for r in range(top + 1):
            rows[r, pw % n] = (int(coef) if pw < n else -int(coef)) % self.c.q[r]
        return rows

    @_batched
    def rescale_one(self, a):
        a.data = self.c.rescale(a.data, a.top)
        a.scale /= self.c.q[a.top]
        a.top -= 1
        return a

    @_batched
    def rotate_and_sum(self, a, start, stop, radix_bits=1):
        return OCt(self.c.rotate_and_sum(a.data, start, stop, a.top, radix_bits), a.top, a.scale, a.slots)

    @_batched
    def rotate(self, a, step):
        return OCt(self.c.rotate(a.data, step, a.top), a.top, a.scale, a.slots)

    @_batched
    def rotate_sum(self, a, steps):
        return OCt(self.c.rotate_sum(a.data, steps, a.top), a.top, a.scale, a.slots)

    @_batched
    def drop_to(self, a, top):
        return OCt(a.data, top, a.scale, a.slots)

    def pt(self, values, top, scale, slots):
        return self.c.encode(values, slots, scale, top)

    @_batched
    def mult_pt(self, a, pt, pt_scale):
        return OCt(self.c.mult_pt(a.data, pt, a.top), a.top, a.scale * pt_scale, a.slots)

    @_batched
    def mult_pt_add(self, a, pt, pt_scale, y, sub=0, out=None):
        """y + a pt (sub 1: y - a pt, 2: a pt - y), the session's fused op as two oracle ops (the same residues)"""
        assert a.top == y.top
        m = self.c.mult_pt(a.data, pt, a.top)
        d = self.c.add(y.data, m, a.top) if sub == 0 else (
            self.c.sub(y.data, m, a.top) if sub == 1 else self.c.sub(m, y.data, a.top))
        return OCt(d, y.top, y.scale, y.slots)

    def mult_pt_sum(self, terms):
        """sum_j x_j * pt_j (the session's one-pass op) as oracle products and sums: the same residues"""
        acc = None
        for x, pt, ps in terms:
            m = self.mult_pt(x, pt, ps)
            acc = m if acc is None else self.add(acc, m)
        return acc

    @_batched
    def add_pt(self, a, pt):
        return OCt(self.c.add_pt(a.data, pt, a.top), a.top, a.scale, a.slots)

    def decrypt_slots(self, a, index=0):
        if isinstance(a, OBatch):
            a = a.cts[index]
        return self.c.decrypt(a.data, a.top, a.slots, a.scale)

    def inplace_add(self, a, b):
        assert a.top == b.top
        a.data = self.c.add(a.data, b.data, a.top)
        return a

    def stack(self, cts):
        out = []
        for c in cts:
            out += c.cts if isinstance(c, OBatch) else [c]
        return OBatch(out)

    def split(self, a, n):
        assert a.k % n == 0
        k = a.k // n
        parts = [a.cts[i * k:(i + 1) * k] for i in range(n)]
        return [p[0] if k == 1 else OBatch(p) for p in parts]

    def sum(self, cts):
        acc = cts[0]
        for c in cts[1:]:
            acc = self.add(acc, c)
        return acc

    def diagonals(self, diags, bstep, top, scale=None, slots=None, stride=1, ext=False):
        """Evaluation-form plaintexts of a BSGS product (diagonal d pre-rotated by -bstep (d // bstep) stride); ext:
        over the Q primes 0..=top and every special prime, for the double-hoisted product."""
        from tests import _oracle as O
        slots = slots or len(diags[0])
        scale = float(self.c.q[top]) if scale is None else scale
        primes = list(self.c.q[: top + 1]) + (list(self.c.p) if ext else [])
        pts = np.zeros((len(diags), len(primes) if ext else self.c.nq, self.c.n), np.uint64)
        for d, v in enumerate(diags):
            vr = np.roll(np.asarray(v), (d // bstep) * bstep * stride)
            rows = self.c.encode_ext(vr, slots, scale, top) if ext else self.c.encode(vr, slots, scale, top)
            O.lib().orc_ntt_fwd(rows, len(primes), np.asarray(primes, np.uint64), self.c.logn)
            pts[d, : len(primes)] = rows
        return OracleDiagonals(pts, bstep, stride, top, scale, ext)

    @_batched
    def linear_transform(self, a, lt, baby_offset=0):
        assert a.top == lt.top and (lt.ext or not baby_offset)
        if lt.ext:
            out = self.c.linear_transform_ext(a.data, lt.pts, lt.bstep, lt.stride, a.top, baby_offset)
        else:
            out = self.c.linear_transform(a.data, lt.pts, lt.bstep, lt.stride, a.top)
        return OCt(out, a.top, a.scale * lt.scale, a.slots)

    def linear_transform_multi(self, a, lts):
        return self.stack([self.linear_transform(a, lt) for lt in lts])
