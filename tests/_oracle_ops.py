"""Test infrastructure: the session op signatures over the oracle context, so the attention driver can run the same
op sequence on the CPU restatement as on the CUDA path."""
from dataclasses import dataclass

import numpy as np


@dataclass
class OCt:
    data: np.ndarray  # [2][rows][N] uint64
    top: int
    scale: float
    slots: int


class OracleOps:
    def __init__(self, ctx):
        self.c = ctx

    def encrypt(self, values, top, scale, slots):
        return OCt(self.c.encrypt(values, slots, scale, top), top, scale, slots)

    def add(self, a, b):
        assert a.top == b.top
        return OCt(self.c.add(a.data, b.data, a.top), a.top, a.scale, a.slots)

    def mult(self, a, b):
        assert a.top == b.top
        return OCt(self.c.mult(a.data, b.data, a.top), a.top, a.scale * b.scale, a.slots)

    def rescale_one(self, a):
        if isinstance(a, OBatch):
            return OBatch([self.rescale_one(c) for c in a.cts])
        a.data = self.c.rescale(a.data, a.top)
        a.scale /= self.c.q[a.top]
        a.top -= 1
        return a

    def rotate_and_sum(self, a, start, stop, radix_bits=1):
        if isinstance(a, OBatch):
            return OBatch([self.rotate_and_sum(c, start, stop, radix_bits) for c in a.cts])
        return OCt(self.c.rotate_and_sum(a.data, start, stop, a.top, radix_bits), a.top, a.scale, a.slots)

    def rotate_sum(self, a, steps):
        return OCt(self.c.rotate_sum(a.data, steps, a.top), a.top, a.scale, a.slots)

    def drop_to(self, a, top):
        return OCt(a.data, top, a.scale, a.slots)

    def pt(self, values, top, scale, slots):
        return self.c.encode(values, slots, scale, top)

    def mult_pt(self, a, pt, pt_scale):
        return OCt(self.c.mult_pt(a.data, pt, a.top), a.top, a.scale * pt_scale, a.slots)

    def add_pt(self, a, pt):
        return OCt(self.c.add_pt(a.data, pt, a.top), a.top, a.scale, a.slots)

    def decrypt_slots(self, a):
        return self.c.decrypt(a.data, a.top, a.slots, a.scale)

    def diagonals(self, diags, bstep, top, scale=None, slots=None, stride=1):
        """Evaluation-form plaintexts of a BSGS product (diagonal d pre-rotated by -bstep (d // bstep) stride)."""
        from tests import _oracle as O
        slots = slots or len(diags[0])
        scale = float(self.c.q[top]) if scale is None else scale
        pts = np.zeros((len(diags), self.c.nq, self.c.n), np.uint64)
        for d, v in enumerate(diags):
            rows = self.c.encode(np.roll(np.asarray(v), (d // bstep) * bstep * stride), slots, scale, top)
            O.lib().orc_ntt_fwd(rows, top + 1, np.asarray(self.c.q[: top + 1], np.uint64), self.c.logn)
            pts[d, : top + 1] = rows
        return OracleDiagonals(pts, bstep, stride, top, scale)

    def linear_transform(self, a, lt):
        assert a.top == lt.top
        out = self.c.linear_transform(a.data, lt.pts, lt.bstep, lt.stride, a.top)
        return OCt(out, a.top, a.scale * lt.scale, a.slots)

    def linear_transform_multi(self, a, lts):
        return OBatch([self.linear_transform(a, lt) for lt in lts])

    def split(self, a, n):
        assert len(a.cts) == n
        return list(a.cts)


@dataclass
class OBatch:
    """A batch of oracle ciphertexts: the batch-taking ops map over its members."""
    cts: list


@dataclass
class OracleDiagonals:
    pts: np.ndarray
    bstep: int
    stride: int
    top: int
    scale: float
