"""CKKS bootstrapping with full slots (the reference's bootstrap of crates/pc-gpu/src/bts/
{raise,cts,evalmod,stc}.rs): a level-0 ciphertext is refreshed to a high level with the same slot values.

Steps, restated from the encoder's algebra (perseus_b200/csrc/host_math.h Encoder, crates/pc-core/src/encode.rs):

1. ModRaise (ops.mod_raise): the level-0 residues lifted to the whole chain; the ciphertext now decrypts to
   t = t_msg + q_0 I, with I a small integer polynomial.
2. CoeffToSlot. With S = N / 2 slots, decoding reads w_i = (t_i + i t_(i + S)) / scale and the slots are
   F(bitrev(w)), F the special FFT's butterfly stages (len 2, 4, .., S). Its inverse stages G (S F^-1) applied
   homomorphically leave bitrev(w) in the slots. A stage of half-length h is a 3-diagonal map of the slot vector,
   y = d_0 x + d_h rot(x, h) + d_-h rot(x, -h); consecutive stages are merged into groups (composition:
   diag_(a+b) += D_a rot(E_b, a)), each group one BSGS plaintext-matrix product (ops.linear_transform) after a rotation
   by -D stride that makes its offsets -D .. D stride non-negative: one level per group.
3. The real and imaginary parts: u = w + conj(w) (conjugation = the automorphism X -> X^(2N-1), one key switch),
   v = (w - conj(w)) X^(3N/2) (X^(N/2) multiplies every slot by i: a plaintext of scale 1, no level).
4. EvalMod on the batch [u, v] (one set of launches for both): with x = t / (K' q_0) in [-1, 1],
   t mod q_0 ~ (q_0 / 2 pi) sin(2 pi K' x) = (q_0 / 2 pi) cos(2 pi K' x - pi / 2), computed as the degree-63
   Chebyshev interpolant of cos((2 pi K' x - pi / 2) / 2^r) followed by r double angles c <- 2 c^2 - 1. The
   interpolant is evaluated in the Chebyshev basis (babies T_1 .. T_7 and giants T_8, T_16, T_32, the polynomial split
   recursively as q T_m + r), every sum at exactly one scale: each term lands at its target scale through a constant
   plaintext chosen for it, so no addition mixes scales.
5. The parts recombined, w' = u' + X^(N/2) v', then SlotToCoeff: the forward stages F on bitrev(w') give the slots
   F(bitrev(w')), the message.

Precision: EvalMod's error is amplified by q_0 / (2 pi Delta) on the way out, and the sine's own error is about
(2 pi^2 / 3) (Delta / q_0)^2 |m / Delta|^3 per coefficient. A level-0 input at a small scale is therefore first
multiplied by the integer 2^b (exact, no level) so that EvalMod runs at q_0 / Delta' = 2^ratio_bits (2^8: about 1e-4
of sine error for a constant slot vector of 1, where |m / Delta| peaks; far less for spread-out slots). The key switches
of SlotToCoeff act on messages of about 2^-8 relative size, so their noise must stay far below the ModDown rounding: the
special modulus P is one prime larger than a digit (config4_chain).

Scales: the ciphertext's `scale` is bookkeeping (slots = decoding / scale). After ModRaise it is set to K' q_0, so
the slots of CoeffToSlot's output are x in [-1, 1]; the last CoeffToSlot group's plaintexts are encoded so that its
output lands at a working scale near the primes (stable products); the factor q_0 / (2 pi Delta) of EvalMod's output
is taken into the scale (free). Levels: CoeffToSlot and SlotToCoeff one per group, EvalMod 7 + r.

Keys: relinearization, conjugation (galois 2N - 1) and the rotations of `rot_steps(...)`.
"""
import math
from dataclasses import dataclass

import numpy as np


# ------------------------------------------------------------------------------------------------ FFT stages
def _rot_group(n):
    """5^k mod 2N for k < N/2 (the slot order of the encoder)."""
    m, out, f = 2 * n, [], 1
    for _ in range(n // 2):
        out.append(f)
        f = f * 5 % m
    return out


def stage_twiddles(n, h, inverse):
    """The encoder's twiddles of the stage of half-length h (host_math.h Encoder: ksi^((5^k mod 8h) (2N / 8h)),
    inverse ksi^((8h - 5^k mod 8h) (2N / 8h)), ksi = e^(2 pi i / 2N)), k < h."""
    m, q = 2 * n, 8 * h
    gap = m // q
    rot = _rot_group(n)
    e = [((q - rot[k] % q) if inverse else rot[k] % q) * gap for k in range(h)]
    return np.exp(2j * np.pi * np.array(e, dtype=np.float64) / m)


def stage_diagonals(n, h, inverse):
    """The stage of half-length h on S = n / 2 slots as {offset: diagonal}: forward (decode direction)
    y[b+k] = x[b+k] + w_k x[b+k+h], y[b+k+h] = x[b+k] - w_k x[b+k+h]; inverse (encode direction)
    y[b+k] = x[b+k] + x[b+k+h], y[b+k+h] = (x[b+k] - x[b+k+h]) w'_k."""
    S = n // 2
    w = stage_twiddles(n, h, inverse)
    k = np.arange(S) % (2 * h)
    first = k < h
    wk = w[np.where(first, k, k - h)]
    d0 = np.where(first, 1.0 + 0j, -wk)
    dp = np.where(first, 1.0 + 0j if inverse else wk, 0j)  # x[j + h] into the first half
    dm = np.where(first, 0j, wk if inverse else 1.0 + 0j)  # x[j - h] into the second half
    return {0: d0, h: dp, -h: dm}


def compose(a, b, S):
    """The diagonals of A(B(x)) from A's and B's: diag_(o_a + o_b) += D_a rot(E_b, o_a) (rot(v, s)[j] = v[j + s])."""
    out = {}
    for oa, da in a.items():
        for ob, db in b.items():
            o = oa + ob
            out[o] = out.get(o, 0) + da * np.roll(db, -oa)
    return out


def groups(n, inverse, per):
    """The stages of G (inverse: h = S/2 .. 1, CoeffToSlot) or F (forward: h = 1 .. S/2, SlotToCoeff) merged `per`
    at a time (the last group may be shorter); returns [(stride, {offset: diagonal})] in application order."""
    S = n // 2
    hs = [S >> (j + 1) for j in range(int(math.log2(S)))] if inverse else [1 << j for j in range(int(math.log2(S)))]
    out = []
    for g0 in range(0, len(hs), per):
        part = hs[g0:g0 + per]
        m = None
        for h in part:  # applied in order: the later stage composes on the left
            d = stage_diagonals(n, h, inverse)
            m = d if m is None else compose(d, m, S)
        out.append((min(part), m))
    return out


# ------------------------------------------------------------------------------------------------ parameters
@dataclass
class Params:
    n: int                 # ring dimension N (S = N / 2 slots)
    K: int = 24            # EvalMod's range: |I| < K - 1/2
    r: int = 3             # double angles after the interpolant
    degree: int = 63
    per_group: int = 5     # FFT stages merged per CoeffToSlot / SlotToCoeff group
    ratio_bits: int = 8    # log2(q_0 / Delta') EvalMod works at: the input is first multiplied by the integer
    #                        2^round(log2(q_0 / Delta) - ratio_bits) when that is above 1
    ext: bool = True       # the groups' BSGS products double-hoisted (babies in the extended basis)

    @property
    def slots(self):
        return self.n // 2


def _bsgs(npts):
    """(bstep, gstep) with bstep gstep >= npts and bstep + gstep smallest (ties to the larger bstep)."""
    best = None
    for b in range(1, npts + 1):
        g = -(-npts // b)
        if best is None or b + g < best[0] + best[1] or (b + g == best[0] + best[1] and b > best[0]):
            best = (b, g)
    return best


def _bsgs_ext(npts):
    """(bstep, gstep) of the double-hoisted product: a baby costs one key inner product, a giant step a ModDown, a
    ModUp and an inner product; with weights 0.7 and 3.1 (in ModDowns, from the config-4 stage timings) the cheapest
    split covering npts (ties to the smaller bstep: fewer keys)."""
    best = None
    for b in range(1, npts + 1):
        g = -(-npts // b)
        cost = 0.7 * (b - 1) + 3.1 * (g - 1)
        if best is None or cost < best[0] - 1e-9:
            best = (cost, b, g)
    return best[1], best[2]


def _group_plan(stride, diags, S, ext=False):
    """(D, npts, bstep, gstep) of a group: its offsets -D .. D strides, rotated by -D stride onto 0 .. 2D. A group whose
    2D + 1 offsets exceed the S / stride distinct rotations is folded mod S instead (D = 0, npts = S / stride: offsets
    congruent mod S are one rotation, their diagonals summed). ext: the split of the double-hoisted product."""
    D = max(abs(o) for o in diags) // stride
    span = S // stride
    if 2 * D + 1 > span:
        D, npts = 0, span
    else:
        npts = 2 * D + 1
    bstep, gstep = _bsgs_ext(npts) if ext else _bsgs(npts)
    return D, npts, bstep, gstep


def _plan_diagonals(stride, diags, S, factor):
    """The npts diagonals of the group's BSGS product, in offset order (d stride for d < npts after the -D stride
    pre-rotation, or mod S when folded)."""
    D, npts, _, _ = _group_plan(stride, diags, S)
    out = [np.zeros(S, np.complex128) for _ in range(npts)]
    for o, d in diags.items():
        j = (o // stride + D) if D else (o % S) // stride
        out[j] = out[j] + factor * d
    return out


def rot_steps(p):
    """Every rotation step the bootstrap uses (the conjugation key is galois 2N - 1, added separately)."""
    steps = set()
    S = p.slots
    for inverse in (True, False):
        for stride, diags in groups(p.n, inverse, p.per_group):
            D, npts, bstep, gstep = _group_plan(stride, diags, S, p.ext)
            if p.ext:  # the pre-rotation by -D stride folded into the babies: steps (b - D) stride
                steps.update((b - D) * stride for b in range(bstep))
            else:
                steps.add(-D * stride)
                steps.update(b * stride for b in range(1, bstep))
            steps.update(j * bstep * stride for j in range(1, gstep))
    return sorted({s % S for s in steps if s % S})


def conj_galois(n):
    return 2 * n - 1


# ------------------------------------------------------------------------------------------------ helpers
def _const_pt(ops, plan, value, top, scale, slots):
    key = ("const", complex(value), top, float(scale), slots)
    pt = plan.get(key)
    if pt is None:
        pt = plan[key] = ops.pt(np.full(slots, value, dtype=np.complex128), top, scale, slots)
    return pt


def _add_const(ops, plan, x, value):
    return ops.add_pt(x, _const_pt(ops, plan, value, x.top, x.scale, x.slots))


def _mul(ops, a, b):
    top = min(a.top, b.top)
    return ops.rescale_one(ops.mult(ops.drop_to(a, top), ops.drop_to(b, top)))


class Cheb:
    """p(x) = sum_k c_k T_k(x) on ciphertexts, every addition at one exact scale (see the module's step 4)."""

    def __init__(self, ops, plan, x, primes):
        self.ops, self.plan, self.primes = ops, plan, primes
        T = {1: x}

        def lin(j, k):  # 2 T_j T_k - T_(j-k) (or - 1 when j == k), one rescale
            top = min(T[j].top, T[k].top)
            m = ops.mult(ops.drop_to(T[j], top), ops.drop_to(T[k], top))
            m2 = ops.add(m, m)
            if j == k:
                return _add_const(ops, plan, ops.rescale_one(m2), -1.0)
            # T_(j-k) times 1 at the product's scale, subtracted before the rescale
            x = ops.drop_to(T[j - k], top)
            pscale = m2.scale / x.scale
            d = ops.mult_pt_add(x, _const_pt(ops, plan, 1.0, top, pscale, x.slots), pscale, m2, sub=1)
            d.scale = m2.scale
            return ops.rescale_one(d)

        T[2] = lin(1, 1)
        T[3] = lin(2, 1)
        T[4] = lin(2, 2)
        T[5] = lin(3, 2)
        T[6] = lin(3, 3)
        T[7] = lin(4, 3)
        T[8] = lin(4, 4)
        T[16] = lin(8, 8)
        T[32] = lin(16, 16)
        self.T = T

    def maxlev(self, d):
        """The highest level at which a polynomial of degree d can be delivered."""
        if d < 8:
            return min(self.T[k].top for k in range(1, max(d, 1) + 1)) - 1
        m = 1 << (d.bit_length() - 1)
        return min(min(self.maxlev(d - m), self.T[m].top) - 1, self.maxlev(m - 1))

    def eval(self, c, scale, level):
        """sum_k c[k] T_k at exactly `scale`, level `level` (<= maxlev(deg))."""
        x, k0 = self.eval_pre(c, scale, level)
        return _add_const(self.ops, self.plan, self.ops.rescale_one(x), k0)

    def eval_pre(self, c, scale, level):
        """(X, k0): the polynomial without its constant term, one rescale short (level + 1, scale scale q_(level+1)),
        and that constant, so that rescale(X) + k0 = sum_k c[k] T_k at `scale`, `level`. Every partial sum meets at
        that one scale before the rescale: a leaf's terms c_k T_k (each T_k taken to level + 1 and times c_k at the
        plaintext scale that lands it there), a node's product Q T_m with its remainder's unrescaled sum."""
        ops, plan, primes = self.ops, self.plan, self.primes
        c = list(c)
        while len(c) > 1 and c[-1] == 0.0:
            c.pop()
        d = len(c) - 1
        pre = scale * primes[level + 1]
        if d < 8:
            terms = []
            for k in range(1, max(d, 1) + 1):
                if d > 0 and c[k] == 0.0:
                    continue  # (a constant keeps a zero c_1 term: c_0 needs a ciphertext at the level and scale)
                x = ops.drop_to(self.T[k], level + 1)
                pscale = pre / x.scale
                terms.append((x, _const_pt(ops, plan, c[k] if d > 0 else 0.0, level + 1, pscale, x.slots), pscale))
            acc = ops.mult_pt_sum(terms)  # every term multiplied and summed in one pass
            acc.scale = pre
            return acc, c[0]
        m = 1 << (d.bit_length() - 1)
        q = [c[m]] + [2.0 * c[m + j] for j in range(1, d - m + 1)]
        r = c[:m]
        for j in range(1, d - m + 1):
            r[m - j] -= c[m + j]
        Tm = self.T[m]
        lq = level + 1
        Q = self.eval(q, pre / Tm.scale, lq)
        P = ops.mult(Q, ops.drop_to(Tm, lq))
        R, k0 = self.eval_pre(r, scale, level)
        X = ops.add(P, R)
        X.scale = pre
        return X, k0


# ------------------------------------------------------------------------------------------------ bootstrap
class Bootstrapper:
    """The encoded CoeffToSlot / SlotToCoeff diagonals and EvalMod coefficients of one chain, and the refresh."""

    def __init__(self, ops, p, primes, q0):
        self.ops, self.p, self.primes, self.q0 = ops, p, list(primes), float(q0)
        self.plan = {}
        self.cts = groups(p.n, True, p.per_group)
        self.stc = groups(p.n, False, p.per_group)
        f = lambda x: np.cos((2 * np.pi * p.K * x - np.pi / 2) / 2**p.r)  # noqa: E731
        self.coeffs = [float(v) for v in np.polynomial.chebyshev.chebinterpolate(f, p.degree)]

    @property
    def levels(self):
        """Levels one refresh spends: one per CoeffToSlot and SlotToCoeff group, 7 + r in EvalMod."""
        return len(self.cts) + 7 + self.p.r + len(self.stc)

    def _transform(self, x, stride, diags, factor, out_scale=None, out_mask=None):
        """x -> sum_o (factor diag_o) rot(x, o) (offsets o = d stride, |d| <= D): x rotated by -D stride (folded into the babies of the double-hoisted product), one BSGS
        product with the diagonals shifted to 0 .. 2D (or folded mod S), one rescale (the output at out_scale when
        given)."""
        ops, S = self.ops, self.p.slots
        D, npts, bstep, _ = _group_plan(stride, diags, S, self.p.ext)
        top = x.top
        key = ("lt", stride, id(diags), top, float(x.scale), out_scale, None if out_mask is None else id(out_mask))
        lt = self.plan.get(key)
        if lt is None:
            dl = _plan_diagonals(stride, diags, S, factor)
            if out_mask is not None:  # output slot j of every diagonal times mask[j]: the masked transform
                dl = [d * out_mask for d in dl]
                self.plan[("mask", id(out_mask))] = out_mask  # kept alive with the entry keyed by its id
            scale = float(self.primes[top]) if out_scale is None else out_scale * self.primes[top] / x.scale
            lt = self.plan[key] = ops.diagonals(dl, bstep, top=top, scale=scale, slots=S, stride=stride,
                                                ext=self.p.ext)
        if self.p.ext:  # rot(x, -D stride) folded into the double-hoisted product's babies
            return ops.rescale_one(ops.linear_transform(x, lt, baby_offset=-D))
        y = ops.rotate(x, -D * stride) if D else x
        return ops.rescale_one(ops.linear_transform(y, lt))

    def coeff_to_slot(self, ct):
        """ct (raised; scale K' q0) -> slots bitrev(t / (K' q0)) / 2 ... times 2 in u, v below: the factor 1 / (2 S)
        spread over the groups; the last group lands at a working scale (its level's prime)."""
        n_g = len(self.cts)
        f = (1.0 / (2 * self.p.slots)) ** (1.0 / n_g)
        x = ct
        for gi, (stride, diags) in enumerate(self.cts):
            last = gi == n_g - 1
            x = self._transform(x, stride, diags, f, out_scale=float(self.primes[x.top - 1]) if last else None)
        return x

    def eval_mod(self, uv, delta):
        ops, p, primes = self.ops, self.p, self.primes
        ch = Cheb(ops, self.plan, uv, primes)
        lev = ch.maxlev(p.degree)
        c = ch.eval(self.coeffs, float(primes[lev + 1]), lev)
        for _ in range(p.r):  # cos(2 a) = 2 cos(a)^2 - 1
            sq = _mul(ops, c, c)
            c = _add_const(ops, self.plan, ops.add(sq, sq), -1.0)
        # (q0 / 2 pi Delta) sin(2 pi t / q0) ~ t_msg / Delta: the factor taken into the scale
        c.scale /= self.q0 / (2 * np.pi * delta)
        return c

    def slot_to_coeff(self, w, out_mask=None):
        """The forward stages; out_mask (a slot vector) multiplies the output slots, folded into the last group."""
        x = w
        for gi, (stride, diags) in enumerate(self.stc):
            last = gi == len(self.stc) - 1
            x = self._transform(x, stride, diags, 1.0, out_mask=out_mask if last else None)
        return x

    def __call__(self, ct, top, out_mask=None):
        """ct at level 0 (full slots; its scale is Delta) -> a ciphertext of the same slots at level `top` minus the
        refresh's levels; out_mask (a slot vector) multiplies the output slots at no level."""
        ops, p, n = self.ops, self.p, self.p.n
        if ct.slots != p.slots:
            raise ValueError(f"bootstrapping takes full slots ({p.slots}), not {ct.slots}")
        delta = float(ct.scale)
        if self.q0 / delta < 8.0:
            raise ValueError(f"a level-0 scale of 2^{math.log2(delta):.1f} leaves the message no room below q0")
        boost = max(0, round(math.log2(self.q0 / delta)) - p.ratio_bits)
        if boost:  # m -> 2^boost m at level 0 (exact; the noise grows by the same factor)
            ct = ops.mult_pt(ct, ops.monomial(0, 0, 1 << boost), 1.0)
            delta *= 1 << boost
        x = ops.mod_raise(ct, top)
        x.scale = p.K * self.q0  # slots: t / (K' q0) (after CoeffToSlot)
        w = self.coeff_to_slot(x)
        cw = ops.conjugate(w)
        u = ops.add(w, cw)                                                          # 2 Re w
        v = ops.mult_pt(ops.sub(w, cw), ops.monomial(3 * n // 2, w.top), 1.0)       # (w - conj w)(-i) = 2 Im w
        uv = self.eval_mod(ops.stack([u, v]), delta)
        u2, v2 = ops.split(uv, 2)
        w2 = ops.add(u2, ops.mult_pt(v2, ops.monomial(n // 2, v2.top), 1.0))        # u' + i v'
        return self.slot_to_coeff(w2, out_mask)
