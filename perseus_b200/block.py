"""The attention block's decode step in the projection layout: Q, K, V projections of the token's activation, the
token's K and V rows pushed into the encrypted cache, attention over the cache, the output projection. The role of the
reference's GPT-2 attention block (python/perseus/impl/attention.py:491-551 KVCache and cache_kv_push, :698-800
complex_qkt, :897-962 complex_softmax_v; python/perseus/impl/linear.py:151-156 linear_multi), laid out on the slots of
the projections (perseus_b200/linear.py: element m of the padded width d at slot m t, t = slots / d lanes per element).

Tokens in lanes: a cache block of t tokens is ONE ciphertext holding every head, slot m t + tau = K[b t + tau][m]
(likewise V); the cache is a batch of T / t blocks. With q replicated over the lanes (q_rep[m t + tau] = q[m]):
1. scores: prod = q_rep K_b, then rotate_and_sum(prod, t, d_h t) sums each head's d_h element blocks at a fixed lane:
   slot (d_h h) t + tau holds s_{h, tau} = <q_h, K_tau,h> (q carries 1 / sqrt(d_h));
2. weights P = mask p7(s) (mask: lane tau of each head's first element block), the polynomial of attention.attend;
3. rotate_and_sum(P, -t, d_h t) replicates P_{h, tau} over the head's element blocks at lane tau;
4. y = P V_b, then rotate_and_sum(y, 1, t) sums the lanes: slot m t holds sum_tau P_{h, tau} V_tau[m], element m of
   the block's attention output, in the layout the output projection reads; the blocks' outputs are added.
The decode math (steps 1-4, its polynomial, levels and scales) is attention.attend's with these three ladders; a block
runs every head and every token of the block in the same launches, and the batch of blocks runs together.

Pushing a token: the projections leave K[m] (V[m]) at lane 0 of element block m and partial sums in the other lanes;
a lane-0 mask (one plaintext product) keeps K[m], a rotation by -(position mod t) moves it to the token's lane, and
the row is added into its block. The query is masked the same way with 1 / sqrt(d_h) folded in, then replicated over
the lanes by rotate_and_sum(q, -1, t).

The attention output is masked to lane 0 as well before the output projection, whose replication ladder reads every
lane. Levels from the activation's top L: projections L - 1, masks L - 2 (the cache's level), attention L - 8, mask
L - 9, output projection L - 10.
"""
import math
from dataclasses import dataclass

import numpy as np

from . import attention as A
from . import linear as LIN
from . import shard as SH
from .attention import ladder_steps


@dataclass
class LaneLayout:
    geo: LIN.Geometry  # the projections' geometry (slots, padded width d, lanes t)
    heads: int  # heads with weights (the rest of the padded width is zero)
    head_dim: int
    blocks: int  # cache blocks of t tokens
    radix_bits: int = 1

    @property
    def slots(self):
        return self.geo.slots

    @property
    def t(self):
        return self.geo.t

    @property
    def tokens(self):
        return self.blocks * self.t

    @property
    def width(self):
        return self.heads * self.head_dim

    def score_ladder(self):
        return self.t, self.head_dim * self.t

    def replicate_ladder(self):
        return -self.t, self.head_dim * self.t

    def sum_ladder(self):
        return 1, self.t

    def query_ladder(self):
        return -1, self.t

    def norm_ladder(self):
        """Every element block's lane 0 summed into every one (LayerNorm's mean and variance)."""
        return self.t, self.t * self.geo.d

    def mask(self):
        """Every lane (token) of each head's first element block: where the scores land."""
        m = np.zeros(self.slots)
        for h in range(self.heads):
            m[h * self.head_dim * self.t:h * self.head_dim * self.t + self.t] = 1.0
        return m

    def lane0(self, value=1.0):
        m = np.zeros(self.slots)
        m[np.arange(self.width) * self.t] = value
        return m

    def push_steps(self, lane):
        """Rotations (each with a key of the query ladder) that move lane 0 to `lane`: the largest available right
        rotation first."""
        avail = sorted({-s for s in ladder_steps(*self.query_ladder(), self.radix_bits)}, reverse=True)
        steps, left = [], lane
        while left:
            s = next(a for a in avail if a <= left)
            steps.append(-s)
            left -= s
        return steps

    def rot_steps(self):
        steps = self.geo.rot_steps(self.radix_bits)
        for lad in (self.score_ladder(), self.replicate_ladder(), self.sum_ladder(), self.query_ladder(),
                    self.norm_ladder()):
            steps += ladder_steps(*lad, self.radix_bits)
        seen = set()
        return [s % self.slots for s in steps if s % self.slots and not (s % self.slots in seen or seen.add(s % self.slots))]


def layout(slots, d, heads, head_dim, tokens, radix_bits=1):
    geo = LIN.geometry(slots, d)
    if heads * head_dim > d or tokens % geo.t:
        raise ValueError(f"{heads} x {head_dim} wider than {d}, or {tokens} tokens not in blocks of {geo.t}")
    return LaneLayout(geo, heads, head_dim, tokens // geo.t, radix_bits)


@dataclass
class Weights:
    """The block's weights (d_real x d_real each, d_real = heads x head_dim) and biases, as numpy arrays."""

    wq: np.ndarray
    bq: np.ndarray
    wk: np.ndarray
    bk: np.ndarray
    wv: np.ndarray
    bv: np.ndarray
    wo: np.ndarray
    bo: np.ndarray


class LaneCache:
    """The encrypted K and V caches as batches of token blocks, at the level the pushed rows arrive at; the decode
    step's plaintexts (masks, encoded weights) are kept in `plan`. `seqs` independent sequences decode together (one
    token each per step, at the same position): their blocks are batch members s nblocks + b, every op of the step
    runs on all of them.

    shard = (world, rank) or (world, rank, group) splits the blocks over the ranks of a process group: this rank holds
    blocks SH.share(blocks, world, rank) (`mine`), attends over them, and decode adds the ranks' partial outputs with
    one exchange (SH.gather_sum). A rank with no block (more ranks than blocks) holds one all-zero block, so it runs
    the same ops and adds zeros. Every rank encrypts every block in the same order and keeps its own, so its blocks
    are word for word those of an unsharded cache of the same session randomness."""

    def __init__(self, ops, lay, top, scale=2.0**40, seqs=1, shard=None):
        self.ops, self.lay, self.top, self.scale, self.seqs = ops, lay, top, scale, seqs
        self.k = self.v = None
        self.count = 0
        self.plan = {}
        self.shard = None if shard is None else (shard + (None,))[:3]
        self.mine = list(range(lay.blocks)) if shard is None else list(SH.share(lay.blocks, shard[0], shard[1]))
        self.idle = not self.mine

    @property
    def nblocks(self):
        """Blocks per sequence held here (an idle rank's zero block counts as one)."""
        return max(len(self.mine), 1)

    def _blocks(self, rows):
        lay = self.lay
        vecs = [np.zeros(lay.slots) for _ in range(lay.blocks)]
        for tok, row in enumerate(rows):
            b, lane = divmod(tok, lay.t)
            vecs[b][np.arange(lay.width) * lay.t + lane] = row
        cts = [self.ops.encrypt(v, top=self.top, scale=self.scale, slots=lay.slots) for v in vecs]
        if self.idle:
            return [_zero_like(cts[0])]
        return [cts[b] for b in self.mine]

    def load(self, K, V):
        """The client's cache of n tokens (n x d_real each; with seqs > 1 a list of one such array per sequence, all of
        n tokens), one encryption per block."""
        Ks, Vs = (K, V) if self.seqs > 1 else ([K], [V])
        if len(Ks) != self.seqs or len({k.shape[0] for k in Ks}) != 1 or Ks[0].shape[0] > self.lay.tokens:
            raise ValueError(f"{self.seqs} caches of one token count up to {self.lay.tokens}")
        self.k = self.ops.stack([c for k in Ks for c in self._blocks(k)])
        self.v = self.ops.stack([c for v in Vs for c in self._blocks(v)])
        self.count = Ks[0].shape[0]

    def push(self, k_row, v_row):
        """The token's K and V rows (batches of `seqs`, at this cache's level and scale, each value at lane 0 of its
        element block, nothing in the other lanes) rotated to the token's lane and added into its block."""
        ops, lay, S = self.ops, self.lay, self.seqs
        if self.count >= lay.tokens:
            raise ValueError(f"KV cache full ({lay.tokens} tokens)")
        b, lane = divmod(self.count, lay.t)
        self.count += 1
        if b not in self.mine:  # another rank holds the token's block
            return
        lb, nb = self.mine.index(b), self.nblocks
        kv = ops.stack([k_row, v_row])
        for st in lay.push_steps(lane):
            kv = ops.rotate(kv, st)
        kr, vr = ops.split(kv, 2)
        kblk, vblk = ops.split(self.k, S * nb), ops.split(self.v, S * nb)
        krs, vrs = (ops.split(kr, S), ops.split(vr, S)) if S > 1 else ([kr], [vr])
        for q in range(S):
            ops.inplace_add(kblk[q * nb + lb], krs[q])
            ops.inplace_add(vblk[q * nb + lb], vrs[q])


@dataclass
class NormCfg:
    """LayerNorm without its affine part: (x - mean) / sqrt(var + eps) over the real width, the inverse square root
    replaced by the degree-7 Chebyshev interpolant of 1 / sqrt(u) on [lo, hi] (the variances of the block's inputs lie
    there), as the softmax is by its polynomial; gamma and beta go into the next linears (fold_norm)."""

    lo: float = 0.5
    hi: float = 2.0
    eps: float = 1e-5

    def coeffs(self):
        """Power-basis coefficients in z = (2 u - lo - hi) / (hi - lo) in [-1, 1]."""
        k = np.arange(8)
        z = np.cos((2 * k + 1) * np.pi / 16)
        u = 0.5 * (self.hi - self.lo) * z + 0.5 * (self.hi + self.lo)
        return [float(c) for c in np.polynomial.polynomial.polyfit(z, 1.0 / np.sqrt(u), 7)]

    def plain(self, x):
        """fp64 reference: the same polynomial in place of 1 / sqrt."""
        c = x - x.mean()
        u = (c @ c) / x.size + self.eps
        z = (2 * u - self.lo - self.hi) / (self.hi - self.lo)
        return c * A.poly_eval(self.coeffs(), z)


def fold_norm(w, gamma, beta):
    """The LayerNorm's affine part folded into the Q, K and V linears: (n gamma + beta) W + b = n (diag(gamma) W) +
    (beta W + b)."""
    return Weights(gamma[:, None] * w.wq, beta @ w.wq + w.bq, gamma[:, None] * w.wk, beta @ w.wk + w.bk,
                   gamma[:, None] * w.wv, beta @ w.wv + w.bv, w.wo, w.bo)


def layer_norm(ops, x, lay, plan, cfg, primes):
    """The normalized activation (projection layout, lane 0 of the real elements, zeros elsewhere), 8 levels below x
    (the input: projection layout with zeros outside lane 0 of the real elements, as the client encrypts it):
    1. every element block's lane 0 summed into every one: rotate_and_sum(x, t, t d) (the layout's other lanes hold
       zeros), centred c = x - sum / d_real on the real elements;
    2. the variance the same way from c^2;
    3. z = (2 (var / d_real + eps) - lo - hi) / (hi - lo), then 1 / sqrt by the polynomial (attention.poly7 under the
       real elements' lane-0 mask), times c."""
    dr = lay.width
    real = lay.lane0()
    s = ops.rotate_and_sum(x, *lay.norm_ladder(), lay.radix_bits)
    c = ops.add(ops.drop_to(x, x.top - 1), _masked(ops, plan, s, real * (-1.0 / dr), x.scale, primes))
    sq = ops.rescale_one(ops.mult(c, c))
    v = ops.rotate_and_sum(sq, *lay.norm_ladder(), lay.radix_bits)
    z = _masked(ops, plan, v, real * (2.0 / (dr * (cfg.hi - cfg.lo))), primes[v.top - 1], primes)
    z0 = A._pt(ops, plan, real * ((2 * cfg.eps - cfg.lo - cfg.hi) / (cfg.hi - cfg.lo)), z.top, z.scale, lay.slots)
    z = ops.add_pt(z, z0)
    inv = A.poly7(ops, plan, z, cfg.coeffs(), real, primes, lay.slots)
    return ops.rescale_one(ops.mult(ops.drop_to(c, inv.top), inv))


def _zero_like(ct):
    """An all-zero ciphertext with ct's level, scale and slots (a session Ct on the device or an oracle one)."""
    import copy

    z = copy.copy(ct)
    z.data = ct.data.clone().zero_() if hasattr(ct.data, "zero_") else np.zeros_like(ct.data)
    return z


def _masked(ops, plan, x, values, target_scale, primes):
    """x * values (a plaintext of the plan), rescaled, landing at target_scale one level below x."""
    pscale = target_scale * primes[x.top] / x.scale
    pt = A._pt(ops, plan, values, x.top, pscale, x.slots)
    return ops.rescale_one(ops.mult_pt(x, pt, pscale))


def _linear(ops, cache, name, W, b, top, scale):
    key = ("linear", name, top, float(scale))
    lin = cache.plan.get(key)
    if lin is None:
        lin = cache.plan[key] = LIN.encode(ops, W, cache.lay.geo, top, scale, bias=b)
    return lin


def decode(ops, x_ct, w, cache, coeffs, primes, norm=None, residual=False, out_scale=None, residual_to=None):
    """One token: x_ct the activation (projection layout; a batch of cache.seqs, one per sequence), w the block's
    Weights (with norm: gamma and beta folded in by fold_norm). With norm the activation is layer-normalized first (8
    levels); it must then sit at the cache's level + 10, else + 2. Pushes the token's K and V into the cache and
    returns the block's output (projection layout), plus the activation itself with residual, or plus `residual_to`
    (another ciphertext, e.g. the stream before a refreshed norm) when given. out_scale: the output projection lands
    there (the residual's scale, so the sum is exact), else at its input's scale."""
    lay = cache.lay
    rb = lay.radix_bits
    x_in = x_ct
    if norm is not None:
        x_ct = layer_norm(ops, x_ct, lay, cache.plan, norm, primes)
    if x_ct.top != cache.top + 2:
        raise ValueError(f"activation at top {x_ct.top} after the norm; the cache lives at {cache.top} (= that - 2)")
    lins = [_linear(ops, cache, n, W, b, x_ct.top, x_ct.scale)
            for n, W, b in (("q", w.wq, w.bq), ("k", w.wk, w.bk), ("v", w.wv, w.bv))]
    q, k, v = LIN.linear_multi(ops, x_ct, lins, rb)
    # the token's K and V rows: lane 0 kept, at the cache's scale
    kv = _masked(ops, cache.plan, ops.stack([k, v]), lay.lane0(), cache.scale, primes)
    kr, vr = ops.split(kv, 2)
    cache.push(kr, vr)
    # the query: lane 0 with 1 / sqrt(d_h), at q_top 2^10 so the products land near the primes' size
    qm = _masked(ops, cache.plan, q, lay.lane0(1.0 / math.sqrt(lay.head_dim)), primes[q.top - 1] * 2.0**10, primes)
    qr = ops.rotate_and_sum(qm, *lay.query_ladder(), rb)
    S, nb = cache.seqs, cache.nblocks
    qs = ops.split(qr, S) if S > 1 else [qr]
    qb = ops.stack([x for x in qs for _ in range(nb)]) if S * nb > 1 else qr  # one copy per block, [sequence][block]
    yb = A.attend(ops, qb, cache, coeffs, primes)
    if nb > 1:  # each sequence's blocks (held here) summed
        ys = ops.split(yb, S * nb)
        y = ops.stack([ops.sum(ys[q * nb:(q + 1) * nb]) for q in range(S)]) if S > 1 else ops.sum(ys)
    else:
        y = yb
    if cache.shard is not None:  # the other ranks' blocks: their partial outputs added, the same words everywhere
        y = SH.gather_sum(ops, y, cache.shard[2])
    # the lane sums leave partial sums in lanes 1 .. t-1; the projection's replication ladder needs them zero
    y = _masked(ops, cache.plan, y, lay.lane0(), y.scale, primes)
    if out_scale is None:
        lin_o = _linear(ops, cache, "o", w.wo, w.bo, y.top, y.scale)
    else:
        key = ("linear", "o", y.top, float(y.scale), float(out_scale))
        lin_o = cache.plan.get(key)
        if lin_o is None:
            lin_o = cache.plan[key] = LIN.encode(ops, w.wo, lay.geo, y.top, y.scale, bias=w.bo, out_scale=out_scale)
    out = LIN.linear(ops, y, lin_o, rb)
    if residual_to is not None:
        out = ops.add(out, ops.drop_to(residual_to, out.top))
    elif residual:  # x + block(x): the scales agree to the last bits (both ~2^40), the sum takes the output's
        out = ops.add(out, ops.drop_to(x_in, out.top))
    return out


def plain_decode(x, w, K, V, coeffs, heads, head_dim, norm=None, residual=False):
    """fp64 reference of the step: (the same polynomial LayerNorm,) projections, the token appended to the cache,
    per-head attention with the same polynomial softmax, output projection (, plus x)."""
    x_in = x
    if norm is not None:
        x = norm.plain(x)
    q, k, v = x @ w.wq + w.bq, x @ w.wk + w.bk, x @ w.wv + w.bv
    Ka, Va = np.vstack([K, k]), np.vstack([V, v])
    out = np.zeros(heads * head_dim)
    for h in range(heads):
        sl = slice(h * head_dim, (h + 1) * head_dim)
        s = Ka[:, sl] @ q[sl] / math.sqrt(head_dim)
        out[sl] = A.poly_eval(coeffs, s) @ Va[:, sl]
    y = out @ w.wo + w.bo
    return y + x_in if residual else y
