"""Config 5: the 12-layer GPT-2-small encrypted decode, the KV cache of every layer resident in HBM, bootstrapping
between the layers' stages (the reference's python/perseus/examples/gpt2/model.py:177-257 `decode_token` over
python/perseus/examples/gpt2/block.py:13-62 `transformer_block`: ln_1 -> MHA -> residual -> ln_2 -> up -> GELU ->
down -> residual), built on the attention block of block.py, the projections of linear.py and the refresh of
bootstrap.py.

One layer, one token (levels on the config-4 chain, where a refresh leaves top 12; the refresh of the residual stream
also masks it to lane 0 of the real elements, which LayerNorm needs, at no level):

  x -> refresh -> LN1 (8 levels) -> refresh -> Q/K/V (gamma1, beta1 folded), push into the layer's cache, attention
  over its blocks, output projection landing at the refreshed input's scale (10 levels) -> + x
    -> refresh -> LN2 -> refresh -> up: three 1024-wide square linears of one prepared input (gamma2, beta2 and 1 / B
  folded in, the output at a scale near the primes) -> GELU: the degree-7 Chebyshev interpolant of GELU(B u) on
  [-1, 1] under the lane-0 mask of all 1024 hidden units of a block (4 levels) -> down: three square linears (the 3072 inputs in blocks of 1024) summed,
  landing at the residual's scale -> + residual.

Four refreshes per layer: LayerNorm's 8 levels and the attention's 10 (or the MLP's 6) do not fit in one refresh's 12.
The fp64 reference (`plain_layer`) computes the same polynomials (LayerNorm's inverse square root, softmax, GELU), so
the decrypted output is compared with it at the tolerance the refreshes leave.
"""
import math
from dataclasses import dataclass, field

import numpy as np
from scipy.special import erf

from . import attention as A
from . import block as B
from . import bootstrap as BS
from . import linear as LIN


# ------------------------------------------------------------------------------------------------ GELU
def gelu(x):
    """GELU(x) = x Phi(x) (the exact form; GPT-2's tanh form differs by < 1e-3)."""
    x = np.asarray(x, np.float64)
    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def gelu_poly(bound, degree=7):
    """Power-basis coefficients in u = x / bound of the degree-7 Chebyshev interpolant of GELU(bound u) on [-1, 1]."""
    k = np.arange(degree + 1)
    u = np.cos((2 * k + 1) * np.pi / (2 * (degree + 1)))
    return [float(c) for c in np.polynomial.polynomial.polyfit(u, gelu(bound * u), degree)]


# ------------------------------------------------------------------------------------------------ weights
@dataclass
class LayerWeights:
    """One GPT-2 block's weights (numpy): attention (B.Weights, d x d), the two LayerNorms' affine parts, the MLP's
    up (d x 4d) and down (4d x d) projections with biases."""

    attn: B.Weights
    gamma1: np.ndarray
    beta1: np.ndarray
    gamma2: np.ndarray
    beta2: np.ndarray
    w_up: np.ndarray
    b_up: np.ndarray
    w_down: np.ndarray
    b_down: np.ndarray


def random_layer(rng, d=768, mlp=3072, std=0.02):
    """Random-init weights N(0, std), biases N(0, std), gamma 1 + N(0, std), beta N(0, std)."""
    nrm = lambda *s: rng.normal(0, std, s)  # noqa: E731
    attn = B.Weights(nrm(d, d), nrm(d), nrm(d, d), nrm(d), nrm(d, d), nrm(d), nrm(d, d), nrm(d))
    return LayerWeights(attn, 1 + nrm(d), nrm(d), 1 + nrm(d), nrm(d), nrm(d, mlp), nrm(mlp), nrm(mlp, d), nrm(d))


@dataclass
class ModelCfg:
    layers: int = 12
    d: int = 768           # real width
    width: int = 1024      # padded width of the projection layout
    heads: int = 12
    head_dim: int = 64
    mlp: int = 3072
    tokens: int = 256      # cache capacity per layer
    gelu_bound: float = 3.0
    norm: B.NormCfg = field(default_factory=lambda: B.NormCfg(lo=0.25, hi=4.0))
    radix_bits: int = 3

    @property
    def mlp_blocks(self):
        return -(-self.mlp // self.width)


# ------------------------------------------------------------------------------------------------ fp64 reference
def plain_layer(x, w, K, V, cfg, coeffs):
    """fp64 layer with the same polynomials; K, V: the layer's cached rows before this token (the token's own rows are
    appended, as the cache sees them). Returns (output, k_row, v_row)."""
    n = cfg.norm.plain(x) * w.gamma1 + w.beta1
    a = w.attn
    q, k, v = n @ a.wq + a.bq, n @ a.wk + a.bk, n @ a.wv + a.bv
    Ka, Va = np.vstack([K, k]), np.vstack([V, v])
    att = np.zeros(cfg.heads * cfg.head_dim)
    for h in range(cfg.heads):
        sl = slice(h * cfg.head_dim, (h + 1) * cfg.head_dim)
        s = Ka[:, sl] @ q[sl] / math.sqrt(cfg.head_dim)
        att[sl] = A.poly_eval(coeffs, s) @ Va[:, sl]
    r = att @ a.wo + a.bo + x
    n2 = cfg.norm.plain(r) * w.gamma2 + w.beta2
    u = (n2 @ w.w_up + w.b_up) / cfg.gelu_bound
    g = A.poly_eval(gelu_poly(cfg.gelu_bound), u)
    return g @ w.w_down + w.b_down + r, k, v


def plain_decode(x, weights, caches, cfg, coeffs):
    """The token through every layer; caches: per layer [K, V] (rows so far), extended in place."""
    for w, kv in zip(weights, caches):
        x, k, v = plain_layer(x, w, kv[0], kv[1], cfg, coeffs)
        kv[0], kv[1] = np.vstack([kv[0], k]), np.vstack([kv[1], v])
    return x


# ------------------------------------------------------------------------------------------------ encrypted
class Decoder:
    """The encrypted decode on `ops` (a session, or the oracle's ops: the same op sequence) over the chain's Q
    `primes`. `bt` refreshes (a bootstrap.Bootstrapper on the same ops): a refresh raises to the chain's top and leaves
    `out_top`; every layer's cache lives at cache_top = out_top - 2, where the pushed rows arrive. shard =
    (world, rank[, group]) splits every layer's cache blocks over the ranks (block.LaneCache). seqs = S independent
    sequences decode together, one token each per step: every op of the step (refreshes included) runs on their batch
    (the session needs k_max >= S x the cache's blocks)."""

    def __init__(self, ops, cfg, weights, primes, bt, shard=None, seqs=1, plan=None):
        """plan: another decoder's plaintext plan (the same weights and session) to share its encodings."""
        self.ops, self.cfg, self.w, self.primes, self.bt = ops, cfg, weights, list(primes), bt
        self.seqs = seqs
        self.raise_top = len(self.primes) - 1
        self.out_top = self.raise_top - bt.levels
        self.cache_top = self.out_top - 2
        if self.out_top < 10:
            raise ValueError(f"a refresh leaves top {self.out_top}; the attention stage needs 10 levels")
        self.lay = B.layout(bt.p.slots, cfg.width, cfg.heads, cfg.head_dim, cfg.tokens, cfg.radix_bits)
        self.coeffs = A.softmax_poly(self.lay.tokens)
        self.gcoef = gelu_poly(cfg.gelu_bound)
        self.caches = []
        self.plan = {} if plan is None else plan
        self.shard = shard
        self.mask = self.lay.lane0()  # lane 0 of the real elements: the residual stream
        self.hidden_mask = np.zeros(self.lay.slots)  # lane 0 of every element: an MLP block's 1024 hidden units
        self.hidden_mask[np.arange(self.lay.geo.d) * self.lay.t] = 1.0
        self.folded = [B.fold_norm(w.attn, w.gamma1, w.beta1) for w in weights]

    # -------------------------------------------------------------- setup
    def load(self, Ks, Vs):
        """The client's caches: per layer K, V (n x d rows; with seqs > 1 a list of one such array per sequence), one
        LaneCache per layer at cache_top."""
        self.caches = []
        for K, V in zip(Ks, Vs):
            c = B.LaneCache(self.ops, self.lay, self.cache_top, seqs=self.seqs, shard=self.shard)
            c.load(K, V)
            self.caches.append(c)

    def _lin(self, name, W, b, top, x_scale, out_scale):
        key = ("lin", name, top, float(x_scale), float(out_scale))
        lin = self.plan.get(key)
        if lin is None:
            lin = self.plan[key] = LIN.encode(self.ops, W, self.lay.geo, top, x_scale, bias=b, out_scale=out_scale)
        return lin

    # -------------------------------------------------------------- stages
    def refresh(self, ct, mask=True):
        """ct (any level) dropped to level 0 and bootstrapped; with mask the output keeps only lane 0 of the real
        elements (folded into SlotToCoeff's last group: no level). A ciphertext whose scale leaves the message too
        little room below q_0 (above q_0 / 16: LayerNorm's output lands near the primes' size) is first brought to
        q_0 / 2^ratio_bits by one product with the lane-0 mask (the values it keeps are already all there are), using
        one of its levels."""
        target = self.primes[0] / 2.0**self.bt.p.ratio_bits
        if ct.scale > self.primes[0] / 16.0:
            if ct.top < 1:
                raise ValueError(f"a level-0 ciphertext at scale 2^{math.log2(ct.scale):.1f} cannot be refreshed")
            ct = B._masked(self.ops, self.plan, ct, self.mask, target, self.primes)
        x = self.ops.drop_to(ct, 0)
        return self.bt(x, self.raise_top, out_mask=self.mask if mask else None)

    def attention(self, l, n, x):
        """The attention part of layer l on the normalized, refreshed activation n (cache top + 2); returns
        x + attention output at the output projection's level, at x's scale."""
        return B.decode(self.ops, n, self.folded[l], self.caches[l], self.coeffs, self.primes, out_scale=x.scale,
                        residual_to=x)

    def mlp(self, l, n2, r):
        """up, GELU, down on the normalized, refreshed activation n2; returns r + MLP output at r's scale."""
        ops, cfg, w, lay = self.ops, self.cfg, self.w[l], self.lay
        d, nb = cfg.width, cfg.mlp_blocks
        g2 = w.gamma2[:, None] * w.w_up
        b2 = w.beta2 @ w.w_up + w.b_up
        Bnd = cfg.gelu_bound
        top = n2.top
        out_scale = float(self.primes[top - 1])  # GELU's input near the primes' size
        ups = [self._lin(f"up{l}.{j}", g2[:, j * d:(j + 1) * d] / Bnd, b2[j * d:(j + 1) * d] / Bnd, top, n2.scale,
                         out_scale) for j in range(nb)]
        us = LIN.linear_multi(ops, n2, ups, lay.radix_bits)
        u = ops.stack(us)
        g = A.poly7(ops, self.plan, u, self.gcoef, self.hidden_mask, self.primes, lay.slots)
        gs = ops.split(g, nb)
        ys = []
        for j, gj in enumerate(gs):
            bias = w.b_down if j == 0 else None
            dn = self._lin(f"down{l}.{j}", w.w_down[j * d:(j + 1) * d], bias, gj.top, gj.scale, r.scale)
            ys.append(LIN.linear(ops, gj, dn, lay.radix_bits))
        y = ops.sum(ys) if len(ys) > 1 else ys[0]
        return ops.add(y, ops.drop_to(r, y.top))

    def layer(self, l, x):
        x1 = self.refresh(x)
        n = self.refresh(B.layer_norm(self.ops, x1, self.lay, self.plan, self.cfg.norm, self.primes), mask=False)
        r = self.attention(l, n, x1)
        r1 = self.refresh(r)
        n2 = self.refresh(B.layer_norm(self.ops, r1, self.lay, self.plan, self.cfg.norm, self.primes), mask=False)
        return self.mlp(l, n2, r1)

    def decode(self, x):
        """One token (the activation in the projection layout; a batch of seqs, one per sequence) through every layer;
        pushes the token's K and V rows into every layer's cache. Returns the last layer's output (lane 0 of each
        element block carries the value)."""
        for l in range(len(self.w)):
            x = self.layer(l, x)
        return x
