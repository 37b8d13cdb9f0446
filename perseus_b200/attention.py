"""Encrypted attention decode over the evaluator: the encrypted KV cache and one decode step (Q K^T, polynomial
softmax, P V), the role of the reference's attention driver (python/perseus/impl/attention.py:491-551 KVCache,
:698-800 complex_qkt, :897-962 complex_softmax_v, :1394 attend) re-laid-out for one head per ciphertext (the reference
interleaves heads in one ciphertext; here heads are separate ciphertexts so a batch of heads runs as one K-batched
launch set and heads shard across GPUs without communication).

Layout (d = head_dim, T = token capacity, both powers of two, d T <= slots):
- K cache: slot t d + j = K[t][j]; V cache: slot t d + j = V[t][j] (tokens pushed by adding an encryption of the
  token's row at its offset, the reference's cache_k_push / cache_v_push).
- query: slot t d + j = Q[j] / sqrt(d) for every t (the client folds the 1/sqrt(d) in and replicates).

Step (all rotations left; rotate_and_sum(x, s, e) = x + rot(x, s) + ... ladder, python/perseus/impl/poly.py:24-39):
1. prod = Q * K, rescale; scores = rotate_and_sum(prod, 1, d): slot t d holds s_t = <Q, K_t> / sqrt(d);
2. P = mask * p(scores), p the degree-7 polynomial standing in for softmax, mask = 1 on slots t d of the T token
   blocks (tokens not yet pushed hold zero K and V, so their weights multiply zeros): baby-step giant-step
   p = (c0 + c1 x + c2 x^2 + c3 x^3) + x^4 (c4 + c5 x + c6 x^2 + c7 x^3), the coefficients as masked plaintexts (the
   mask costs no level), each term's plaintext scale chosen so all terms meet at one scale; these plaintexts are
   constants of the layout, encoded on the first step and kept in the cache's plan;
3. replicate: R = rotate_and_sum(P, -1, d) puts P_t on slots t d .. t d + d - 1;
4. out = rotate_and_sum(rescale(R * V), d, d T): slot j holds sum_t P_t V[t][j].
Depth 6: from top L the output lands at top L - 6 (config 1: 8 limbs, decrypted at top 1).

Scales are tracked exactly (doubles). The inputs K, V are encrypted at 2^40 (BASELINE); the query is encoded at
q_top 2^10 so the score lands near 2^50, the size of the primes, which keeps every power of the polynomial near 2^50
after each rescale. The same function runs on the CUDA session and, in the tests, on an oracle-backed adapter.
"""
import math
from dataclasses import dataclass

import numpy as np

INPUT_SCALE = 2.0**40


def softmax_poly(n_tokens, lo=-1.0, hi=1.0, degree=7):
    """Power-basis coefficients c_0..c_7 of the degree-7 Chebyshev interpolant of exp(x) / n_tokens on [lo, hi]:
    the polynomial that replaces softmax (weights ~ exp(s_t) / sum_u exp(s_u) for scores near 0)."""
    k = np.arange(degree + 1)
    xs = np.cos((2 * k + 1) * np.pi / (2 * (degree + 1)))  # Chebyshev nodes on [-1, 1]
    xt = 0.5 * (hi - lo) * xs + 0.5 * (hi + lo)
    coef = np.polynomial.polynomial.polyfit(xt, np.exp(xt) / n_tokens, degree)
    return [float(c) for c in coef]


def poly_eval(coeffs, x):
    return sum(c * x**i for i, c in enumerate(coeffs))


def plain_attention(q, k, v, coeffs):
    """fp64 reference of the decode step with the same polynomial softmax."""
    d = q.shape[-1]
    s = k @ q / math.sqrt(d)
    w = poly_eval(coeffs, s)
    return w @ v


@dataclass
class Layout:
    head_dim: int
    tokens: int
    slots: int
    radix_bits: int = 1  # rotate_and_sum ladders: 1 = rung by rung; >= 2 = groups of that many gaps (rotate_sum)

    def ladders(self):
        return [self.score_ladder(), self.replicate_ladder(), self.sum_ladder()]

    # the decode step's three rotate_and_sum ladders (start, stop) and its score mask
    def score_ladder(self):
        return 1, self.head_dim

    def replicate_ladder(self):
        return -1, self.head_dim

    def sum_ladder(self):
        return self.head_dim, self.head_dim * self.tokens

    def mask(self):
        """Slot 0 of every token block of the cache's capacity. Tokens not yet in the cache hold zero K and V
        words: their scores are zero and the weights they get multiply zero values, so the mask does not follow the
        token count and the masked coefficient plaintexts are constants of the layout."""
        m = np.zeros(self.slots)
        m[0 : self.tokens * self.head_dim : self.head_dim] = 1.0
        return m

    def rot_steps(self):
        """The rotation keys the decode step needs: every rung (gap) of the three ladders, and with radix groups
        every step j g (j < 2^n) of each group."""
        steps = []
        for start, stop in self.ladders():
            steps += ladder_steps(start, stop, self.radix_bits)
        seen = set()
        return [s for s in steps if not (s in seen or seen.add(s))]


def ladder_steps(start, stop, radix_bits=1):
    """The rotation steps of rotate_and_sum(x, start, stop) (gaps |start| 2^k below stop, signed like start): each
    gap alone, or with radix_bits >= 2 every step j g (j < 2^n) of each group of n gaps."""
    sign, gaps = (1 if start > 0 else -1), []
    g = abs(start)
    while g < stop:
        gaps.append(g)
        g *= 2
    rb = radix_bits if radix_bits >= 2 else 1
    steps = []
    for i0 in range(0, len(gaps), rb):
        n = min(rb, len(gaps) - i0)
        if n > 1:
            steps += [sign * j * gaps[i0] for j in range(1, 1 << n)]
        else:
            steps.append(sign * gaps[i0])
    return steps


class KVCache:
    """One head's encrypted K and V caches (one ciphertext each), tokens appended in place."""

    def __init__(self, ops, layout, top):
        self.ops, self.lay, self.top = ops, layout, top
        self.k = None
        self.v = None
        self.count = 0
        self.plan = {}  # the decode step's plaintexts, encoded once (attend)

    def _row_ct(self, row, t):
        vec = np.zeros(self.lay.slots)
        vec[t * self.lay.head_dim:(t + 1) * self.lay.head_dim] = row
        return self.ops.encrypt(vec, top=self.top, scale=INPUT_SCALE, slots=self.lay.slots)

    def push(self, k_row, v_row):
        """cache_k_push / cache_v_push: the token's rows encrypted at its offset and added into the caches."""
        t = self.count
        if t >= self.lay.tokens:
            raise ValueError(f"KV cache full ({self.lay.tokens} tokens)")
        kc, vc = self._row_ct(k_row, t), self._row_ct(v_row, t)
        self.k = kc if self.k is None else self.ops.add(self.k, kc)
        self.v = vc if self.v is None else self.ops.add(self.v, vc)
        self.count += 1

    def load(self, K, V):
        """The whole cache at once (T x d each): one encryption per cache."""
        n = K.shape[0]
        d = self.lay.head_dim
        kv, vv = np.zeros(self.lay.slots), np.zeros(self.lay.slots)
        kv[: n * d] = K.ravel()
        vv[: n * d] = V.ravel()
        self.k = self.ops.encrypt(kv, top=self.top, scale=INPUT_SCALE, slots=self.lay.slots)
        self.v = self.ops.encrypt(vv, top=self.top, scale=INPUT_SCALE, slots=self.lay.slots)
        self.count = n


class HeadBatch:
    """Several heads' caches as one K-batched cache (the session's ops run every head in the same launches)."""

    def __init__(self, ops, caches):
        self.lay = caches[0].lay
        self.count = caches[0].count
        if any(c.count != self.count for c in caches):
            raise ValueError("heads of one batch hold the same number of tokens")
        self.k = ops.stack([c.k for c in caches])
        self.v = ops.stack([c.v for c in caches])
        self.plan = {}


def encrypt_query(ops, q, layout, top, q_top_prime):
    """The client's query ciphertext: Q / sqrt(d) replicated per token block, at scale q_top 2^10 (see above)."""
    d, t = layout.head_dim, layout.tokens
    vec = np.zeros(layout.slots)
    vec[: d * t] = np.tile(q / math.sqrt(d), t)
    return ops.encrypt(vec, top=top, scale=q_top_prime * 2.0**10, slots=layout.slots)


def _pt(ops, plan, values, top, scale, slots):
    """A plaintext of the decode step (mask x polynomial coefficient at a fixed level and scale): encoded on first use
    and kept in the cache's plan, so later tokens reuse it."""
    key = (top, float(scale), slots, np.asarray(values, np.float64).tobytes())
    pt = plan.get(key)
    if pt is None:
        pt = plan[key] = ops.pt(values, top, scale, slots)
    return pt


def poly7(ops, plan, x, coeffs, mask, primes, slots):
    """mask * p(x) for a polynomial of degree <= 7 (power-basis coefficients), x at a scale near its level's prime:
    baby steps x, x^2, x^3, giant step x^4, p = (c0 + c1 x + c2 x^2 + c3 x^3) + x^4 (c4 + c5 x + c6 x^2 + c7 x^3), the
    coefficients as masked plaintexts (the mask costs no level) whose scales make every term meet at one scale; the
    plaintexts are kept in `plan`. Four levels: the result sits at x.top - 4."""
    L1 = x.top
    x2 = ops.rescale_one(ops.mult(x, x))  # L-2
    x3 = ops.rescale_one(ops.mult(x2, ops.drop_to(x, L1 - 1)))  # L-3
    x4 = ops.rescale_one(ops.mult(x2, x2))  # L-3
    lvl = L1 - 2  # the level of x^3 / x^4

    def inner_pre(cs, pre, level):
        # sum_{i >= 1} c_i mask x^i at `level`, one rescale short: each x^i taken to `level` times its coefficient at
        # the plaintext scale that puts the product at `pre`, summed in the same pass (the constant returned apart)
        terms = []
        for pw, c in zip((x, x2, x3), cs[1:]):
            src = ops.drop_to(pw, level)
            pscale = pre / src.scale
            terms.append((src, _pt(ops, plan, mask * c, level, pscale, slots), pscale))
        acc = ops.mult_pt_sum(terms)  # the terms multiplied and summed in one pass
        acc.scale = pre
        return acc, cs[0]

    def with_const(acc, c0):
        return ops.add_pt(acc, _pt(ops, plan, mask * c0, acc.top, acc.scale, slots))

    # p = A + x^4 B: B at lvl - 1 with scale S q_(lvl-1) / scale(x^4); the product x^4 B and A's terms meet at
    # level lvl - 1 before one rescale to lvl - 2 (scale ~ S)
    S = primes[lvl - 1]  # the result's scale (~2^50)
    x4d = ops.drop_to(x4, lvl - 1)
    b_pre, b0 = inner_pre(coeffs[4:8] if len(coeffs) > 4 else [0.0], S * primes[lvl - 1] / x4d.scale * primes[lvl],
                          lvl)
    B = with_const(ops.rescale_one(b_pre), b0)
    P = ops.mult(x4d, B)
    a_pre, a0 = inner_pre(coeffs[:4], P.scale, lvl - 1)
    X = ops.add(P, a_pre)
    X.scale = P.scale
    return with_const(ops.rescale_one(X), a0)


def attend(ops, q_ct, cache, coeffs, primes):
    """One decode step: the encrypted attention output (one head: slots 0..d-1; the lane layout of the block: slot m t
    per block). `primes` = the chain's Q primes (bottom first); `ops` provides mult, rescale_one, rotate_and_sum,
    drop_to, add, pt, mult_pt, add_pt. The layout gives the three ladders and the score mask."""
    lay = cache.lay
    top = q_ct.top
    # 1. scores
    k_ct = ops.drop_to(cache.k, top)
    prod = ops.rescale_one(ops.mult(q_ct, k_ct))
    x = ops.rotate_and_sum(prod, *lay.score_ladder(), lay.radix_bits)  # top L-1
    # 2. masked polynomial
    P = poly7(ops, cache.plan, x, coeffs, lay.mask(), primes, lay.slots)
    # 3. replicate each weight over its block
    R = ops.rotate_and_sum(P, *lay.replicate_ladder(), lay.radix_bits)
    # 4. weighted values, summed over tokens
    v_ct = ops.drop_to(cache.v, R.top)
    y = ops.rescale_one(ops.mult(R, v_ct))
    return ops.rotate_and_sum(y, *lay.sum_ladder(), lay.radix_bits)


class DecodeGraph:
    """The decode step of one cache as a CUDA graph: the query is copied into a fixed device buffer and the graph
    replays every kernel of attend, with no host work per token (at N = 2^14 the step is otherwise bound by the
    hundreds of launches and the host's op dispatch). Session ops only (device buffers from torch); the first,
    eager step runs at construction and fills the cache's plan, so capture sees no host copies. The returned
    ciphertext is the graph's output buffer, overwritten by the next call."""

    def __init__(self, ops, cache, coeffs, primes, q_ct):
        import torch

        self.q = ops.ct_like(q_ct)
        self.q.data.copy_(q_ct.data)
        attend(ops, self.q, cache, coeffs, primes)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = attend(ops, self.q, cache, coeffs, primes)
        torch.cuda.synchronize()

    def __call__(self, q_ct):
        if q_ct.top != self.q.top or q_ct.scale != self.q.scale or q_ct.data.shape != self.q.data.shape:
            raise ValueError("the query must have the captured level, scale and batch")
        self.q.data.copy_(q_ct.data)
        self.graph.replay()
        return self.out
