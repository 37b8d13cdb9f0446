"""Plaintext-weight linear layers y = x W + b over the evaluator: the Q / K / V / output projections of the attention
block, in the reference's slot layout (python/perseus/impl/linear.py:63-103 prepare_linear_input / apply_linear /
linear_multi; the geometry and packing of python/perseus/impl/layout.py:77-98 cm_params, :126-139
encode_linear_input, :141-162 encode_weight_matrix, :239-255 encode_bias_vector, :257-270 decode_linear_output),
for square weights d x d with d^2 >= slots (GPT-2: d = 1024, the 768-wide hidden state zero-padded).

The layout, restated (S slots, t = S / d, R = d^2 / S weight plaintexts):
- the activation x sits at slots m t (m < d), zeros between;
- prepare: X = rotate_and_sum(x, t - 1, t (t - 1)) = sum_{k < t} rot(x, k (t - 1)), which puts
  x[(i // t + i % t) mod d] on slot i (slot i + k (t - 1) is a multiple of t exactly when k = i mod t);
- product: Y = sum_{j < R} rot(X, j t^2) * w_j with w_j[i] = W[(i // t + i % t + j t) mod d, i // t]
  (rot(X, j t^2)[i] = x[(i // t + i % t + j t) mod d]), run as a baby-step giant-step product with stride t^2:
  babies b < bstep, giants bstep g; the plaintext of j = bstep g + b is w_j pre-rotated by -bstep g t^2 so the
  giant rotation can follow the baby sum (pcb_linear_transform);
- fold: rotate_and_sum(Y, 1, t) sums the t slots of each block: slot m t gets sum_{u < t, j < R}
  W[(m + u + j t) mod d, m] x[(m + u + j t) mod d] = (x W)[m], since u + j t runs over 0 .. d - 1;
- bias: b[m] on every slot of block m (added after the fold).
bstep g = R with bstep + gstep minimal, ties to the larger bstep (the reference's choice, so the rotation keys and
the plaintext order are the same) for the plain product; the double-hoisted product (babies in the extended basis,
pcb_linear_transform_ext, the default) takes the divisor split of least cost with a baby at 0.7 and a giant step at
3.1 ModDowns (R = 32: 16 x 2 instead of 8 x 4).

One rescale after the product: the output sits one level below the input at the input's scale (the weight
plaintexts are encoded at q_top). The same functions run on the CUDA session and, in the tests, on an oracle-backed
adapter.
"""
from dataclasses import dataclass

import numpy as np

from .attention import ladder_steps


@dataclass(frozen=True)
class Geometry:
    slots: int
    d: int  # padded width (power of two)
    t: int  # slots per element: S / d
    npts: int  # weight plaintexts R = d^2 / S
    bstep: int
    gstep: int
    ext: bool = False  # the double-hoisted product (plaintexts over the special primes too)

    @property
    def stride(self):
        return self.t * self.t

    def prep_ladder(self):
        return self.t - 1, self.t * (self.t - 1)

    def fold_ladder(self):
        return 1, self.t

    def rot_steps(self, radix_bits=1):
        """Every rotation key a linear layer of this shape uses."""
        steps = ladder_steps(*self.prep_ladder(), radix_bits)
        steps += [b * self.stride for b in range(1, self.bstep)]
        steps += [g * self.bstep * self.stride for g in range(1, self.gstep)]
        steps += ladder_steps(*self.fold_ladder(), radix_bits)
        seen = set()
        return [s % self.slots for s in steps if s % self.slots and not (s % self.slots in seen or seen.add(s % self.slots))]


def geometry(slots, d, ext=True):
    """The square-layer geometry of cm_params (layout.py:77-98) for d_in = d_out = d; ext: the double-hoisted
    product's split (else the reference's)."""
    if d & (d - 1) or slots & (slots - 1) or d > slots or d * d < slots:
        raise ValueError(f"width {d} must be a power of two with d^2 >= slots ({slots}) and d <= slots")
    t, r = slots // d, d * d // slots
    splits = [(b, r // b) for b in range(1, r + 1) if r % b == 0]
    if ext:
        best = min(splits, key=lambda s: (0.7 * (s[0] - 1) + 3.1 * (s[1] - 1), s[0]))
    else:
        best = (r, 1)
        for b, g in splits:
            if b + g < sum(best) or (b + g == sum(best) and b > best[0]):
                best = (b, g)
    return Geometry(slots, d, t, r, best[0], best[1], bool(ext))


def input_vector(x, geo):
    """The activation's slot vector (encode_linear_input, layout.py:126-139): x[m] at slot m t."""
    x = np.asarray(x, np.float64).ravel()
    if x.size > geo.d:
        raise ValueError(f"{x.size} inputs for width {geo.d}")
    v = np.zeros(geo.slots)
    v[np.arange(x.size) * geo.t] = x
    return v


def output_values(vec, geo, n_out):
    """The first n_out outputs of a linear layer's slot vector (decode_linear_output, layout.py:257-270)."""
    return np.asarray(vec)[np.arange(n_out) * geo.t]


def weight_vectors(W, geo):
    """The R weight slot vectors w_j (before the giant pre-rotation) of W (d_in x d_out <= d x d, zero-padded)."""
    W = np.asarray(W, np.float64)
    Wp = np.zeros((geo.d, geo.d))
    Wp[: W.shape[0], : W.shape[1]] = W
    i = np.arange(geo.slots)
    col = i // geo.t
    base = col + i % geo.t
    return np.stack([Wp[(base + j * geo.t) % geo.d, col] for j in range(geo.npts)])


def bias_vector(b, geo):
    """b[m] on the t slots of block m (encode_bias_vector with fill, layout.py:239-255)."""
    b = np.asarray(b, np.float64).ravel()
    v = np.zeros(geo.slots)
    v[: b.size * geo.t] = np.repeat(b, geo.t)
    return v


@dataclass
class Linear:
    geo: Geometry
    lt: object  # the ops' encoded diagonals
    bias: object  # the ops' bias plaintext at the output level, or None
    bias_scale: float


def encode(ops, W, geo, top, x_scale, bias=None, out_scale=None):
    """Encode W (and b) for inputs at level `top` and scale x_scale: R plaintexts at q_top, the bias at level top - 1;
    the output lands at x_scale, or at out_scale when given (the plaintexts encoded at out_scale q_top / x_scale)."""
    pscale = None if out_scale is None else out_scale * ops.chain.q[top] / x_scale
    lt = ops.diagonals(weight_vectors(W, geo), geo.bstep, top=top, scale=pscale, slots=geo.slots, stride=geo.stride,
                       ext=geo.ext)
    y_scale = x_scale if out_scale is None else out_scale
    bpt = None
    if bias is not None:
        bpt = ops.pt(bias_vector(bias, geo), top - 1, y_scale, geo.slots)
    return Linear(geo, lt, bpt, y_scale)


def prepare(ops, x, geo, radix_bits=1):
    """prepare_linear_input (linear.py:63-77): the replication ladder."""
    return ops.rotate_and_sum(x, *geo.prep_ladder(), radix_bits)


def finish(ops, y, lin, radix_bits=1):
    y = ops.rescale_one(y)
    y = ops.rotate_and_sum(y, *lin.geo.fold_ladder(), radix_bits)
    if lin.bias is not None:
        y = ops.add_pt(y, lin.bias)
    return y


def linear(ops, x, lin, radix_bits=1):
    """y = x W + b (linear.py:147-149)."""
    return finish(ops, ops.linear_transform(prepare(ops, x, lin.geo, radix_bits), lin.lt), lin, radix_bits)


def linear_multi(ops, x, lins, radix_bits=1):
    """One prepared input, one output per weight (linear.py:151-156: K, V and Q of one activation). The babies of the
    product are shared too, and the weights' results form one batch through the giant rotations, the rescale and the
    fold; the biases go on per weight."""
    xp = prepare(ops, x, lins[0].geo, radix_bits)
    y = ops.linear_transform_multi(xp, [l.lt for l in lins])
    y = ops.rescale_one(y)
    y = ops.rotate_and_sum(y, *lins[0].geo.fold_ladder(), radix_bits)
    ys = ops.split(y, len(lins))
    return [ops.add_pt(y, l.bias) if l.bias is not None else y for y, l in zip(ys, lins)]
