"""The plaintext-weight linear layer on the GPU against the oracle, word for word: the BSGS plaintext-matrix product
(hoisted babies, one pt_dot launch, giant rotations summed in the extended basis) and mult_pt_add, on the integer
chain of config 1, the FP64 path at N = 2^14 and config 2's chain; decrypted results against the generalized
diagonal method in numpy."""
import numpy as np
import pytest

from perseus_b200 import fhe
from tests import _oracle as O

pytestmark = pytest.mark.gpu

SEED, H, SIGMA = 0, 192, 3.2


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


def _session(ch, steps, k_max):
    s = fhe.Session(ch, rot_steps=steps, k_max=k_max, seed=SEED, h=H, sigma=SIGMA)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(SEED, H, SIGMA, s.galois)
    return s, o


def _lt_steps(bstep, npts, stride=1):
    # -stride: the babies of the double-hoisted product with a baby offset of -1
    return ([b * stride for b in range(1, bstep)] + [j * bstep * stride for j in range(1, -(-npts // bstep))] +
            [-stride])


CASES = {
    # name: (chain, bstep, npts, stride, K)
    "int14": (fhe.config1_chain, 4, 14, 1, 1),
    "fp64_14": (lambda: fhe.Chain(14, tuple(fhe.ntt_primes(50, 14, 8)), tuple(fhe.ntt_primes(50, 14, 2, skip=8)), 4),
                4, 16, 2, 2),
    "config2": (fhe.config2_chain, 8, 30, 1, 1),
}


@pytest.fixture(scope="module", params=sorted(CASES))
def case(request):
    mk, bstep, npts, stride, k = CASES[request.param]
    s, o = _session(mk(), _lt_steps(bstep, npts, stride), k)
    return request.param, s, o, bstep, npts, stride, k


def _oracle_pts(s, o, lt, diags):
    """The diagonals encoded and transformed by the oracle: they must equal the product's device plaintexts."""
    top = lt.top
    pts = np.zeros((len(diags), s.nq, s.n), np.uint64)
    for d, v in enumerate(diags):
        g = (d // lt.bstep) * lt.bstep * lt.stride
        rows = o.encode(np.roll(v, g), lt.slots, lt.scale, top)
        O.lib().orc_ntt_fwd(rows, top + 1, np.asarray(o.q[: top + 1], np.uint64), s.log_n)
        pts[d, : top + 1] = rows
    return pts


def test_linear_transform_bit_exact(case):
    name, s, o, bstep, npts, stride, k = case
    rng = np.random.default_rng(40)
    slots = s.n // 2
    top = s.top()
    xs = [rng.normal(0, 1, slots) / 4 for _ in range(k)]
    cts = [s.encrypt(x, top=top, slots=slots) for x in xs]
    a = s.stack(cts) if k > 1 else cts[0]
    diags = [rng.normal(0, 1, slots) / 4 for _ in range(npts)]
    lt = s.diagonals(diags, bstep, top=top, stride=stride)
    opts = _oracle_pts(s, o, lt, diags)
    assert (host(lt.pts) == opts).all()
    out = s.linear_transform(a, lt)
    for c in range(k):
        oc = o.encrypt(xs[c], slots, cts[c].scale, top)
        assert (host(cts[c].data[0])[:, : top + 1] == oc[:, : top + 1]).all()
        want = o.linear_transform(oc, opts, bstep, stride, top)
        assert (host(out.data[c])[:, : top + 1] == want[:, : top + 1]).all(), (name, c)
    s.rescale_one(out)
    for c in range(k):
        got = s.decrypt_slots(out, c).real
        ref = sum(dg * np.roll(xs[c], -d * stride) for d, dg in enumerate(diags))
        assert np.abs(got - ref).max() < 1e-4, name


def test_linear_transform_ext_bit_exact(case):
    """The double-hoisted product (pcb_linear_transform_ext: babies in the extended basis, plaintexts over the
    special primes too) equals the oracle's restatement word for word, below the top level too, and decrypts to the
    generalized diagonal method."""
    name, s, o, bstep, npts, stride, k = case
    rng = np.random.default_rng(41)
    slots = s.n // 2
    for top, off in ((s.top(), 0), (s.top() - 2, 0), (s.top(), -1)):  # off: the product of rot(x, off stride)
        xs = [rng.normal(0, 1, slots) / 4 for _ in range(k)]
        cts = [s.encrypt(x, top=top, slots=slots) for x in xs]
        a = s.stack(cts) if k > 1 else cts[0]
        diags = [rng.normal(0, 1, slots) / 4 for _ in range(npts)]
        lt = s.diagonals(diags, bstep, top=top, stride=stride, ext=True)
        primes = list(o.q[: top + 1]) + list(o.p)
        opts = np.zeros((npts, len(primes), s.n), np.uint64)
        for d, v in enumerate(diags):
            rows = o.encode_ext(np.roll(v, (d // bstep) * bstep * stride), slots, lt.scale, top)
            O.lib().orc_ntt_fwd(rows, len(primes), np.asarray(primes, np.uint64), s.log_n)
            opts[d] = rows
        assert (host(lt.pts) == opts).all()
        out = s.linear_transform(a, lt, baby_offset=off)
        for c in range(k):
            oc = o.encrypt(xs[c], slots, cts[c].scale, top)
            want = o.linear_transform_ext(oc, opts, bstep, stride, top, off)
            assert (host(out.data[c])[:, : top + 1] == want[:, : top + 1]).all(), (name, top, off, c)
        s.rescale_one(out)
        for c in range(k):
            got = s.decrypt_slots(out, c).real
            ref = sum(dg * np.roll(xs[c], -(d + off) * stride) for d, dg in enumerate(diags))
            assert np.abs(got - ref).max() < 1e-4, (name, top, off)


def test_mult_pt_add_bit_exact(case):
    name, s, o, *_ = case
    rng = np.random.default_rng(41)
    top = s.top()
    x, y, w = (rng.normal(0, 1, 256) / 4 for _ in range(3))
    # residue-level parity: the operands' scales need not match for the words to be compared
    a = s.encrypt(x, top=top)
    yv = s.encrypt(y, top=top)
    sc = 2.0**30
    pt = s.pt(w, top, sc, a.slots)
    rows = s.encode(w, slots=a.slots, scale=sc, top=top)
    oa = o.encrypt(x, a.slots, a.scale, top)
    oy = o.encrypt(y, a.slots, yv.scale, top)
    prod = o.mult_pt(oa, rows, top)
    for sub, want in ((0, o.add(oy, prod, top)), (1, o.sub(oy, prod, top)), (2, o.sub(prod, oy, top))):
        out = s.mult_pt_add(a, pt, sc, yv, sub)
        assert (host(out.data[0])[:, : top + 1] == want[:, : top + 1]).all(), (name, sub)


def test_mult_pt_sum_bit_exact(case):
    """pcb_mult_pt_sum (a polynomial's terms in one pass, the mul_add_n launcher): 1, 3 and 8 terms of ciphertexts at
    one level, below the top too, equal the oracle's products summed, word for word."""
    name, s, o, *_ = case
    rng = np.random.default_rng(43)
    for top, n in ((s.top(), 1), (s.top(), 3), (s.top() - 1, 8)):
        xs = [rng.normal(0, 1, 256) / 4 for _ in range(n)]
        ws = [rng.normal(0, 1, 256) / 4 for _ in range(n)]
        cts = [s.encrypt(x, top=top) for x in xs]
        pts = [s.pt(w, top, 2.0**30, cts[0].slots) for w in ws]
        out = s.mult_pt_sum([(c, p, 2.0**30) for c, p in zip(cts, pts)])
        want = None
        for x, c, w in zip(xs, cts, ws):
            m = o.mult_pt(o.encrypt(x, c.slots, c.scale, top), s.encode(w, slots=c.slots, scale=2.0**30, top=top), top)
            want = m if want is None else o.add(want, m, top)
        assert (host(out.data[0])[:, : top + 1] == want[:, : top + 1]).all(), (name, top, n)


# ------------------------------------------------------------------------------------------------ projections

from perseus_b200 import linear as LIN  # noqa: E402
from tests._oracle_ops import OracleOps  # noqa: E402


def _fp64_14():
    return fhe.Chain(14, tuple(fhe.ntt_primes(50, 14, 8)), tuple(fhe.ntt_primes(50, 14, 2, skip=8)), 4)


@pytest.mark.parametrize("mk,d,n,nw,radix", [(_fp64_14, 256, 200, 1, 1), (_fp64_14, 256, 256, 2, 2),
                                            (fhe.config2_chain, 1024, 768, 3, 1)])
def test_projection_bit_exact(mk, d, n, nw, radix):
    """y = x W + b in the reference's layout, GPU against the same op sequence on the oracle, word for word; the
    config-2 case is GPT-2's geometry (768 of 1024, 2^15 slots) with three weights sharing the input (Q, K, V)."""
    ch = mk()
    geo = LIN.geometry(ch.n // 2, d)
    s, o = _session(ch, geo.rot_steps(radix), nw)  # the weights' giant steps run as one batch of nw
    oops = OracleOps(o)
    rng = np.random.default_rng(d + nw)
    x = rng.normal(0, 1, n)
    Ws = [rng.normal(0, 0.02, (n, n)) for _ in range(nw)]
    bs = [rng.normal(0, 0.02, n) for _ in range(nw)]
    top = s.top()
    vec = LIN.input_vector(x, geo)
    a = s.encrypt(vec, top=top, scale=2.0**40, slots=geo.slots)
    oa = oops.encrypt(vec, top, 2.0**40, geo.slots)
    lins = [LIN.encode(s, W, geo, top, a.scale, bias=b) for W, b in zip(Ws, bs)]
    olins = [LIN.encode(oops, W, geo, top, oa.scale, bias=b) for W, b in zip(Ws, bs)]
    ys = LIN.linear_multi(s, a, lins, radix) if nw > 1 else [LIN.linear(s, a, lins[0], radix)]
    oys = LIN.linear_multi(oops, oa, olins, radix) if nw > 1 else [LIN.linear(oops, oa, olins[0], radix)]
    for w, (y, oy) in enumerate(zip(ys, oys)):
        assert y.top == oy.top == top - 1
        assert (host(y.data[0])[:, : y.top + 1] == oy.data[:, : y.top + 1]).all(), w
        got = LIN.output_values(s.decrypt_slots(y).real, geo, n)
        assert np.abs(got - (x @ Ws[w] + bs[w])).max() < 1e-3, w
