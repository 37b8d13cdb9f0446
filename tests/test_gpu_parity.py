"""Parity of the CUDA path (through the C ABI) with the oracle: bit-exact residues on the same seeded keys,
encryption randomness and inputs, decrypted values against the plaintext math.

Launcher-level tests drive the reference-compatible table entries (ntt_fwd / ntt_inv with their epilogues and
out-of-place sources, bconv, ks_dot, tensor, automorph) on rows of both rings; evaluator-level tests compare keys,
encryptions, products, rescales and rotations of a Session with the oracle context built from the same seed.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from perseus_b200 import _lib as L
from perseus_b200 import fhe
from tests import _oracle as O

pytestmark = pytest.mark.gpu

SEED, H, SIGMA = 0, 192, 3.2
STEPS1 = (1, 2, 4, 8, 16, 32, 64, -1)


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()


def vp(t):
    return C.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def s1():
    ch = fhe.config1_chain()
    s = fhe.Session(ch, rot_steps=STEPS1, k_max=4, seed=SEED, h=H, sigma=SIGMA)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(SEED, H, SIGMA, s.galois)
    return s, o


@pytest.fixture(scope="module")
def s2():
    ch = fhe.config2_chain()
    s = fhe.Session(ch, rot_steps=(1, 5), k_max=2, seed=SEED, h=H, sigma=SIGMA)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(SEED, H, SIGMA, s.galois)
    return s, o


@pytest.fixture(scope="module")
def s3():
    # N = 2^14 with every prime below 2^50 (8 Q + 2 special, dnum 4): the FP64 kernels at the smaller ring
    ch = fhe.Chain(14, tuple(fhe.ntt_primes(50, 14, 8)), tuple(fhe.ntt_primes(50, 14, 2, skip=8)), 4)
    s = fhe.Session(ch, rot_steps=(1, 3, 2), k_max=2, seed=SEED, h=H, sigma=SIGMA)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(SEED, H, SIGMA, s.galois)
    return s, o


# ------------------------------------------------------------------------------------------------ launchers


def _ntt_args(s, x, rows_pid, **kw):
    pr, fw, fws, iw, iws, ni, nis = s.tables()
    nrows = len(rows_pid)
    roff = torch.arange(nrows, dtype=torch.int32, device="cuda")
    rprime = torch.tensor(rows_pid, dtype=torch.int32, device="cuda")
    a = L.NttArgs()
    a.base, a.roff, a.rprime = x.data_ptr(), roff.data_ptr(), rprime.data_ptr()
    a.fw, a.fws, a.iw, a.iws, a.ninv, a.ninvs, a.pr = fw, fws, iw, iws, ni, nis, pr
    a.nrows, a.snum, a.xnum = nrows, 1, 1
    for k, v in kw.items():
        setattr(a, k, v)
    return a, (roff, rprime)


def _table(s):
    return L.kernel_table() if s.log_n == 16 else L.ring_table(14)


@pytest.mark.parametrize("which", ["s1", "s2"])
def test_ntt_launchers_match_oracle(which, request):
    s, o = request.getfixturevalue(which)
    rng = np.random.default_rng(11)
    pids = [0, 1, s.nq - 1, s.nq, s.rows - 1, 2]
    primes = [o.q[i] if i < o.nq else o.p[i - o.nq] for i in pids]
    x = np.stack([rng.integers(0, p, s.n, dtype=np.uint64) for p in primes])
    xd = dev(x)
    a, keep = _ntt_args(s, xd, pids)
    t = _table(s)
    assert t.ntt_fwd(C.cast(C.pointer(a), C.c_void_p), None) == 0
    want = x.copy()
    O.lib().orc_ntt_fwd(want, len(pids), np.array(primes, np.uint64), s.log_n)
    assert (host(xd) == want).all()
    assert t.ntt_inv(C.cast(C.pointer(a), C.c_void_p), None) == 0
    assert (host(xd) == x).all()


def test_ntt_batch_fp64_path_matches_oracle(s2):
    """Config 2's primes are all below 2^50, so the evaluator's transforms take the FP64 butterflies; rows with the
    extreme words (0, p - 1, (p +- 1) / 2) and uniform rows, forward and inverse, against the oracle."""
    s, o = s2
    rng = np.random.default_rng(14)
    nrows = 2 * s.nq + 5
    x = np.empty((nrows, s.n), np.uint64)
    for i in range(nrows):
        p = o.q[i % s.nq]
        kind = i % 5
        if kind == 0:
            x[i] = p - 1
        elif kind == 1:
            x[i] = np.where(np.arange(s.n) % 2 == 0, p - 1, 0)
        elif kind == 2:
            x[i] = rng.choice(np.array([0, 1, (p - 1) // 2, (p + 1) // 2, p - 1], np.uint64), s.n)
        else:
            x[i] = rng.integers(0, p, s.n, dtype=np.uint64)
    xd = dev(x)
    s.ntt_batch(xd, nrows)
    want = x.copy()
    O.lib().orc_ntt_batch(o.h, want, nrows, 0)
    assert (host(xd) == want).all()
    s.ntt_batch(xd, nrows, inverse=True)
    assert (host(xd) == x).all()
    inv_want = x.copy()
    O.lib().orc_ntt_batch(o.h, inv_want, nrows, 1)
    xd = dev(x)
    s.ntt_batch(xd, nrows, inverse=True)
    assert (host(xd) == inv_want).all()
    assert L.lib().pcb_device_timeouts() == 0  # the pipelined passes' bounded waits never ran out


def test_ntt_epilogues_and_sources(s2):
    s, o = s2
    rng = np.random.default_rng(12)
    pids = [3, 7, 30]
    primes = np.array([o.q[3], o.q[7], o.p[6]], np.uint64)
    n = s.n
    src = np.stack([rng.integers(0, int(p), n, dtype=np.uint64) for p in primes for _ in range(2)])  # 2 sources/row
    ex = np.stack([rng.integers(0, int(p), n, dtype=np.uint64) for p in primes])
    sc = rng.integers(1, int(min(primes)), s.rows, dtype=np.uint64)
    scs = np.array([(int(v) << 64) // int(primes[pids.index(i)]) if i in pids else 0 for i, v in enumerate(sc)], np.uint64)
    summed = np.stack([(src[2 * i].astype(object) + src[2 * i + 1]) % int(primes[i]) for i in range(3)]).astype(np.uint64)
    ref = summed.copy()
    O.lib().orc_ntt_fwd(ref, 3, primes, s.log_n)
    srcd, exd, scd, scsd = dev(src), dev(ex), dev(sc), dev(scs)
    soff = torch.tensor([0, 2, 4], dtype=torch.int32, device="cuda")
    t = _table(s)
    for epi in (1, 2, 3):
        base = torch.zeros((3, n), dtype=torch.int64, device="cuda")
        eout = dev(np.stack([rng.integers(0, int(p), n, dtype=np.uint64) for p in primes]))
        before = host(eout).astype(object)
        a, keep = _ntt_args(s, base, pids, src=srcd.data_ptr(), soff=soff.data_ptr(), snum=2, sstride=n, epi=epi,
                            eout=eout.data_ptr(), ex=exd.data_ptr(), es=scd.data_ptr(), ess=scsd.data_ptr())
        assert t.ntt_fwd(C.cast(C.pointer(a), C.c_void_p), None) == 0
        got = host(eout).astype(object)
        for i, pid in enumerate(pids):
            p, v, xs, w = int(primes[i]), ref[i].astype(object), ex[i].astype(object), int(sc[pid])
            if epi == 1:
                want = (xs - v) % p * w % p
            elif epi == 2:
                want = (before[i] + (xs - v) % p * w) % p
            else:
                want = (xs * w + v) % p
            assert (got[i] == want).all(), f"epilogue {epi} row {i}"


def test_bconv_launcher(s2):
    s, o = s2
    rng = np.random.default_rng(13)
    srcp = [0, 1, 2, 3]
    tgtp = [5, 9, 24, 31]
    primes = list(o.q) + list(o.p)
    bp = [primes[i] for i in srcp]
    pool = []
    pool += srcp + srcp
    B = 1
    for b in bp:
        B *= b
    pool += [pow(B // b % b, -1, b) for b in bp]
    pool += tgtp + tgtp
    for b in bp:
        pool += [(B // b) % primes[t] for t in tgtp]
    x = np.zeros((s.rows, s.n), np.uint64)
    for i in srcp:
        x[i] = rng.integers(0, primes[i], s.n, dtype=np.uint64)
    out = torch.zeros((s.rows, s.n), dtype=torch.int64, device="cuda")
    xd, poold = dev(x), dev(np.array(pool, np.uint64))
    jobs = (L.BconvJob * 1)(L.BconvJob(0, 0, 4, 4, 0, 0, 0, 0))
    jd = torch.from_numpy(np.frombuffer(bytes(jobs), np.uint8).copy()).cuda()
    a = L.BconvArgs()
    a.src, a.dst, a.jobs, a.pool, a.pr = xd.data_ptr(), out.data_ptr(), jd.data_ptr(), poold.data_ptr(), s.tables()[0]
    a.njobs, a.max_tgt = 1, 4
    assert _table(s).bconv(C.cast(C.pointer(a), C.c_void_p), None) == 0
    got = host(out)
    xs = x.astype(object)
    for j, t in enumerate(tgtp):
        y = [(xs[i] * pool[8 + k]) % bp[k] for k, i in enumerate(srcp)]
        want = sum(y[k] * ((B // bp[k]) % primes[t]) for k in range(4)) % primes[t]
        assert (got[t].astype(object) == want).all()


# ------------------------------------------------------------------------------------------------ evaluator


@pytest.mark.parametrize("which", ["s1", "s2"])
def test_keys_bit_exact(which, request):
    s, o = request.getfixturevalue(which)
    for idx in range(len(s.galois)):
        b, a = s.key_tensors(idx)
        ob, oa, _ = o.key(idx)
        assert (host(a) == oa).all(), f"key {idx} a"
        assert (host(b) == ob).all(), f"key {idx} b"


def _pair(s, o, x, top, slots=None):
    ct = s.encrypt(x, top=top, slots=slots)
    oc = o.encrypt(x, ct.slots, ct.scale, top)
    return ct, oc


def _eq(ct, oc, top, rows):
    g = host(ct.data[0])
    return (g[:, : top + 1] == oc[:, : top + 1]).all()


@pytest.mark.parametrize("which", ["s1", "s2"])
def test_encrypt_bit_exact_and_decrypts(which, request):
    s, o = request.getfixturevalue(which)
    rng = np.random.default_rng(1)
    x = rng.normal(0, 1, 256) / 8
    top = s.top()
    ct, oc = _pair(s, o, x, top)
    assert _eq(ct, oc, top, s.rows)
    got = s.decrypt_slots(ct)
    assert np.abs(got.real - x).max() < 1e-6


def test_mult_rescale_bit_exact(s1):
    s, o = s1
    rng = np.random.default_rng(2)
    x, y = rng.normal(0, 1, 512) / 8, rng.normal(0, 1, 512) / 8
    top = s.top()
    a, oa = _pair(s, o, x, top)
    b, ob = _pair(s, o, y, top)
    m = s.mult(a, b)
    om = o.mult(oa, ob, top)
    assert _eq(m, om, top, s.rows)
    s.rescale_one(m)
    om = o.rescale(om, top)
    assert _eq(m, om, top - 1, s.rows)
    got = s.decrypt_slots(m)
    assert np.abs(got.real - x * y).max() < 1e-6


@pytest.mark.parametrize("step", [1, 4, 64, -1])
def test_rotate_bit_exact(s1, step):
    s, o = s1
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 8192) / 8
    top = s.top()
    a, oa = _pair(s, o, x, top)
    r = s.rotate(a, step)
    assert _eq(r, o.rotate(oa, step, top), top, s.rows)
    assert np.abs(s.decrypt_slots(r).real - np.roll(x, -step)).max() < 1e-6


def test_rotate_lower_level_and_sum(s1):
    s, o = s1
    rng = np.random.default_rng(4)
    x = rng.normal(0, 1, 8192) / 8
    top = 4
    a, oa = _pair(s, o, x, top)
    r = s.rotate_and_sum(a, 1, 16)
    assert _eq(r, o.rotate_and_sum(oa, 1, 16, top), top, s.rows)
    want = sum(np.roll(x, -k) for k in range(16))
    assert np.abs(s.decrypt_slots(r).real - want).max() < 1e-5


def test_pt_ops_bit_exact(s1):
    s, o = s1
    rng = np.random.default_rng(5)
    x, w = rng.normal(0, 1, 512) / 8, rng.normal(0, 1, 512)
    top = s.top()
    a, oa = _pair(s, o, x, top)
    pt = s.pt(w, top, 2.0**40, a.slots)
    rows = s.encode(w, slots=a.slots, scale=2.0**40, top=top)
    assert (rows == o.encode(w, a.slots, 2.0**40, top)).all()
    assert _eq(s.mult_pt(a, pt, 2.0**40), o.mult_pt(oa, rows, top), top, s.rows)
    assert _eq(s.add_pt(a, pt), o.add_pt(oa, rows, top), top, s.rows)


def test_config2_relin_and_rotation_bit_exact(s2):
    s, o = s2
    rng = np.random.default_rng(6)
    x, y = rng.normal(0, 1, 1024) / 8, rng.normal(0, 1, 1024) / 8
    top = s.top()
    a, oa = _pair(s, o, x, top)
    b, ob = _pair(s, o, y, top)
    m = s.mult(a, b)
    assert _eq(m, o.mult(oa, ob, top), top, s.rows)
    r = s.rotate(a, 5)
    assert _eq(r, o.rotate(oa, 5, top), top, s.rows)
    # a level with a partial top digit (limbs 0..12: digits of 8 + 5 limbs)
    lo = 12
    a2, oa2 = _pair(s, o, x, lo)
    r2 = s.rotate(a2, 1)
    assert _eq(r2, o.rotate(oa2, 1, lo), lo, s.rows)
    # config 2's digits are as large as P (8 x 50 bits each), so a key switch adds ~N sigma digit / P ~ 2^18 to the
    # coefficients: ~1e-6 on slots at scale 2^40
    assert np.abs(s.decrypt_slots(r2).real[:1024] - np.roll(np.pad(x, (0, r2.slots - 1024)), -1)[:1024]).max() < 2e-5


def test_config2_rotate_sum_bit_exact(s2):
    # the rotations summed in the extended basis with one ModDown (the reference's rotate_sum): FP64 inner products
    # accumulated across keys, the ModDown epilogue adding x
    s, o = s2
    rng = np.random.default_rng(9)
    x = rng.normal(0, 1, 1024) / 8
    top = s.top() - 2
    a, oa = _pair(s, o, x, top)
    r = s.rotate_sum(a, [1, 5])
    assert _eq(r, o.rotate_sum(oa, [1, 5], top), top, s.rows)
    # five keys: two groups of inner products (4 + 1) summed by the ModDown as it reads them
    r5 = s.rotate_sum(a, [1, 5, 1, 5, 1])
    assert _eq(r5, o.rotate_sum(oa, [1, 5, 1, 5, 1], top), top, s.rows)
    want = x + np.roll(np.pad(x, (0, r.slots - 1024)), -1)[:1024] + np.roll(np.pad(x, (0, r.slots - 1024)), -5)[:1024]
    assert np.abs(s.decrypt_slots(r).real[:1024] - want).max() < 5e-5
    with pytest.raises(L.PcbError, match="identity"):
        s.rotate_sum(a, [1, s.n // 2])


def test_batched_ops_equal_single(s1):
    s, o = s1
    rng = np.random.default_rng(7)
    top = s.top()
    cts = [s.encrypt(rng.normal(0, 1, 512) / 8, top=top) for _ in range(3)]
    batch = fhe.Ct(torch.cat([c.data for c in cts]), top, cts[0].scale, cts[0].slots)
    rb = s.rotate(batch, 2)
    for i, c in enumerate(cts):
        r = s.rotate(c, 2)
        assert torch.equal(rb.data[i, :, : top + 1], r.data[0, :, : top + 1])


@pytest.mark.parametrize("which", ["s1", "s2"])
def test_sum_equals_pairwise_adds(which, request):
    s, o = request.getfixturevalue(which)
    rng = np.random.default_rng(8)
    top = s.top() - 1
    cts = [s.encrypt(rng.normal(0, 1, 64) / 8, top=top) for _ in range(5)]
    want = cts[0]
    for c in cts[1:]:
        want = s.add(want, c)
    got = s.sum(cts)
    assert torch.equal(got.data[:, :, : top + 1], want.data[:, :, : top + 1])
    inplace = s.sum(cts, out=cts[0])  # the output may be one of the inputs
    assert torch.equal(inplace.data[:, :, : top + 1], want.data[:, :, : top + 1])
    with pytest.raises(L.PcbError, match="33 inputs"):
        s.sum([cts[1]] * 33)


@pytest.mark.parametrize("which", ["s1", "s2"])
def test_hoisted_rotations_equal_plain(which, request):
    # one shared ModUp (crates/pc-gpu/src/rotate.rs:456): every output word for word the plain rotation's
    s, o = request.getfixturevalue(which)
    # config 2 (FP64 chain) takes its inner products in groups of up to 4 keys: 6 keyed steps make groups of 4 and 2
    steps = [1, 4, 0, -1] if which == "s1" else [5, 1, 1 << 15, 1, 5, 5, 1]
    rng = np.random.default_rng(8)
    top = s.top() - 1
    a = s.encrypt(rng.normal(0, 1, 256) / 8, top=top)
    if which == "s2":
        a = s.stack([a, s.encrypt(rng.normal(0, 1, 256) / 8, top=top)])  # a batch of two
    outs = s.rotate_hoisted(a, steps)
    for st, h in zip(steps, outs):
        p = s.rotate(a, st) if st % (s.n // 2) else a
        assert torch.equal(h.data[:, :, : top + 1], p.data[:, :, : top + 1]), st


def test_fp64_small_ring_bit_exact(s3):
    """The FP64 path at N = 2^14 (column pass in rounds of 3 stages): NTT batch, relinearized product, rotation,
    hoisted rotations in one group, rotate_sum and the radix ladder, all against the oracle word for word."""
    s, o = s3
    rng = np.random.default_rng(15)
    x = np.empty((2 * s.nq, s.n), np.uint64)
    for i in range(2 * s.nq):
        x[i] = rng.integers(0, o.q[i % s.nq], s.n, dtype=np.uint64)
    xd = dev(x)
    s.ntt_batch(xd, 2 * s.nq)
    want = x.copy()
    O.lib().orc_ntt_batch(o.h, want, 2 * s.nq, 0)
    assert (host(xd) == want).all()
    s.ntt_batch(xd, 2 * s.nq, inverse=True)
    assert (host(xd) == x).all()
    top = s.top()
    v, w = rng.normal(0, 1, 256) / 8, rng.normal(0, 1, 256) / 8
    a, oa = _pair(s, o, v, top)
    b, ob = _pair(s, o, w, top)
    assert _eq(s.mult(a, b), o.mult(oa, ob, top), top, s.rows)
    assert _eq(s.rotate(a, 3), o.rotate(oa, 3, top), top, s.rows)
    outs = s.rotate_hoisted(a, [1, 3, 2])
    for st, h in zip([1, 3, 2], outs):
        assert torch.equal(h.data[:, :, : top + 1], s.rotate(a, st).data[:, :, : top + 1]), st
    assert _eq(s.rotate_sum(a, [1, 2, 3]), o.rotate_sum(oa, [1, 2, 3], top), top, s.rows)
    r = s.rotate_and_sum(a, 1, 4, radix_bits=2)
    assert _eq(r, o.rotate_and_sum(oa, 1, 4, top, 2), top, s.rows)
    assert np.abs(s.decrypt_slots(r).real - sum(np.roll(v, -k) for k in range(4))).max() < 1e-4
