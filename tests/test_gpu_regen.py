"""The regenerated-key inner products (ks_dot_regen, ks_dot_key) through the launcher table, word for word against
exact sums whose key `a` rows come from the oracle's u64 expander lane (pinned to the reference's frozen KSKB vectors):
dense and table-addressed `b`, the relinearization epilogue, Galois outputs, c0 modes, accumulation, and digits past
nregen read from a resident `a` (crates/pc-kernels/kernels/args.cuh:273-304, :764-768)."""
import ctypes as C

import numpy as np
import pytest
import torch

from perseus_b200 import _lib as L
from tests import _oracle as O

pytestmark = pytest.mark.gpu

LOGN = 16
N = 1 << LOGN


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()


def ptr(x):
    return C.cast(C.pointer(x), C.c_void_p)


@pytest.fixture(scope="module")
def env():
    q = O.ntt_primes(50, LOGN, 3)
    p = O.ntt_primes(60, LOGN, 1)
    primes = q + p  # prime ids 0..2 Q, 3 special
    pc = np.zeros((4, 8), np.uint64)
    for i, x in enumerate(primes):
        O.lib().orc_prime_const(x, pc[i])
    return primes, dev(pc), L.kernel_table()


def rand_rows(rng, primes, shape):
    out = np.empty(shape + (len(primes), N), np.uint64)
    for r, x in enumerate(primes):
        out[..., r, :] = rng.integers(0, x, shape + (N,), dtype=np.uint64)
    return out


def a_row(seed, d, p):
    return O.expand_row(seed, d, p, O.TAG_KSKA, LOGN).astype(object)


def ks_base(primes, pc, K, ndig, c1d, mud, rows, digit_of):
    a = L.KsArgs()
    a.c1, a.modup, a.pr = c1d.data_ptr(), mud.data_ptr(), pc.data_ptr()
    a.rows, a.digit_of = rows.data_ptr(), digit_of.data_ptr()
    a.ct_stride = len(primes) * N
    a.mu_ct_stride, a.mu_digit_stride = ndig * len(primes) * N, len(primes) * N
    a.out_ct_stride = len(primes) * N
    a.key_digit_stride = len(primes) * N
    a.K, a.R, a.ndig, a.nq, a.nrows = K, 1, ndig, 3, rows.numel()
    return a


def digit_sum(primes, K, ndig, c1, mu, rows, dof, b_of, a_of):
    """[K][2][t] exact sums mod p: part 0 = sum_d x_d b_d, part 1 = sum_d x_d a_d (x_d = c1 on the row's own digit)."""
    out = {}
    for t in rows:
        p = primes[t]
        for c in range(K):
            s0 = np.zeros(N, object)
            s1 = np.zeros(N, object)
            for d in range(ndig):
                x = (c1[c, t] if t < 3 and dof[t] == d else mu[c, d, t]).astype(object)
                s0 += x * b_of(d, t)
                s1 += x * a_of(d, t)
            out[c, t] = (s0 % p, s1 % p)
    return out


@pytest.mark.parametrize("K,tab", [(1, False), (2, False), (3, True)])
def test_ks_dot_regen(env, K, tab):
    primes, pc, T = env
    rng = np.random.default_rng(K)
    ndig, R = 2, len(primes)
    seed = rng.integers(0, 2**32, 8, dtype=np.uint64).astype(np.uint32)
    c1 = rand_rows(rng, primes, (K,))
    mu = rand_rows(rng, primes, (K, ndig))
    b = rand_rows(rng, primes, (ndig,))
    dof = [0, 0, 1]
    rows_l = [0, 1, 3] if tab else [0, 1, 2, 3]
    rows = torch.tensor(rows_l, dtype=torch.int32, device="cuda")
    digit_of = torch.tensor(dof, dtype=torch.int32, device="cuda")
    c1d, mud = dev(c1), dev(mu)
    out0 = torch.zeros((K, R, N), dtype=torch.int64, device="cuda")
    out1 = torch.zeros_like(out0)
    a = L.KsRegenArgs()
    a.ks = ks_base(primes, pc, K, ndig, c1d, mud, rows, digit_of)
    a.ks.out0, a.ks.out1 = out0.data_ptr(), out1.data_ptr()
    seedd = torch.from_numpy(seed.view(np.int32).copy()).cuda()
    a.seed = seedd.data_ptr()
    keep = []
    if tab:  # key holding Q rows 0..1 (q_top 1) and the special row at slot 2: [digit][slot][N]
        bt = np.stack([b[:, 0], b[:, 1], b[:, 3]], 1)
        btd = dev(bt)
        tabd = dev(np.array([btd.data_ptr()], np.uint64))
        keep += [btd, tabd]
        a.key.kb, a.key.row_words, a.key.q_top, a.key.srows = tabd.data_ptr(), N, 1, 3
    else:
        bd = dev(b)
        kbd = dev(np.array([bd.data_ptr()], np.uint64))
        keep += [bd, kbd]
        a.ks.kb = kbd.data_ptr()
    assert T.ks_dot_regen(ptr(a), None) == 0
    want = digit_sum(primes, K, ndig, c1, mu, rows_l, dof, lambda d, t: b[d, t].astype(object),
                     lambda d, t: a_row(seed, d, primes[t]))
    g0, g1 = host(out0), host(out1)
    for (c, t), (s0, s1) in want.items():
        assert (g0[c, t].astype(object) == s0).all() and (g1[c, t].astype(object) == s1).all(), (c, t)


def test_ks_dot_regen_epilogue(env):
    """use_epi: dst = alpha dst + (dot - conv) binv, + k on part 0, + add (both parts)."""
    primes, pc, T = env
    rng = np.random.default_rng(7)
    K, ndig, R = 2, 2, len(primes)
    seed = rng.integers(0, 2**32, 8, dtype=np.uint64).astype(np.uint32)
    c1, mu, b = rand_rows(rng, primes, (K,)), rand_rows(rng, primes, (K, ndig)), rand_rows(rng, primes, (ndig,))
    dst, conv, add = (rand_rows(rng, primes, (K, 2)) for _ in range(3))
    dof, rows_l = [0, 0, 1], [0, 1, 2]
    sc = [int(rng.integers(1, x)) for x in primes]
    al = [int(rng.integers(1, x)) for x in primes]
    kk = [int(rng.integers(0, x)) for x in primes]
    kk[1] = primes[1]  # a raw word equal to p
    sh = lambda v: [(x << 64) // p for x, p in zip(v, primes)]
    dev_u = lambda v: dev(np.array(v, np.uint64))
    rows = torch.tensor(rows_l, dtype=torch.int32, device="cuda")
    digit_of = torch.tensor(dof, dtype=torch.int32, device="cuda")
    c1d, mud, bd = dev(c1), dev(mu), dev(b)
    dstd, convd, addd = dev(dst), dev(conv), dev(add)
    kbd = dev(np.array([bd.data_ptr()], np.uint64))
    seedd = torch.from_numpy(seed.view(np.int32).copy()).cuda()
    keep = [dev_u(sc), dev_u(sh(sc)), dev_u(al), dev_u(sh(al)), dev_u(kk)]
    a = L.KsRegenArgs()
    a.ks = ks_base(primes, pc, K, ndig, c1d, mud, rows, digit_of)
    a.ks.kb, a.ks.out_ct_stride = kbd.data_ptr(), 2 * R * N
    a.seed = seedd.data_ptr()
    a.use_epi = 1
    e = a.epi
    e.dst, e.conv, e.part_stride = dstd.data_ptr(), convd.data_ptr(), R * N
    e.binv, e.binvs, e.alpha, e.alphas, e.k = [x.data_ptr() for x in keep]
    a.add = addd.data_ptr()
    assert T.ks_dot_regen(ptr(a), None) == 0
    want = digit_sum(primes, K, ndig, c1, mu, rows_l, dof, lambda d, t: b[d, t].astype(object),
                     lambda d, t: a_row(seed, d, primes[t]))
    got = host(dstd)
    for (c, t), sums in want.items():
        p = primes[t]
        for part in range(2):
            v = (al[t] * dst[c, part, t].astype(object) + (sums[part] - conv[c, part, t].astype(object)) * sc[t]) % p
            if part == 0:
                v = (v + kk[t] % p) % p
            v = (v + add[c, part, t].astype(object)) % p
            assert (got[c, part, t].astype(object) == v).all(), (c, t, part)
    assert (got[:, :, 3] == dst[:, :, 3]).all()  # rows outside the launch untouched


def test_ks_dot_key(env):
    """R = 2 keys through a table (digit 0 regenerated, digit 1 resident), Galois outputs, c0 mode 1, accumulate."""
    primes, pc, T = env
    rng = np.random.default_rng(21)
    K, ndig, R = 2, 2, len(primes)
    seeds = [rng.integers(0, 2**32, 8, dtype=np.uint64).astype(np.uint32) for _ in range(2)]
    c1, mu, c0 = rand_rows(rng, primes, (K,)), rand_rows(rng, primes, (K, ndig)), rand_rows(rng, primes, (K,))
    bs = [rand_rows(rng, primes, (ndig,)) for _ in range(2)]
    kas = [rand_rows(rng, primes, (ndig,)) for _ in range(2)]  # digit 1 of each key read from here
    prev = rand_rows(rng, primes, (2, K, 2))  # [key][c][part] previous outputs (accumulate)
    dof, rows_l = [0, 0, 1], [0, 1, 2, 3]
    gal = [O.lib().orc_rotation_galois(3, LOGN), O.lib().orc_rotation_galois(-5, LOGN)]
    Pm = [primes[3] % x for x in primes]
    rows = torch.tensor(rows_l, dtype=torch.int32, device="cuda")
    digit_of = torch.tensor(dof, dtype=torch.int32, device="cuda")
    c1d, mud, c0d = dev(c1), dev(mu), dev(c0)
    bds, kads = [dev(x) for x in bs], [dev(x) for x in kas]
    kbt = dev(np.array([x.data_ptr() for x in bds], np.uint64))
    kat = dev(np.array([x.data_ptr() for x in kads], np.uint64))
    sds = [torch.from_numpy(s_.view(np.int32).copy()).cuda() for s_ in seeds]
    seedt = dev(np.array([x.data_ptr() for x in sds], np.uint64))
    autok = torch.tensor(gal, dtype=torch.int32, device="cuda")
    pm = dev(np.array(Pm, np.uint64))
    pms = dev(np.array([(x << 64) // p for x, p in zip(Pm, primes)], np.uint64))
    outs = dev(np.ascontiguousarray(prev[:, :, 0]))
    outs1 = dev(np.ascontiguousarray(prev[:, :, 1]))
    a = L.KsKeyArgs()
    a.ks = ks_base(primes, pc, K, ndig, c1d, mud, rows, digit_of)
    a.ks.c0, a.ks.ka, a.ks.autok, a.ks.pmod, a.ks.pmods = c0d.data_ptr(), kat.data_ptr(), autok.data_ptr(), \
        pm.data_ptr(), pms.data_ptr()
    a.ks.out0, a.ks.out1 = outs.data_ptr(), outs1.data_ptr()
    a.ks.out_rot_stride = K * R * N
    a.ks.R, a.ks.c0_mode = 2, 1 | 4
    a.ks.ct_stride = R * N
    a.key.kb, a.key.seed, a.key.row_words, a.key.q_top, a.key.srows, a.key.nregen = kbt.data_ptr(), \
        seedt.data_ptr(), N, -1, R, 1
    assert T.ks_dot_key(ptr(a), None) == 0
    g0, g1 = host(outs), host(outs1)
    for r in range(2):
        want = digit_sum(primes, K, ndig, c1, mu, rows_l, dof, lambda d, t: bs[r][d, t].astype(object),
                         lambda d, t: a_row(seeds[r], d, primes[t]) if d < 1 else kas[r][d, t].astype(object))
        slots = np.array([O.lib().orc_automorph_slot(gal[r], i, LOGN) for i in range(N)])
        for (c, t), (s0, s1) in want.items():
            p = primes[t]
            if t < 3:
                s0 = (s0 + Pm[t] * c0[c, t].astype(object)) % p
            e0 = prev[r, c, 0, t].astype(object).copy()
            e1 = prev[r, c, 1, t].astype(object).copy()
            e0[slots] = (e0[slots] + s0) % p
            e1[slots] = (e1[slots] + s1) % p
            assert (g0[r, c, t].astype(object) == e0).all() and (g1[r, c, t].astype(object) == e1).all(), (r, c, t)
