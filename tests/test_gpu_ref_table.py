"""The reference's OWN kernel table beside this build's: the same arguments must give the same words.

`oracle/_ref/libpcref_u64.so` is the reference's `pc_table_u64_barrett64` and `oracle/_ref/libpcref_ring14.so` its
`pc_ring_u64_14`, compiled from the reference's sources for sm_100a by `make -C oracle ref REF=<reference root>`
(test infrastructure only: the product never loads them). Two kinds of checks:

1. Launchers. Every entry that both tables implement runs on the same inputs and arguments (fresh copies for each
   table) and must write the same words: the NTT (both directions, every epilogue, out-of-place and summed sources,
   per-row inverse scales), base conversion, the key inner products (c0 modes, accumulation, automorphism; with
   `a` regenerated from a seed, key tables, the fused relinearization epilogue), tensor,
   ModDown epilogue, rescale (one and two dropped primes), automorphism, the element-wise and plaintext-operand
   entries, key expansion, key generation and encryption; rows mix 50-bit and 60-bit primes.
2. Compositions. The reference's launchers run in its device runtime's order — ModUp (INTT with the digit pre factor,
   bconv of every live digit, NTT of the targets: crates/pc-gpu/src/ks.rs:954-1043), the key inner product
   (crates/pc-gpu/src/ks.rs:1109), ModDown (INTT of the special rows, bconv P -> Q, NTT with epilogue 1:
   crates/pc-gpu/src/ks.rs:1620-1656), relinearization (crates/pc-gpu/src/relin.rs:84-134) and rescale (INTT of the
   top, rescale_coef, NTT, rescale_combine: crates/pc-gpu/src/rescale.rs:230) — on the keys of a config-2 session,
   and must equal the oracle's rotation, relinearized product and rescale word for word. This pins the oracle's
   compositions (and through it every evaluator parity test) to the reference's own code.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

from perseus_b200 import _lib as L
from perseus_b200 import fhe
from tests import _oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_U64 = os.path.join(ROOT, "oracle", "_ref", "libpcref_u64.so")
REF_R14 = os.path.join(ROOT, "oracle", "_ref", "libpcref_ring14.so")

LOGN = 16
N = 1 << LOGN
KS_ACC = 4


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.uint64)).view(np.int64)).cuda()


def ptr(x):
    return C.cast(C.pointer(x), C.c_void_p)


def shoup(w, p):
    return (int(w) << 64) // int(p)


_REF = {}


def ref_table(ring14=False):
    path = REF_R14 if ring14 else REF_U64
    if not os.path.exists(path):
        pytest.skip(f"{os.path.relpath(path, ROOT)} not built (make -C oracle ref REF=<reference root>)")
    if path not in _REF:
        lib = C.CDLL(path)
        if ring14:
            f = lib.pc_ring_u64_14
            f.restype = C.POINTER(L.RingTable)
        else:
            f = lib.pc_table_u64_barrett64
            f.restype = C.POINTER(L.KernelTable)
        _REF[path] = (lib, f().contents)
    return _REF[path][1]


def tables():
    return [("ours", L.kernel_table()), ("ref", ref_table())]


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def run_both(entry, make, tabs=None):
    """make() builds fresh device inputs/outputs and returns (args, outputs, keep-alive); the entry of each table runs
    on its own set. Returns {table name: [host copies of the outputs]}."""
    got = {}
    for name, t in tabs or tables():
        args, outs, keep = make()
        rc = getattr(t, entry)(ptr(args), stream())
        assert rc == 0, f"{name} {entry} returned {rc}"
        torch.cuda.synchronize()
        got[name] = [host(o) for o in outs]
    return got


def same(got):
    a, b = got["ours"], got["ref"]
    assert len(a) == len(b)
    for i, (x, y) in enumerate(zip(a, b)):
        assert x.shape == y.shape and (x == y).all(), f"output {i} differs ({int((x != y).sum())} words)"


# ------------------------------------------------------------------------------------------------ environment


class Env:
    """Prime ids 0..11: 8 primes below 2^50 then 4 below 2^60 (both arithmetic widths of the u64 word), with the
    reference's constant and twiddle tables ([prime id][N], Shoup companions; N^-1 per prime id)."""

    def __init__(self, logn=LOGN):
        self.logn, self.n = logn, 1 << logn
        self.primes = O.ntt_primes(50, logn, 8) + O.ntt_primes(60, logn, 4)
        self.R = len(self.primes)
        pc = np.zeros((self.R, 8), np.uint64)
        fw = np.zeros((self.R, self.n), np.uint64)
        fws, iw, iws = np.zeros_like(fw), np.zeros_like(fw), np.zeros_like(fw)
        ninv, ninvs = np.zeros(self.R, np.uint64), np.zeros(self.R, np.uint64)
        for i, p in enumerate(self.primes):
            O.lib().orc_prime_const(p, pc[i])
            psi = O.lib().orc_root_of_unity(2 * self.n, p)
            O.lib().orc_twiddles(p, psi, logn, fw[i], fws[i], iw[i], iws[i])
            ninv[i] = pow(self.n, -1, p)
            ninvs[i] = shoup(ninv[i], p)
        self.pc, self.fw, self.fws, self.iw, self.iws = dev(pc), dev(fw), dev(fws), dev(iw), dev(iws)
        self.ninv, self.ninvs = dev(ninv), dev(ninvs)
        self.P = np.array(self.primes, np.uint64)

    def rows(self, rng, pids, lead=()):
        """random canonical rows [*lead, len(pids), N], row j mod primes[pids[j]]"""
        out = np.empty(tuple(lead) + (len(pids), self.n), np.uint64)
        for j, pid in enumerate(pids):
            out[..., j, :] = rng.integers(0, self.primes[pid], tuple(lead) + (self.n,), dtype=np.uint64)
        return out

    def cts(self, rng, K):
        """K ciphertexts [K][2][R][N] (row r mod prime id r)"""
        return self.rows(rng, range(self.R), lead=(K, 2))

    def ntt_args(self, base, roff, rprime, keep, **kw):
        a = L.NttArgs()
        ro = torch.tensor(roff, dtype=torch.int32, device="cuda")
        rp = torch.tensor(rprime, dtype=torch.int32, device="cuda")
        keep += [ro, rp]
        a.base, a.roff, a.rprime = base.data_ptr(), ro.data_ptr(), rp.data_ptr()
        a.fw, a.fws, a.iw, a.iws = self.fw.data_ptr(), self.fws.data_ptr(), self.iw.data_ptr(), self.iws.data_ptr()
        a.ninv, a.ninvs, a.pr = self.ninv.data_ptr(), self.ninvs.data_ptr(), self.pc.data_ptr()
        a.nrows, a.snum, a.xnum = len(roff), 1, 1
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    def cref(self, t):
        return L.PolyRef(t.data_ptr(), 2 * self.R * self.n, self.R * self.n)


@pytest.fixture(scope="module")
def env():
    return Env()


def test_headers_agree():
    ours, ref = L.kernel_table(), ref_table()
    assert (ours.abi, ours.word_bytes, ours.mm, ours.log_n) == (ref.abi, ref.word_bytes, ref.mm, ref.log_n)
    r14o, r14r = L.ring_table(14), ref_table(ring14=True)
    assert (r14o.abi, r14o.word_bytes, r14o.mm, r14o.log_n) == (r14r.abi, r14r.word_bytes, r14r.mm, r14r.log_n)


# ------------------------------------------------------------------------------------------------ NTT


@pytest.mark.parametrize("chunk", [0, 5])
def test_ntt_plain_both_directions(env, chunk):
    rng = np.random.default_rng(1)
    pids = [0, 3, 7, 8, 11, 2, 9, 1, 10, 4, 5]
    x = env.rows(rng, pids)
    x[0, :8] = env.primes[0] - 1  # extreme words
    x[4, 8:16] = 0

    def make(inverse):
        def mk():
            keep = []
            xd = dev(x)
            a = env.ntt_args(xd, list(range(len(pids))), pids, keep, chunk=chunk)
            return a, [xd], keep
        return mk

    fwd = run_both("ntt_fwd", make(False))
    same(fwd)
    want = x.copy()
    O.lib().orc_ntt_fwd(want, len(pids), env.P[pids], LOGN)
    assert (fwd["ours"][0] == want).all()
    inv = run_both("ntt_inv", make(True))
    same(inv)
    want = x.copy()
    O.lib().orc_ntt_inv(want, len(pids), env.P[pids], LOGN)
    assert (inv["ref"][0] == want).all()


@pytest.mark.parametrize("epi,with_ed", [(1, False), (2, False), (2, True), (3, False)])
def test_ntt_epilogues_sources(env, epi, with_ed):
    """Out-of-place first pass summing snum = 2 source rows, the epilogue's x summed over xnum = 2 rows."""
    rng = np.random.default_rng(10 + epi)
    pids = [1, 6, 9, 11]
    nr = len(pids)
    src = env.rows(rng, pids, lead=(2,))          # [2][nr][N]: source j of row i at soff[i] + j sstride
    ex = env.rows(rng, pids, lead=(2,))           # x = ex[0] + ex[1]
    eo0 = env.rows(rng, pids)
    ed = env.rows(rng, pids)
    es = np.array([rng.integers(1, p) for p in env.primes], np.uint64)
    ess = np.array([shoup(v, p) for v, p in zip(es, env.primes)], np.uint64)

    def mk():
        keep = []
        base = torch.zeros((nr, N), dtype=torch.int64, device="cuda")
        s, x, eo, e, sc, scs = dev(src), dev(ex), dev(eo0), dev(ed), dev(es), dev(ess)
        soff = torch.arange(nr, dtype=torch.int32, device="cuda")
        keep += [s, x, e, sc, scs, soff]
        a = env.ntt_args(base, list(range(nr)), pids, keep, src=s.data_ptr(), soff=soff.data_ptr(), snum=2,
                         sstride=nr * N, epi=epi, eout=eo.data_ptr(), ex=x.data_ptr(), xnum=2, xstride=nr * N,
                         es=sc.data_ptr(), ess=scs.data_ptr(), ed=e.data_ptr() if with_ed else None)
        # the result is eout; base only holds the first pass's intermediate (the ABI's out-of-place form with an
        # epilogue writes no transform to base), which is not an output
        return a, [eo], keep

    same(run_both("ntt_fwd", mk))


def test_ntt_inverse_row_scales(env):
    rng = np.random.default_rng(3)
    pids = [0, 8, 5, 10, 7]
    x = env.rows(rng, pids)
    es = np.array([rng.integers(1, env.primes[p]) for p in pids], np.uint64)  # per ROW (not per prime id)
    ess = np.array([shoup(v, env.primes[p]) for v, p in zip(es, pids)], np.uint64)

    def mk():
        keep = []
        xd, sc, scs = dev(x), dev(es), dev(ess)
        keep += [sc, scs]
        return env.ntt_args(xd, list(range(len(pids))), pids, keep, es=sc.data_ptr(), ess=scs.data_ptr()), [xd], keep

    same(run_both("ntt_inv", mk))


def test_ring14_tables():
    """The 2^14 ring tables: NTT both directions, bconv and the element-wise entries."""
    e14 = Env(14)
    tabs = [("ours", L.ring_table(14)), ("ref", ref_table(ring14=True))]
    rng = np.random.default_rng(4)
    pids = list(range(e14.R))
    x = e14.rows(rng, pids)

    def mk():
        keep = []
        xd = dev(x)
        return e14.ntt_args(xd, pids, pids, keep), [xd], keep

    for entry in ("ntt_fwd", "ntt_inv"):
        got = run_both(entry, mk, tabs)
        same(got)
        want = x.copy()
        (O.lib().orc_ntt_fwd if entry == "ntt_fwd" else O.lib().orc_ntt_inv)(want, e14.R, e14.P, 14)
        assert (got["ours"][0] == want).all()
    _bconv_case(e14, tabs, seed=5)
    _ew_cases(e14, tabs, seed=6)


# ------------------------------------------------------------------------------------------------ bconv


def _bconv_pool(primes, srcp, tgtp, src_rows, tgt_rows, rng):
    B = 1
    for i in srcp:
        B *= primes[i]
    pre = [pow(B // primes[i] % primes[i], -1, primes[i]) for i in srcp]
    M = [[(B // primes[i]) % primes[t] for t in tgtp] for i in srcp]
    return list(src_rows) + list(srcp) + pre + list(tgt_rows) + list(tgtp) + [v for row in M for v in row]


def _bconv_case(e, tabs, seed, entry="bconv"):
    """Four jobs over one source buffer: 1, 3, 8 and 12 sources, prescaled and not, row offsets on both sides."""
    rng = np.random.default_rng(seed)
    n = e.n
    nsrc_rows = 2 * e.R
    x = np.zeros((nsrc_rows, n), np.uint64)  # row r (and r + R) holds residues mod prime id r
    for r in range(nsrc_rows):
        x[r] = rng.integers(0, e.primes[r % e.R], n, dtype=np.uint64)
    specs = [  # (src prime ids, tgt prime ids, src_off, dst_off, prescaled)
        ([4], [0, 11, 7], 0, 0, 0),
        ([0, 1, 2], [3, 8, 9, 10, 11, 5], e.R, e.R, 1),
        ([0, 1, 2, 3, 4, 5, 6, 7], [8, 9, 10, 11], 0, 2 * e.R, 0),
        (list(range(4, 12)) + [0, 1, 2], [3], 0, 3 * e.R, 1),  # 11 sources, 50- and 60-bit
    ]
    pool, jobs = [], []
    for srcp, tgtp, soff, doff, pres in specs:
        off = len(pool)
        pool += _bconv_pool(e.primes, srcp, tgtp, srcp, tgtp, rng)
        jobs.append(L.BconvJob(soff, doff, len(srcp), len(tgtp), off, 0, pres, 0))
    jarr = (L.BconvJob * len(jobs))(*jobs)
    jbytes = np.frombuffer(bytes(jarr), np.uint8).copy()
    max_tgt = max(len(s[1]) for s in specs)

    def mk():
        keep = []
        xd, pd = dev(x), dev(np.array(pool, np.uint64))
        jd = torch.from_numpy(jbytes.copy()).cuda()
        out = torch.zeros((4 * e.R, n), dtype=torch.int64, device="cuda")
        keep += [xd, pd, jd]
        a = L.BconvArgs()
        a.src, a.dst, a.jobs, a.pool, a.pr = xd.data_ptr(), out.data_ptr(), jd.data_ptr(), pd.data_ptr(), e.pc.data_ptr()
        a.njobs, a.max_tgt = len(jobs), max_tgt
        return a, [out], keep

    got = run_both(entry, mk, tabs)
    same(got)
    # and the exact fast-conversion sum for job 2 (8 sources -> the 60-bit targets)
    srcp, tgtp, soff, doff, pres = specs[2]
    B = 1
    for i in srcp:
        B *= e.primes[i]
    xs = x.astype(object)
    for k, t in enumerate(tgtp):
        y = [xs[soff + i] * pow(B // e.primes[i] % e.primes[i], -1, e.primes[i]) % e.primes[i] for i in srcp]
        want = sum(yv * ((B // e.primes[i]) % e.primes[t]) for yv, i in zip(y, srcp)) % e.primes[t]
        assert (got["ref"][0][doff + t].astype(object) == want).all()


def test_bconv(env):
    _bconv_case(env, tables(), seed=20)


def test_bconv_wide(env):
    """bconv_wide: on 64-bit words the reference's wide kernel takes jobs of up to 16 sources, as bconv does"""
    _bconv_case(env, tables(), seed=21, entry="bconv_wide")


# ------------------------------------------------------------------------------------------------ key inner product


@pytest.mark.parametrize("K,R,c0_mode,autok", [(1, 1, 0, 1), (3, 2, 1, 0), (2, 2, 2, 0), (4, 1, 1 | KS_ACC, 0),
                                              (8, 1, 0, 0)])
def test_ks_dot(env, K, R, c0_mode, autok):
    rng = np.random.default_rng(30 + K + 7 * R + c0_mode)
    nq, ndig = 8, 3
    digit_of = np.array([t // 3 for t in range(nq)] + [-1] * (env.R - nq), np.int32)
    rows = np.array(list(range(7)) + [8, 9, 10, 11], np.uint32)  # Q rows 0..6 (a partial top digit), 4 special rows
    ks = [(int(2 * rng.integers(1, N) + 1) if autok == 0 else 1) for _ in range(R)]
    c1 = env.cts(rng, K)[:, 1]                     # [K][R][N]
    c0 = env.cts(rng, K)[:, 0]
    mu = env.rows(rng, range(env.R), lead=(K, ndig))   # [K][ndig][R][N]
    kb = [env.rows(rng, range(env.R), lead=(ndig,)) for _ in range(R)]
    ka = [env.rows(rng, range(env.R), lead=(ndig,)) for _ in range(R)]
    o0 = env.rows(rng, range(env.R), lead=(K, R))      # [K][R keys][rows][N] (accumulated onto in KS_ACC)
    o1 = env.rows(rng, range(env.R), lead=(K, R))
    pm = np.array([rng.integers(1, p) for p in env.primes], np.uint64)
    pms = np.array([shoup(v, p) for v, p in zip(pm, env.primes)], np.uint64)

    def mk():
        keep = [dev(c1), dev(c0), dev(mu), dev(pm), dev(pms)]
        c1d, c0d, mud, pmd, pmsd = keep[:5]
        kbd, kad = [dev(v) for v in kb], [dev(v) for v in ka]
        keep += kbd + kad
        kbt = dev(np.array([t.data_ptr() for t in kbd], np.uint64))
        kat = dev(np.array([t.data_ptr() for t in kad], np.uint64))
        autd = torch.tensor(ks, dtype=torch.int32, device="cuda")
        rowd = torch.tensor(rows.astype(np.int32), dtype=torch.int32, device="cuda")
        digd = torch.tensor(digit_of, dtype=torch.int32, device="cuda")
        out0, out1 = dev(o0), dev(o1)
        keep += [kbt, kat, autd, rowd, digd]
        a = L.KsArgs()
        a.c1, a.modup, a.c0, a.out0, a.out1 = c1d.data_ptr(), mud.data_ptr(), c0d.data_ptr(), out0.data_ptr(), \
            out1.data_ptr()
        a.kb, a.ka, a.autok, a.rows, a.digit_of = kbt.data_ptr(), kat.data_ptr(), autd.data_ptr(), rowd.data_ptr(), \
            digd.data_ptr()
        a.pmod, a.pmods, a.pr = pmd.data_ptr(), pmsd.data_ptr(), env.pc.data_ptr()
        a.ct_stride, a.mu_ct_stride, a.mu_digit_stride = env.R * N, ndig * env.R * N, env.R * N
        a.out_ct_stride, a.out_rot_stride, a.key_digit_stride = R * env.R * N, env.R * N, env.R * N
        a.K, a.R, a.ndig, a.c0_mode, a.nq, a.nrows = K, R, ndig, c0_mode, nq, len(rows)
        return a, [out0, out1], keep

    same(run_both("ks_dot", mk))


@pytest.mark.parametrize("K,tab,epi", [(1, False, False), (3, True, False), (4, False, True), (2, True, True)])
def test_ks_dot_regen(env, K, tab, epi):
    """The relinearization inner product with `a` regenerated from the seed: dense or key-table `b`, plain outputs or
    the fused epilogue (alpha, dbl, k, add)."""
    rng = np.random.default_rng(140 + K)
    nq, ndig = 8, 3
    digit_of = np.array([t // 3 for t in range(nq)] + [-1] * (env.R - nq), np.int32)
    rows = list(range(6)) + [8, 10, 11]
    seed = rng.integers(0, 1 << 32, 8, dtype=np.uint64).astype(np.uint32)
    c1 = env.cts(rng, K)[:, 1]
    mu = env.rows(rng, range(env.R), lead=(K, ndig))
    b = env.rows(rng, range(env.R), lead=(ndig,))
    q_top, srows = 5, 6 + 4
    bt = np.concatenate([b[:, :6], b[:, 8:12]], 1)  # key table: Q ids 0..5 at their slot, specials after
    dst, conv, add = env.cts(rng, K), env.cts(rng, K), env.cts(rng, K)
    vals = [np.array([rng.integers(1, p) for p in env.primes], np.uint64) for _ in range(3)]
    binv, alpha, kc = vals
    sh = [np.array([shoup(v, p) for v, p in zip(arr, env.primes)], np.uint64) for arr in (binv, alpha)]

    def mk():
        keep = [dev(c1), dev(mu), dev(b), dev(bt), torch.tensor(rows, dtype=torch.int32, device="cuda"),
                torch.tensor(digit_of, dtype=torch.int32, device="cuda"),
                torch.from_numpy(seed.view(np.int32).copy()).cuda()]
        c1d, mud, bd, btd, rd, dd, sd = keep
        kb = dev(np.array([bd.data_ptr()], np.uint64))
        kt = dev(np.array([btd.data_ptr()], np.uint64))
        extra = [dev(binv), dev(sh[0]), dev(alpha), dev(sh[1]), dev(kc), dev(conv), dev(add)]
        keep += [kb, kt] + extra
        out0 = torch.zeros((K, env.R, N), dtype=torch.int64, device="cuda")
        out1 = torch.zeros_like(out0)
        dd_ = dev(dst)
        a = L.KsRegenArgs()
        k = a.ks
        k.c1, k.modup, k.pr, k.rows, k.digit_of = c1d.data_ptr(), mud.data_ptr(), env.pc.data_ptr(), rd.data_ptr(), \
            dd.data_ptr()
        k.ct_stride, k.mu_ct_stride, k.mu_digit_stride = env.R * N, ndig * env.R * N, env.R * N
        k.key_digit_stride = env.R * N
        k.K, k.R, k.ndig, k.nq, k.nrows = K, 1, ndig, nq, len(rows)
        a.seed = sd.data_ptr()
        if tab:
            a.key.kb, a.key.row_words, a.key.q_top, a.key.srows = kt.data_ptr(), N, q_top, srows
        else:
            k.kb = kb.data_ptr()
        if epi:
            k.out_ct_stride = 2 * env.R * N
            a.use_epi, a.add = 1, extra[6].data_ptr()
            e = a.epi
            e.dst, e.conv, e.part_stride, e.dbl = dd_.data_ptr(), extra[5].data_ptr(), env.R * N, 1
            e.binv, e.binvs, e.alpha, e.alphas, e.k = [x.data_ptr() for x in extra[:5]]
            return a, [dd_], keep
        k.out_ct_stride = env.R * N
        k.out0, k.out1 = out0.data_ptr(), out1.data_ptr()
        return a, [out0, out1], keep

    same(run_both("ks_dot_regen", mk))


@pytest.mark.parametrize("K,R,nregen,c0_mode", [(1, 1, 3, 0), (2, 2, 1, 1 | KS_ACC), (4, 3, 2, 2), (3, 1, 0, 1)])
def test_ks_dot_key(env, K, R, nregen, c0_mode):
    """ks_dot through a key table: `a` regenerated below nregen, resident above; automorphism, c0 modes, accumulate."""
    rng = np.random.default_rng(150 + 10 * K + R)
    nq, ndig = 8, 3
    digit_of = np.array([t // 3 for t in range(nq)] + [-1] * (env.R - nq), np.int32)
    rows = list(range(8)) + [8, 9, 10, 11]
    seeds = [rng.integers(0, 1 << 32, 8, dtype=np.uint64).astype(np.uint32) for _ in range(R)]
    c1, c0 = env.cts(rng, K)[:, 1], env.cts(rng, K)[:, 0]
    mu = env.rows(rng, range(env.R), lead=(K, ndig))
    bs = [env.rows(rng, range(env.R), lead=(ndig,)) for _ in range(R)]
    kas = [env.rows(rng, range(env.R), lead=(ndig,)) for _ in range(R)]
    gal = [int(fhe.rotation_galois(int(s), LOGN)) for s in rng.integers(1, 1000, R)]
    o0, o1 = env.rows(rng, range(env.R), lead=(K, R)), env.rows(rng, range(env.R), lead=(K, R))
    pm = np.array([rng.integers(1, p) for p in env.primes], np.uint64)
    pms = np.array([shoup(v, p) for v, p in zip(pm, env.primes)], np.uint64)

    def mk():
        keep = [dev(c1), dev(c0), dev(mu), dev(pm), dev(pms), torch.tensor(rows, dtype=torch.int32, device="cuda"),
                torch.tensor(digit_of, dtype=torch.int32, device="cuda"), torch.tensor(gal, dtype=torch.int32,
                                                                                      device="cuda")]
        c1d, c0d, mud, pmd, pmsd, rd, dd, gd = keep
        bds, kads = [dev(x) for x in bs], [dev(x) for x in kas]
        sds = [torch.from_numpy(x.view(np.int32).copy()).cuda() for x in seeds]
        kbt = dev(np.array([x.data_ptr() for x in bds], np.uint64))
        kat = dev(np.array([x.data_ptr() for x in kads], np.uint64))
        st = dev(np.array([x.data_ptr() for x in sds], np.uint64))
        keep += bds + kads + sds + [kbt, kat, st]
        out0, out1 = dev(o0), dev(o1)
        a = L.KsKeyArgs()
        k = a.ks
        k.c1, k.modup, k.c0, k.pr, k.rows, k.digit_of = c1d.data_ptr(), mud.data_ptr(), c0d.data_ptr(), \
            env.pc.data_ptr(), rd.data_ptr(), dd.data_ptr()
        k.ka, k.autok, k.pmod, k.pmods = kat.data_ptr(), gd.data_ptr(), pmd.data_ptr(), pmsd.data_ptr()
        k.out0, k.out1 = out0.data_ptr(), out1.data_ptr()
        k.ct_stride, k.mu_ct_stride, k.mu_digit_stride = env.R * N, ndig * env.R * N, env.R * N
        k.out_ct_stride, k.out_rot_stride, k.key_digit_stride = R * env.R * N, env.R * N, env.R * N
        k.K, k.R, k.ndig, k.c0_mode, k.nq, k.nrows = K, R, ndig, c0_mode, nq, len(rows)
        a.key.kb, a.key.seed, a.key.row_words, a.key.q_top, a.key.srows, a.key.nregen = kbt.data_ptr(), \
            st.data_ptr(), N, -1, env.R, nregen
        return a, [out0, out1], keep

    same(run_both("ks_dot_key", mk))


# ------------------------------------------------------------------------------------------------ fused CtS stage


def _brev(x, bits):
    return int(format(x, f"0{bits}b")[::-1], 2)


def _auto_slot(k, o, logn):
    j = _brev(o, logn)
    return _brev((((2 * j + 1) * k) % (2 << logn)) >> 1, logn)


def _cts_case(env, rng, K, B, G, npts, ptw, enc, x0, ndig=3, nq=8):
    digit_of = np.array([t // 3 for t in range(nq)] + [-1] * (env.R - nq), np.int32)
    rows = [5, 0, 1, 2, 3, 4, 6, 7, 11, 8, 9, 10]  # every prime id, out of order
    nb = max(B - 1, 0)
    case = dict(K=K, B=B, G=G, npts=npts, ptw=ptw, enc=enc, ndig=ndig, nq=nq, digit_of=digit_of, rows=rows)
    case["x"] = env.cts(rng, K)
    case["x0"] = env.cts(rng, K) if x0 else None
    case["mu"] = env.rows(rng, range(env.R), lead=(K, ndig))
    case["kb"] = [env.rows(rng, range(env.R), lead=(ndig,)) for _ in range(nb)]
    case["ka"] = [env.rows(rng, range(env.R), lead=(ndig,)) for _ in range(nb)]
    case["kinv"] = [int(fhe.rotation_galois(int(v), LOGN)) for v in rng.integers(1, 5000, nb)]
    pts = []
    for _ in range(npts):  # Q rows at their prime id, special rows at pt_prow = nq: R rows of ptw words
        pt = np.empty((env.R, ptw), np.uint64)
        for t in range(env.R):
            pt[t] = rng.integers(0, env.primes[t], ptw, dtype=np.uint64)
        pts.append(pt)
    case["pts"] = pts
    case["pm"] = np.array([rng.integers(1, p) for p in env.primes], np.uint64)
    case["pms"] = np.array([shoup(v, p) for v, p in zip(case["pm"], env.primes)], np.uint64)
    case["seeds"] = [rng.integers(0, 1 << 32, 8, dtype=np.uint64).astype(np.uint32) for _ in range(nb)]
    return case


def _cts_args(env, cs, keep, regen=False, nregen=0, ka_rows=None):
    K, B, G = cs["K"], cs["B"], cs["G"]
    xd, mud = dev(cs["x"]), dev(cs["mu"])
    res = torch.zeros((K * G, 2, env.R, N), dtype=torch.int64, device="cuda")
    kbs, kas = [dev(v) for v in cs["kb"]], [dev(v) for v in (ka_rows or cs["ka"])]
    pts = [dev(v) for v in cs["pts"]]
    sds = [torch.from_numpy(v.view(np.int32).copy()).cuda() for v in cs["seeds"]]
    tabs = [dev(np.array([v.data_ptr() for v in lst] or [0], np.uint64)) for lst in (kbs, kas, pts, sds)]
    small = [torch.tensor(v, dtype=torch.int32, device="cuda") for v in (cs["rows"], cs["digit_of"], cs["kinv"] or [1])]
    pmd, pmsd = dev(cs["pm"]), dev(cs["pms"])
    x0d = dev(cs["x0"]) if cs["x0"] is not None else None
    keep += [xd, mud, res, pmd, pmsd] + kbs + kas + pts + sds + tabs + small + ([x0d] if x0d is not None else [])
    a = L.CtsRegenArgs() if regen else L.CtsArgs()
    c = a.cts if regen else a
    c.x, c.modup, c.res = xd.data_ptr(), mud.data_ptr(), res.data_ptr()
    c.kb, c.ka, c.pts = tabs[0].data_ptr(), tabs[1].data_ptr(), tabs[2].data_ptr()
    c.kinv, c.rows, c.digit_of = small[2].data_ptr(), small[0].data_ptr(), small[1].data_ptr()
    c.pmod, c.pmods, c.pr = pmd.data_ptr(), pmsd.data_ptr(), env.pc.data_ptr()
    c.ct_stride, c.part_stride = 2 * env.R * N, env.R * N
    c.mu_ct_stride, c.mu_digit_stride, c.key_digit_stride = cs["ndig"] * env.R * N, env.R * N, env.R * N
    c.K, c.B, c.G, c.npts, c.ndig, c.nq, c.nlive = K, B, G, cs["npts"], cs["ndig"], cs["nq"], cs["ndig"]
    # the reference runs the x0 form one ciphertext per group at 64-bit words (kmax 1); the grouping is its own choice
    c.ptw, c.pt_prow, c.enc, c.nrows = cs["ptw"], cs["nq"], cs["enc"], len(cs["rows"])
    c.kmax = 1 if cs["x0"] is not None else 4
    c.x0 = x0d.data_ptr() if x0d is not None else None
    if regen:
        a.key.kb, a.key.seed, a.key.row_words = tabs[0].data_ptr(), tabs[3].data_ptr(), N
        a.key.q_top, a.key.srows, a.key.nregen = -1, env.R, nregen
    return a, res


def _pt_word(cs, o):
    enc = cs["enc"]
    return o if enc == 0xFFFFFFFF else (o >> (enc & 0xFF) if (enc >> 24) == 0x7F else o & enc)


def _cts_formula(env, cs, res, slots):
    """res_j[o] = sum_i rot_i[o] pts[B j + i][o] from the definition, on a few slots of every row"""
    P = env.primes
    for t in range(env.R):
        p, isq, dt = P[t], t < cs["nq"], int(cs["digit_of"][t])
        prow = t  # pt_prow = nq: special ids follow the Q ids
        for c in range(cs["K"]):
            x = cs["x"][c]
            for o in slots:
                rot = []
                for i in range(cs["B"]):
                    if i == 0:
                        if cs["x0"] is not None:
                            rot.append((int(cs["x0"][c, 0, t, o]), int(cs["x0"][c, 1, t, o])))
                        else:
                            pm = int(cs["pm"][t])
                            rot.append((int(x[0, t, o]) * pm % p, int(x[1, t, o]) * pm % p) if isq else (0, 0))
                        continue
                    s = _auto_slot(cs["kinv"][i - 1], o, LOGN)
                    D = [int(x[1, t, s]) if d == dt else int(cs["mu"][c, d, t, s]) for d in range(cs["ndig"])]
                    r0 = sum(D[d] * int(cs["kb"][i - 1][d, t, s]) for d in range(cs["ndig"]))
                    r1 = sum(D[d] * int(cs["ka"][i - 1][d, t, s]) for d in range(cs["ndig"]))
                    if isq:
                        r0 += int(x[0, t, s]) * int(cs["pm"][t])
                    rot.append((r0 % p, r1 % p))
                for j in range(cs["G"]):
                    w = [int(cs["pts"][cs["B"] * j + i][prow, _pt_word(cs, o)]) if cs["B"] * j + i < cs["npts"] else 0
                         for i in range(cs["B"])]
                    want = (sum(r[0] * wi for r, wi in zip(rot, w)) % p, sum(r[1] * wi for r, wi in zip(rot, w)) % p)
                    got = (int(res[c * cs["G"] + j, 0, t, o]), int(res[c * cs["G"] + j, 1, t, o]))
                    assert got == want, (t, c, o, j)


@pytest.mark.parametrize("K,B,G,npts,compact,x0", [(1, 4, 1, 4, False, False), (5, 5, 2, 9, False, False),
                                                     (3, 9, 2, 18, True, False), (2, 3, 2, 6, False, True),
                                                     (4, 1, 2, 2, False, False)])
def test_cts_fused(env, K, B, G, npts, compact, x0):
    """cts_fused: one BSGS stage of CoeffToSlot with the baby rotations formed in the extended basis at the slot they
    are used, over every row of both widths; diagonals past npts skipped; compact plaintexts; the x0 form; more than
    8 baby steps (the sums' periodic reduction). Word for word with the reference's launcher, and the definition on
    sampled slots."""
    rng = np.random.default_rng(300 + 7 * K + B)
    ptw, enc = (N // 4, 0x7F000002) if compact else (N, 0xFFFFFFFF)
    cs = _cts_case(env, rng, K, B, G, npts, ptw, enc, x0)

    def mk():
        keep = []
        a, res = _cts_args(env, cs, keep)
        return a, [res], keep

    got = run_both("cts_fused", mk)
    same(got)
    res = got["ours"][0].reshape(K * G, 2, env.R, N)
    _cts_formula(env, cs, res, [0, 1, 37, N // 2 + 5, N - 1])


@pytest.mark.parametrize("K,B,G,nregen", [(1, 4, 1, 3), (5, 6, 2, 2), (2, 3, 2, 0)])
def test_cts_fused_regen(env, K, B, G, nregen):
    """cts_fused_regen: the baby keys through a key table, `a` regenerated below nregen. Word for word with the
    reference's launcher, and equal to cts_fused given the expanded `a` rows (ksk_expand of the same seeds)."""
    rng = np.random.default_rng(330 + K + B)
    cs = _cts_case(env, rng, K, B, G, 2 * B - 1, N, 0xFFFFFFFF, False)

    def mk():
        keep = []
        a, res = _cts_args(env, cs, keep, regen=True, nregen=nregen)
        return a, [res], keep

    got = run_both("cts_fused_regen", mk)
    same(got)
    # the dense form with `a` expanded: digits below nregen from the seeds, the others as stored
    t = L.kernel_table()
    ka_rows = []
    for i, sd in enumerate(cs["seeds"]):
        out = torch.zeros((cs["ndig"], env.R, N), dtype=torch.int64, device="cuda")
        sdd = torch.from_numpy(sd.view(np.int32).copy()).cuda()
        ids = torch.arange(env.R, dtype=torch.int32, device="cuda")
        e = L.KskExpandArgs(out.data_ptr(), sdd.data_ptr(), ids.data_ptr(), env.pc.data_ptr(), env.R, cs["ndig"], 0, 0)
        assert t.ksk_expand(ptr(e), stream()) == 0
        torch.cuda.synchronize()
        a = host(out).reshape(cs["ndig"], env.R, N).copy()
        a[nregen:] = cs["ka"][i][nregen:]
        ka_rows.append(a)
    keep = []
    cs_dense = dict(cs, ka=ka_rows)
    a, res = _cts_args(env, cs_dense, keep)
    assert t.cts_fused(ptr(a), stream()) == 0
    torch.cuda.synchronize()
    assert (host(res) == got["ours"][0]).all()


# ------------------------------------------------------------------------------------------------ streamed weights


@pytest.mark.parametrize("n,nl,acc", [(1, 3, 0), (11, 12, 1), (32, 5, 0)])
def test_coeff_sum(env, n, nl, acc):
    """coeff_sum: float32 coefficient rows expanded (scale, round half to even, clamped and counted past the int64
    range, NaN included), transformed, and summed against n ciphertexts over nl limbs of both widths; word for word
    with the reference's launcher (output and overflow count), and this build's scratch equal to ntt_fwd of the
    expected residues."""
    rng = np.random.default_rng(500 + n)
    scale = 2.0 ** 40
    rows = rng.standard_normal((n, N)).astype(np.float32)
    rows[0, :6] = [0.5 / scale, 1.5 / scale, -2.5 / scale, 1e30, -np.inf, np.nan]  # ties to even; clamps
    cts = env.cts(rng, n)
    o = env.cts(rng, 1)[0]

    def mk():
        rd = torch.from_numpy(rows.copy()).cuda()
        cd = dev(cts)
        out = dev(o)
        scratch = torch.zeros((n, nl, N), dtype=torch.int64, device="cuda")
        ovf = torch.zeros(1, dtype=torch.int64, device="cuda")
        a = L.CoeffArgs()
        a.scratch, a.out, a.fw, a.fws, a.pr = scratch.data_ptr(), out.data_ptr(), env.fw.data_ptr(), \
            env.fws.data_ptr(), env.pc.data_ptr()
        a.overflow, a.part_stride, a.scale, a.n, a.L, a.accumulate = ovf.data_ptr(), env.R * N, scale, n, nl, acc
        for r in range(n):
            a.rows[r] = rd.data_ptr() + r * N * 4
            a.ct[r] = cd.data_ptr() + r * 2 * env.R * N * 8
        return a, [out, ovf, scratch], [rd, cd]

    got = run_both("coeff_sum", mk)
    same({k: v[:2] for k, v in got.items()})
    assert int(got["ours"][1][0]) == 3 * nl  # 1e30, -inf and NaN, once per limb
    # the expansion, transformed by ntt_fwd, equals this build's scratch
    x = rows.astype(np.float64) * scale
    big = ~(np.abs(x) < 9.2e18)
    m = np.where(big, np.where(x < 0, -(2.0 ** 62), 2.0 ** 62), np.rint(np.where(big, 0, x))).astype(np.int64)
    want = np.empty((n, nl, N), np.uint64)
    for l in range(nl):
        want[:, l] = np.mod(m, np.int64(env.primes[l])).astype(np.uint64)
    wd = dev(want.reshape(n * nl, N))
    keep = []
    na = env.ntt_args(wd, list(range(n * nl)), [i % nl for i in range(n * nl)], keep)
    assert L_tab().ntt_fwd(ptr(na), stream()) == 0
    torch.cuda.synchronize()
    assert (host(wd).reshape(n, nl, N) == got["ours"][2].reshape(n, nl, N)).all()
    # and the sum on a few words of every limb
    pt = host(wd).reshape(n, nl, N)
    out = got["ours"][0].reshape(2, env.R, N)
    for part in range(2):
        for l in range(nl):
            sl = slice(0, 32)
            v = sum(cts[r, part, l, sl].astype(object) * pt[r, l, sl].astype(object) for r in range(n))
            if acc:
                v = v + o[part, l, sl].astype(object)
            assert (out[part, l, sl].astype(object) == v % env.primes[l]).all()
    assert (out[:, nl:] == o[:, nl:]).all()


def L_tab():
    return L.kernel_table()


# ------------------------------------------------------------------------------------------------ subring switch


@pytest.mark.parametrize("sub,nq,K", [(2, 8, 1), (4, 5, 3), (16, 12, 2)])
def test_pack_split_dot(env, sub, nq, K):
    """pack_split (digit j = the coefficients at exponents j mod sub) and pack_dot (the digits against a key, + P c0 on
    the Q rows) over Q rows then special rows; the key rows by row index, c0 and the outputs by prime id."""
    rng = np.random.default_rng(400 + sub)
    nrows = env.R
    rows = list(range(nq)) + list(range(nq, env.R))[::-1]  # the special rows in reverse prime-id order
    q = env.rows(rng, rows[:nq], lead=(K,)) if nq else np.zeros((K, 0, N), np.uint64)
    pv = env.rows(rng, rows[nq:], lead=(K,))
    sp = np.zeros((K, sub, nrows, N), np.uint64)

    def mk_split():
        qd, pd = dev(q if nq else np.zeros((K, 1, N), np.uint64)), dev(pv)
        out = dev(sp)
        a = L.PackSplitArgs(qd.data_ptr(), pd.data_ptr(), out.data_ptr(), nq * N if nq else N, (nrows - nq) * N,
                            sub * nrows * N, K, sub, nq, nrows)
        return a, [out], [qd, pd]

    got = run_both("pack_split", mk_split)
    same(got)
    dig = got["ours"][0].reshape(K, sub, nrows, N)
    src = np.concatenate([q, pv], axis=1)
    cls = np.arange(N) % sub
    for j in range(sub):
        assert (dig[:, j] == np.where(cls == j, src, 0)).all()
    kb = np.stack([env.rows(rng, rows) for _ in range(sub)])  # [digit][row y][N], row y mod prime rows[y]
    ka = np.stack([env.rows(rng, rows) for _ in range(sub)])
    # the digits reduced per target row: D_j on row y mod prime rows[y] (pack_split leaves the residues as read)
    c0 = env.cts(rng, K)[:, 0]
    pm = np.array([rng.integers(1, p) for p in env.primes], np.uint64)
    pms = np.array([shoup(v, p) for v, p in zip(pm, env.primes)], np.uint64)
    o0, o1 = env.cts(rng, K)[:, 0], env.cts(rng, K)[:, 1]

    def mk_dot():
        keep = [dev(dig), dev(kb), dev(ka), dev(c0), dev(pm), dev(pms),
                torch.tensor(rows, dtype=torch.int32, device="cuda")]
        out0, out1 = dev(o0), dev(o1)
        a = L.PackDotArgs(keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), keep[3].data_ptr(),
                          out0.data_ptr(), out1.data_ptr(), keep[6].data_ptr(), keep[4].data_ptr(), keep[5].data_ptr(),
                          env.pc.data_ptr(), sub * nrows * N, env.R * N, env.R * N, K, sub, nq, nrows)
        return a, [out0, out1], keep

    got = run_both("pack_dot", mk_dot)
    same(got)
    out0 = got["ours"][0].reshape(K, env.R, N)
    for y in (0, nq - 1, nq, nrows - 1):
        if y < 0 or y >= nrows:
            continue
        t, p = rows[y], env.primes[rows[y]]
        for c in range(K):
            sl = slice(0, 64)
            want = sum(dig[c, j, y, sl].astype(object) * kb[j, y, sl].astype(object) for j in range(sub))
            if y < nq:
                want = want + c0[c, t, sl].astype(object) * int(pm[t])
            assert (out0[c, t, sl].astype(object) == want % p).all(), (y, c)


# ------------------------------------------------------------------------------------------------ element-wise


def _ew_cases(e, tabs, seed):
    rng = np.random.default_rng(seed)
    K = 2
    a, b = e.cts(rng, K), e.cts(rng, K)
    sc = np.array([rng.integers(1, p) for p in e.primes], np.uint64)
    scs = np.array([shoup(v, p) for v, p in zip(sc, e.primes)], np.uint64)
    rs = L.RowSet(5, 3, e.R - 4, 0)  # Q rows 0..4, special rows R-4 .. R-2

    for entry, sub, zero_p, nparts in [("ew_add", 0, 0, 2), ("ew_add", 1, 0, 1), ("ew_scale", 0, 1, 2),
                                       ("ew_scale", 0, 0, 2), ("ew_sub_mul", 0, 0, 2), ("ew_copy", 0, 0, 2)]:
        def mk():
            keep = [dev(a), dev(b), dev(sc), dev(scs)]
            ad, bd, scd, scsd = keep
            out = dev(np.full_like(a, 7))
            x = L.EwArgs(e.cref(out), e.cref(ad), e.cref(bd), rs, scd.data_ptr(), scsd.data_ptr(), e.pc.data_ptr(),
                         K, nparts, sub, zero_p)
            return x, [out], keep

        got = run_both(entry, mk, tabs)
        same(got)


def test_elementwise(env):
    _ew_cases(env, tables(), seed=40)


@pytest.mark.parametrize("npairs,acc,dbl,acc_d2,coef", [(1, 0, 0, 0, 0), (2, 1, 1, 1, 1)])
def test_tensor(env, npairs, acc, dbl, acc_d2, coef):
    rng = np.random.default_rng(50 + npairs)
    K, n = 3, 10
    ins = [env.cts(rng, K) for _ in range(4)]
    o, d2, cf = env.cts(rng, K), env.cts(rng, K), env.rows(rng, range(env.R), lead=(K,))

    def mk():
        keep = [dev(v) for v in ins]
        out, d2d, cfd = dev(o), dev(d2), dev(cf)
        x = L.TensorArgs(env.cref(out), env.cref(d2d), env.cref(keep[0]), env.cref(keep[1]), env.cref(keep[2]),
                         env.cref(keep[3]), cfd.data_ptr() if coef else None, env.R * N, env.pc.data_ptr(), npairs, acc,
                         n, K, dbl, acc_d2)
        return x, [out, d2d, cfd], keep

    same(run_both("tensor", mk))


@pytest.mark.parametrize("sub,dbl", [(0, 0), (1, 1)])
def test_tensor_y(env, sub, dbl):
    """tensor_y: the tensor, then (c0, c1) +/-= c[row] y after the doubling (EvalMod's x y +/- c t)"""
    rng = np.random.default_rng(56 + sub)
    K, n = 2, 10
    ins = [env.cts(rng, K) for _ in range(5)]
    o, d2 = env.cts(rng, K), env.cts(rng, K)
    c = np.array([int(rng.integers(0, p)) for p in env.primes], np.uint64)
    cs = np.array([shoup(int(v), p) for v, p in zip(c, env.primes)], np.uint64)

    def mk():
        keep = [dev(v) for v in ins] + [dev(c), dev(cs)]
        out, d2d = dev(o), dev(d2)
        t = L.TensorArgs(env.cref(out), env.cref(d2d), env.cref(keep[0]), env.cref(keep[1]), env.cref(keep[2]),
                         env.cref(keep[3]), None, 0, env.pc.data_ptr(), 2, 1, n, K, dbl, 0)
        x = L.TensorYArgs(t, env.cref(keep[4]), keep[5].data_ptr(), keep[6].data_ptr(), sub, 0)
        return x, [out, d2d], keep

    got = run_both("tensor_y", mk)
    same(got)
    # the formula on the rows of both widths
    P = np.array(env.primes, dtype=object)[None, :, None]
    a0, b0, a1, b1, y = (v.astype(object) for v in ins)  # pair 0 (a0, b0), pair 1 (a1, b1), as the args
    r0 = (a0[:, 0] * b0[:, 0] + a1[:, 0] * b1[:, 0] + o[:, 0].astype(object)) % P
    r0 = r0 * (1 + dbl) % P
    cy = c.astype(object)[None, :, None] * y[:, 0] % P
    r0 = (r0 - cy if sub else r0 + cy) % P
    out = got["ours"][0].reshape(o.shape)
    assert (out[:, 0, :n] == r0[:, :n].astype(np.uint64)).all()
    assert (out[:, :, n:] == o[:, :, n:]).all()


@pytest.mark.parametrize("mc,sh,nrows,nparts", [(None, 60, 12, 2), (None, 64, 9, 1), (1 << 52, 100, 12, 2),
                                                  (3, 1, 12, 2), (None, 127, 5, 2), (None, 65, 12, 2)])
def test_small_int1(env, mc, sh, nrows, nparts):
    """small_int1: row 0 centred, times mc 2^-sh rounded half up, onto rows [0, nrows) of both widths (in place);
    a 53-bit mc is a double's mantissa, the raise's exact scale"""
    rng = np.random.default_rng(97 + sh)
    K = 3
    x0 = env.cts(rng, K)
    q = env.primes
    x0[:, :, 0, :4] = np.array([0, q[0] // 2, q[0] // 2 + 1, q[0] - 1], np.uint64)  # the centring edges
    mcv = int(rng.integers(1 << 52, 1 << 53)) if mc is None else mc
    a = L.SmallInt1Args()

    def mk():
        xd = dev(x0)
        a.x, a.pr = xd.data_ptr(), env.pc.data_ptr()
        a.ct_stride, a.part_stride = 2 * env.R * env.n, env.R * env.n
        a.mc, a.sh, a.nrows, a.K, a.nparts = mcv, sh, nrows, K, nparts
        return a, [xd], []

    got = run_both("small_int1", mk)
    same(got)
    out = got["ours"][0].reshape(x0.shape)
    for c in range(K):
        for part in range(nparts):
            v = x0[c, part, 0, :256].astype(object)
            xc = [int(w) - q[0] if int(w) > q[0] // 2 else int(w) for w in v]
            m = [(abs(w) * mcv + (1 << (sh - 1))) >> sh for w in xc]
            for t in range(nrows):
                want = [(-mm if w < 0 else mm) % q[t] for w, mm in zip(xc, m)]
                assert [int(u) for u in out[c, part, t, :256]] == want, (c, part, t)
    assert (out[:, :, nrows:] == x0[:, :, nrows:]).all()
    assert (out[:, nparts:] == x0[:, nparts:]).all()


@pytest.mark.parametrize("dbl,with_k", [(0, False), (1, True)])
def test_md_epilogue(env, dbl, with_k):
    rng = np.random.default_rng(60 + dbl)
    K, n = 2, 9
    dst, x, t = env.cts(rng, K), env.cts(rng, K), env.cts(rng, K)
    bi = np.array([rng.integers(1, p) for p in env.primes], np.uint64)
    bis = np.array([shoup(v, p) for v, p in zip(bi, env.primes)], np.uint64)
    k = np.array([rng.integers(0, p + 1) for p in env.primes], np.uint64)  # k == p allowed

    def mk():
        keep = [dev(x), dev(t), dev(bi), dev(bis), dev(k)]
        dd = dev(dst)
        a = L.MdEpiArgs(env.cref(dd), env.cref(keep[0]), env.cref(keep[1]), keep[2].data_ptr(), keep[3].data_ptr(),
                        keep[4].data_ptr() if with_k else None, env.pc.data_ptr(), dbl, n, K, 0)
        return a, [dd], keep

    same(run_both("md_epilogue", mk))


@pytest.mark.parametrize("has_add", [0, 1])
def test_automorph(env, has_add):
    rng = np.random.default_rng(70 + has_add)
    K = 2
    x, ad = env.cts(rng, K), env.cts(rng, K)
    k = int(fhe.rotation_galois(37, LOGN))

    def mk():
        keep = [dev(x), dev(ad)]
        out = dev(np.zeros_like(x))
        a = L.AutomorphArgs(env.cref(out), env.cref(keep[0]), env.cref(keep[1]), L.RowSet(6, 2, 9, 0), env.pc.data_ptr(),
                            k, K, 2, has_add)
        return a, [out], keep

    same(run_both("automorph", mk))


@pytest.mark.parametrize("ndrop", [1, 2])
def test_rescale_launchers(env, ndrop):
    """rescale_coef (one and two dropped primes, constant pre-factors ca/cb) and rescale_combine."""
    rng = np.random.default_rng(80 + ndrop)
    K, top = 2, 7
    x = env.cts(rng, K)
    q = env.primes
    a_, b_ = top, top - 1
    nrows = top + 1 - ndrop

    def qlql(xp, i):
        return (-pow(q[xp], -1, q[i])) % q[i]

    A = [((pow(q[b_], -1, q[i]) * qlql(a_, i)) % q[i] if ndrop == 2 else qlql(a_, i)) for i in range(env.R)
         if i < nrows] + [0] * (env.R - nrows)
    B = [qlql(b_, i) if (ndrop == 2 and i < nrows) else 0 for i in range(env.R)]
    al = [((pow(q[a_], -1, q[i]) * (pow(q[b_], -1, q[i]) if ndrop == 2 else 1)) % q[i]) if i < nrows else 1
          for i in range(env.R)]
    As, Bs, als = ([shoup(v, q[i]) for i, v in enumerate(arr)] for arr in (A, B, al))
    qam = [q[a_] % q[i] for i in range(env.R)]
    qbm = [q[b_] % q[i] for i in range(env.R)]
    qinv_ab = pow(q[a_], -1, q[b_])
    C_ab = qlql(a_, b_)
    ca, cb = int(rng.integers(2, q[a_])), int(rng.integers(2, q[b_]))
    tmp0 = env.cts(rng, K)

    def mk_coef():
        keep = [dev(x)] + [dev(v) for v in (A, B, As, Bs, qam, qbm)]
        tmp = dev(tmp0)
        r = L.RescaleArgs(env.cref(keep[0]), env.cref(tmp), *[v.data_ptr() for v in keep[1:]], env.pc.data_ptr(),
                          qinv_ab, C_ab, ca, cb, top, nrows, K, ndrop)
        return r, [tmp], keep

    got = run_both("rescale_coef", mk_coef)
    same(got)
    tmp_h = got["ref"][0]

    def mk_comb():
        keep = [dev(tmp_h), dev(al), dev(als)]
        xd = dev(x)
        r = L.RescaleCombineArgs(env.cref(xd), env.cref(keep[0]), keep[1].data_ptr(), keep[2].data_ptr(),
                                 env.pc.data_ptr(), nrows, K)
        return r, [xd], keep

    same(run_both("rescale_combine", mk_comb))


@pytest.mark.parametrize("d,r0,r1,nparts", [(1, 1, 12, 2), (2, 2, 9, 1), (3, 5, 12, 2), (4, 4, 12, 2)])
def test_mod_raise(env, d, r0, r1, nparts):
    """mod_raise: composite raise from the d bottom rows (random Garner constants), onto rows [r0, r1) of both widths;
    d = 1 with unit constants is bootstrapping's level-0 raise."""
    rng = np.random.default_rng(95 + d)
    K = 3
    x0 = env.cts(rng, K)
    q = env.primes
    a = L.ModRaiseArgs()
    for k in range(d):
        a.qhatinv[k] = 1 if d == 1 else int(rng.integers(1, q[k]))
        for t in range(env.R):
            a.qhat[k][t] = 1 if d == 1 else int(rng.integers(0, q[t]))

    def mk():
        xd = dev(x0)
        a.x, a.pr = xd.data_ptr(), env.pc.data_ptr()
        a.ct_stride, a.part_stride = 2 * env.R * env.n, env.R * env.n
        a.K, a.d, a.r0, a.r1, a.nparts = K, d, r0, r1, nparts
        return a, [xd], []

    got = run_both("mod_raise", mk)
    same(got)
    if d == 1:  # every raised row holds the centred lift of row 0
        x, out = x0[:, :nparts, 0].astype(object), got["ours"][0].reshape(x0.shape)
        c = np.where(x > q[0] // 2, x - q[0], x)
        for t in range(r0, r1):
            assert (out[:, :nparts, t] == (c % q[t]).astype(np.uint64)).all()
        assert (out[:, nparts:] == x0[:, nparts:]).all()


@pytest.mark.parametrize("bits", [1, 20, 28, 32])
def test_ksk_unpack(env, bits):
    """ksk_unpack: packed rows (random words, the guard word included) to dense u64 rows, at the widths the
    reference's u64 table takes."""
    rng = np.random.default_rng(97 + bits)
    nrows = 3
    rw = ((env.n * bits // 32 + 1) + 3) // 4 * 4
    packed = rng.integers(0, 2**32, (nrows, rw), dtype=np.uint64).astype(np.uint32)

    def mk():
        inp = torch.from_numpy(packed.view(np.int32).copy()).cuda()
        out = torch.zeros((nrows, env.n), dtype=torch.int64, device="cuda")
        a = L.KskUnpackArgs(out.data_ptr(), inp.data_ptr(), rw, nrows, bits)
        return a, [out], [inp]

    same(run_both("ksk_unpack", mk))


# ------------------------------------------------------------------------------------------------ plaintext operands


def test_plaintext_operand_entries(env):
    rng = np.random.default_rng(90)
    K, n = 3, 11
    x, y = env.cts(rng, K), env.cts(rng, K)
    xs = [env.cts(rng, K) for _ in range(8)]
    ts = [env.rows(rng, range(env.R)) for _ in range(8)]
    kc = np.array([rng.integers(0, p + 1) for p in env.primes], np.uint64)

    def mk_const():
        kd = dev(kc)
        xd = dev(x)
        return L.AddConstArgs(env.cref(xd), kd.data_ptr(), env.pc.data_ptr(), n, K), [xd], [kd]

    same(run_both("add_const", mk_const))

    def mk_table():
        xd, td = dev(x), dev(ts[0])
        out = dev(y)
        return L.MulTableArgs(env.cref(out), env.cref(xd), td.data_ptr(), env.pc.data_ptr(), n, K), [out], [xd, td]

    same(run_both("mul_table", mk_table))
    for sub in (0, 1, 2):
        def mk_add():
            xd, td, yd = dev(x), dev(ts[1]), dev(y)
            m = L.MulTableArgs(env.cref(yd), env.cref(xd), td.data_ptr(), env.pc.data_ptr(), n, K)
            return L.MulAddArgs(m, env.cref(yd), sub, 0), [yd], [xd, td]

        same(run_both("mul_add", mk_add))
    for nterm, lazy, with_y in [(1, 0, True), (5, 1, False), (8, 0, True), (8, 1, True)]:
        def mk_n():
            keep = [dev(v) for v in xs[:nterm]] + [dev(v) for v in ts[:nterm]]
            yd = dev(y)
            out = dev(np.zeros_like(y))
            a = L.MulAddNArgs()
            a.out, a.y = env.cref(out), (env.cref(yd) if with_y else L.PolyRef())
            for j in range(nterm):
                a.x[j], a.t[j] = env.cref(keep[j]), keep[nterm + j].data_ptr()
            a.pr, a.n, a.K, a.nterm, a.lazy = env.pc.data_ptr(), n, K, nterm, lazy
            return a, [out], keep + [yd]

        same(run_both("mul_add_n", mk_n))


@pytest.mark.parametrize("K,enc,ptw", [(3, 0xFFFFFFFF, N), (5, 0x7F000001, N // 2), (1, N // 4 - 1, N // 4)])
def test_pt_dot(env, K, enc, ptw):
    rng = np.random.default_rng(100 + K)
    bstep, gstep, npts = 3, 2, 5
    nq, np_, qmax, pt_prow = 5, 2, 9, 5
    rot = env.cts(rng, K * bstep)
    pts = [rng.integers(0, 1 << 49, (pt_prow + np_, ptw), dtype=np.uint64) for _ in range(npts)]

    def mk():
        rd = dev(rot)
        pd = [dev(v) for v in pts]
        tab = dev(np.array([t.data_ptr() for t in pd], np.uint64))
        res = torch.zeros((K * gstep, 2, env.R, N), dtype=torch.int64, device="cuda")
        a = L.PtDotArgs()
        a.rot = L.PolyRef(rd.data_ptr(), bstep * 2 * env.R * N, env.R * N)
        a.res = L.PolyRef(res.data_ptr(), gstep * 2 * env.R * N, env.R * N)
        a.rot_stride, a.res_stride = 2 * env.R * N, 2 * env.R * N
        a.pts, a.pr, a.rs = tab.data_ptr(), env.pc.data_ptr(), L.RowSet(nq, np_, qmax, 0)
        a.npts, a.bstep, a.gstep, a.K, a.ptw, a.pt_prow, a.enc = npts, bstep, gstep, K, ptw, pt_prow, enc
        return a, [res], [rd, tab] + pd

    same(run_both("pt_dot", mk))


# ------------------------------------------------------------------------------------------------ keys, encryption


def test_key_entries(env):
    rng = np.random.default_rng(110)
    seed = rng.integers(0, 1 << 32, 8, dtype=np.uint64).astype(np.uint32)
    ids = np.array([0, 2, 5, 8, 11], np.int32)
    dnum = 3

    def mk_expand():
        sd = torch.from_numpy(seed.view(np.int32).copy()).cuda()
        idd = torch.tensor(ids, dtype=torch.int32, device="cuda")
        out = torch.zeros((dnum - 1, len(ids), N), dtype=torch.int64, device="cuda")
        return L.KskExpandArgs(out.data_ptr(), sd.data_ptr(), idd.data_ptr(), env.pc.data_ptr(), len(ids), dnum, 1,
                               0), [out], [sd, idd]

    same(run_both("ksk_expand", mk_expand))

    nq, ndig = 8, 3
    rows_ids = np.array(list(range(nq)) + [8, 9, 10, 11], np.int32)
    digit_of = np.array([t // 3 for t in range(nq)] + [-1] * 4, np.int32)
    e = env.rows(rng, rows_ids, lead=(ndig,))
    s_new = env.rows(rng, range(env.R))
    s_old = env.rows(rng, range(env.R))
    pm = np.array([rng.integers(1, p) for p in env.primes], np.uint64)
    pms = np.array([shoup(v, p) for v, p in zip(pm, env.primes)], np.uint64)
    for sq in (0, 1):
        def mk_gen():
            keep = [dev(e), dev(s_new), dev(s_old), dev(pm), dev(pms)]
            sd = torch.from_numpy(seed.view(np.int32).copy()).cuda()
            idd = torch.tensor(rows_ids, dtype=torch.int32, device="cuda")
            dg = torch.tensor(digit_of, dtype=torch.int32, device="cuda")
            b = torch.zeros((ndig, len(rows_ids), N), dtype=torch.int64, device="cuda")
            a = torch.zeros_like(b)
            g = L.KskGenArgs(b.data_ptr(), a.data_ptr(), *[k.data_ptr() for k in keep[:3]], sd.data_ptr(),
                             idd.data_ptr(), dg.data_ptr(), keep[3].data_ptr(), keep[4].data_ptr(), env.pc.data_ptr(),
                             N, len(rows_ids), ndig, nq, 0, sq, 0)
            return g, [b, a], keep + [sd, idd, dg]

        same(run_both("ksk_gen", mk_gen))

    s = env.rows(rng, range(env.R))
    err = env.rows(rng, range(env.R))
    m = env.rows(rng, range(env.R))
    for with_m, with_c1 in [(True, True), (False, False)]:
        def mk_enc():
            keep = [dev(s), dev(err), dev(m)]
            sd = torch.from_numpy(seed.view(np.int32).copy()).cuda()
            c0 = torch.zeros((env.R, N), dtype=torch.int64, device="cuda")
            c1 = torch.zeros_like(c0)
            a = L.EncryptArgs(c0.data_ptr(), c1.data_ptr() if with_c1 else None, keep[0].data_ptr(), keep[1].data_ptr(),
                              keep[2].data_ptr() if with_m else None, sd.data_ptr(), env.pc.data_ptr(), 77, env.R)
            return a, [c0, c1], keep + [sd]

        same(run_both("encrypt", mk_enc))


# ------------------------------------------------------------------------------------------------ compositions


class RefRuntime:
    """The reference's device runtime order (crates/pc-gpu) driven through the reference's own launchers, on the
    tables and keys of a perseus-b200 session (the same prime-id layout)."""

    def __init__(self, s, t):
        self.s, self.t = s, t
        self.n, self.rows, self.nq, self.kp = s.n, s.rows, s.nq, s.kp
        self.primes = list(s.chain.q) + list(s.chain.p)
        self.alpha = -(-self.nq // s.chain.dnum)
        self.pr, self.fw, self.fws, self.iw, self.iws, self.ninv, self.ninvs = s.tables()
        self.keep = []

    def call(self, entry, args):
        rc = getattr(self.t, entry)(ptr(args), stream())
        assert rc == 0, f"reference {entry} returned {rc}"

    def ntt(self, inverse, base, roff, rprime, **kw):
        a = L.NttArgs()
        ro = torch.tensor(roff, dtype=torch.int32, device="cuda")
        rp = torch.tensor(rprime, dtype=torch.int32, device="cuda")
        self.keep += [ro, rp]
        a.base, a.roff, a.rprime = base.data_ptr(), ro.data_ptr(), rp.data_ptr()
        a.fw, a.fws, a.iw, a.iws, a.ninv, a.ninvs, a.pr = self.fw, self.fws, self.iw, self.iws, self.ninv, \
            self.ninvs, self.pr
        a.nrows, a.snum, a.xnum = len(roff), 1, 1
        for k, v in kw.items():
            setattr(a, k, v)
        self.call("ntt_inv" if inverse else "ntt_fwd", a)

    def bconv(self, src, dst, jobs_spec):
        """jobs_spec: [(src row list, src prime ids, tgt row list, tgt prime ids, src_off, dst_off, pre or None)]"""
        pool, jobs = [], []
        for srows, sp, trows, tp, soff, doff, prescaled in jobs_spec:
            B = 1
            for i in sp:
                B *= self.primes[i]
            pre = [pow(B // self.primes[i] % self.primes[i], -1, self.primes[i]) for i in sp]
            M = [(B // self.primes[i]) % self.primes[t] for i in sp for t in tp]
            off = len(pool)
            pool += list(srows) + list(sp) + pre + list(trows) + list(tp) + M
            jobs.append(L.BconvJob(soff, doff, len(sp), len(tp), off, 0, prescaled, 0))
        jarr = (L.BconvJob * len(jobs))(*jobs)
        jd = torch.from_numpy(np.frombuffer(bytes(jarr), np.uint8).copy()).cuda()
        pd = dev(np.array(pool, np.uint64))
        self.keep += [jd, pd]
        a = L.BconvArgs()
        a.src, a.dst, a.jobs, a.pool, a.pr = src.data_ptr(), dst.data_ptr(), jd.data_ptr(), pd.data_ptr(), self.pr
        a.njobs, a.max_tgt = len(jobs), max(len(j[3]) for j in jobs_spec)
        self.call("bconv", a)

    def digit_range(self, d, top):
        return d * self.alpha, min((d + 1) * self.alpha, self.nq, top + 1)

    def keyswitch_ext(self, d, c0, c0_mode, kidx, autok, top):
        """ModUp(d) then the inner product against key kidx: ext [2][rows][N] (Q rows 0..=top, special rows)."""
        n, rows, nq, kp = self.n, self.rows, self.nq, self.kp
        ndig = top // self.alpha + 1
        # 1. INTT of rows 0..=top, the digit pre factor folded into the last pass (ks.rs:954-980)
        coef = d[: top + 1].clone()
        es, ess = [], []
        for t in range(top + 1):
            lo, hi = self.digit_range(t // self.alpha, top)
            h = 1
            for k in range(lo, hi):
                if k != t:
                    h = h * self.primes[k] % self.primes[t]
            v = pow(self.n, -1, self.primes[t]) * pow(h, -1, self.primes[t]) % self.primes[t]
            es.append(v)
            ess.append(shoup(v, self.primes[t]))
        esd, essd = dev(es), dev(ess)
        self.keep += [esd, essd]
        self.ntt(True, coef, list(range(top + 1)), list(range(top + 1)), es=esd.data_ptr(), ess=essd.data_ptr())
        # 2. bconv of every live digit to its targets (prescaled sources), 3. NTT of the targets (ks.rs:1037-1043)
        D = torch.zeros((ndig, rows, n), dtype=torch.int64, device="cuda")
        spec, roff, rprime = [], [], []
        for dg in range(ndig):
            lo, hi = self.digit_range(dg, top)
            tg = [t for t in range(top + 1) if t < lo or t >= hi] + [nq + j for j in range(kp)]
            spec.append((list(range(lo, hi)), list(range(lo, hi)), tg, tg, 0, dg * rows, 1))
            roff += [dg * rows + t for t in tg]
            rprime += tg
        self.bconv(coef, D, spec)
        self.ntt(False, D, roff, rprime)
        # 4. the inner product (ks.rs:1109)
        b, a = self.s.key_tensors(kidx)
        ext = torch.zeros((2, rows, n), dtype=torch.int64, device="cuda")
        kb = dev(np.array([b.data_ptr()], np.uint64))
        ka = dev(np.array([a.data_ptr()], np.uint64))
        krows = list(range(top + 1)) + [nq + j for j in range(kp)]
        digit_of = [t // self.alpha for t in range(nq)] + [-1] * kp
        pmod = [1] * rows
        P = 1
        for j in range(kp):
            P *= self.primes[nq + j]
        pmod = [P % self.primes[t] for t in range(rows)]
        pms = [shoup(v, self.primes[t]) for t, v in enumerate(pmod)]
        aut = torch.tensor([autok], dtype=torch.int64, device="cuda").to(torch.int32)
        rd = torch.tensor(krows, dtype=torch.int32, device="cuda")
        dd = torch.tensor(digit_of, dtype=torch.int32, device="cuda")
        pmd, pmsd = dev(pmod), dev(pms)
        self.keep += [b, a, kb, ka, aut, rd, dd, pmd, pmsd]
        k = L.KsArgs()
        k.c1, k.modup, k.c0 = d.data_ptr(), D.data_ptr(), (c0.data_ptr() if c0 is not None else None)
        k.out0, k.out1 = ext[0].data_ptr(), ext[1].data_ptr()
        k.kb, k.ka, k.autok, k.rows, k.digit_of = kb.data_ptr(), ka.data_ptr(), aut.data_ptr(), rd.data_ptr(), \
            dd.data_ptr()
        k.pmod, k.pmods, k.pr = pmd.data_ptr(), pmsd.data_ptr(), self.pr
        k.ct_stride, k.mu_ct_stride, k.mu_digit_stride = rows * n, ndig * rows * n, rows * n
        k.out_ct_stride, k.out_rot_stride, k.key_digit_stride = 2 * rows * n, 0, rows * n
        k.K, k.R, k.ndig, k.c0_mode, k.nq, k.nrows = 1, 1, ndig, c0_mode, nq, len(krows)
        self.call("ks_dot", k)
        return ext

    def moddown(self, ext, top):
        """INTT of the special rows (N^-1 times the conversion's pre factor), bconv P -> Q rows 0..=top, NTT whose
        epilogue writes (x - conv) P^-1 (ks.rs:1620-1656)."""
        n, rows, nq, kp = self.n, self.rows, self.nq, self.kp
        y = ext.clone()
        sp = [nq + j for j in range(kp)]
        P = 1
        for t in sp:
            P *= self.primes[t]
        es = [pow(n, -1, self.primes[t]) * pow(P // self.primes[t] % self.primes[t], -1, self.primes[t])
              % self.primes[t] for t in sp] * 2
        ess = [shoup(v, self.primes[sp[i % kp]]) for i, v in enumerate(es)]
        esd, essd = dev(es), dev(ess)
        self.keep += [esd, essd]
        self.ntt(True, y, [part * rows + t for part in (0, 1) for t in sp], sp * 2, es=esd.data_ptr(),
                 ess=essd.data_ptr())
        conv = torch.zeros((2, rows, n), dtype=torch.int64, device="cuda")
        tq = list(range(top + 1))
        self.bconv(y, conv, [(sp, sp, tq, tq, part * rows, part * rows, 1) for part in (0, 1)])
        pinv = [pow(P, -1, self.primes[t]) if t < nq else 0 for t in range(rows)]
        pinvs = [shoup(v, self.primes[t]) for t, v in enumerate(pinv)]
        pd, psd = dev(pinv), dev(pinvs)
        out = torch.zeros((2, rows, n), dtype=torch.int64, device="cuda")
        self.keep += [pd, psd]
        self.ntt(False, conv, [part * rows + t for part in (0, 1) for t in tq], tq * 2, epi=1, eout=out.data_ptr(),
                 ex=ext.data_ptr(), es=pd.data_ptr(), ess=psd.data_ptr())
        return out

    def rotate(self, x, step, top):
        g = fhe.rotation_galois(step, self.s.log_n)
        ginv = pow(g, -1, 2 * self.n)
        ext = self.keyswitch_ext(x[1], x[0], 1, self.s.galois.index(g), ginv, top)
        return self.moddown(ext, top)

    def mult(self, a, b, top):
        rows, n = self.rows, self.n
        c01 = torch.zeros((2, rows, n), dtype=torch.int64, device="cuda")
        d2 = torch.zeros((2, rows, n), dtype=torch.int64, device="cuda")
        pref = lambda t: L.PolyRef(t.data_ptr(), 2 * rows * n, rows * n)  # noqa: E731
        ta = L.TensorArgs(pref(c01), pref(d2), pref(a), pref(b), pref(a), pref(b), None, 0, self.pr, 1, 0, top + 1,
                          1, 0, 0)
        self.call("tensor", ta)
        md = self.moddown(self.keyswitch_ext(d2[1], None, 0, 0, 1, top), top)
        out = torch.zeros((2, rows, n), dtype=torch.int64, device="cuda")
        ew = L.EwArgs(pref(out), pref(c01), pref(md), L.RowSet(top + 1, 0, self.nq, 0), None, None, self.pr, 1, 2, 0, 0)
        self.call("ew_add", ew)
        return out

    def rescale(self, x, top):
        rows, n, q = self.rows, self.n, self.primes
        y = x.clone()
        self.ntt(True, y, [top, rows + top], [top, top])  # the top row of both parts to coefficient form
        tmp = torch.zeros((2, rows, n), dtype=torch.int64, device="cuda")
        A = [(-pow(q[top], -1, q[i])) % q[i] if i < top else 0 for i in range(rows)]
        As = [shoup(v, q[i]) for i, v in enumerate(A)]
        qam = [q[top] % q[i] for i in range(rows)]
        al = [pow(q[top], -1, q[i]) if i < top else 1 for i in range(rows)]
        als = [shoup(v, q[i]) for i, v in enumerate(al)]
        Ad, Asd, qd, ald, alsd, zd = dev(A), dev(As), dev(qam), dev(al), dev(als), dev([0] * rows)
        self.keep += [Ad, Asd, qd, ald, alsd, zd]
        pref = lambda t: L.PolyRef(t.data_ptr(), 2 * rows * n, rows * n)  # noqa: E731
        r = L.RescaleArgs(pref(y), pref(tmp), Ad.data_ptr(), zd.data_ptr(), Asd.data_ptr(), zd.data_ptr(), qd.data_ptr(),
                          qd.data_ptr(), self.pr, 0, 0, 1, 1, top, top, 1, 1)
        self.call("rescale_coef", r)
        self.ntt(False, tmp, [part * rows + t for part in (0, 1) for t in range(top)], list(range(top)) * 2)
        out = x.clone()
        c = L.RescaleCombineArgs(pref(out), pref(tmp), ald.data_ptr(), alsd.data_ptr(), self.pr, top, 1)
        self.call("rescale_combine", c)
        return out


SEED, H, SIGMA = 0, 192, 3.2


@pytest.fixture(scope="module")
def cfg2():
    ch = fhe.config2_chain()
    s = fhe.Session(ch, rot_steps=(1, 5, -3), k_max=1, seed=SEED, h=H, sigma=SIGMA)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(SEED, H, SIGMA, s.galois)
    return s, o


@pytest.mark.parametrize("top,step", [(23, 1), (23, -3), (11, 5)])
def test_reference_rotation_equals_oracle(cfg2, top, step):
    s, o = cfg2
    rt = RefRuntime(s, ref_table())
    rng = np.random.default_rng(120 + top)
    x = rng.normal(0, 1, 2048) / 8
    ct = s.encrypt(x, top=top)
    oc = o.encrypt(x, ct.slots, ct.scale, top)
    assert (host(ct.data[0])[:, : top + 1] == oc[:, : top + 1]).all()
    got = host(rt.rotate(ct.data[0], step, top))
    want = o.rotate(oc, step, top)
    assert (got[:, : top + 1] == want[:, : top + 1]).all(), "reference launchers' rotation != oracle"
    ours = host(s.rotate(ct, step).data[0])
    assert (ours[:, : top + 1] == got[:, : top + 1]).all()


@pytest.mark.parametrize("top", [23, 12])
def test_reference_relin_and_rescale_equal_oracle(cfg2, top):
    s, o = cfg2
    rt = RefRuntime(s, ref_table())
    rng = np.random.default_rng(130 + top)
    x, y = rng.normal(0, 1, 1024) / 8, rng.normal(0, 1, 1024) / 8
    a, b = s.encrypt(x, top=top), s.encrypt(y, top=top)
    oa, ob = o.encrypt(x, a.slots, a.scale, top), o.encrypt(y, b.slots, b.scale, top)
    m = host(rt.mult(a.data[0], b.data[0], top))
    om = o.mult(oa, ob, top)
    assert (m[:, : top + 1] == om[:, : top + 1]).all(), "reference launchers' relinearized product != oracle"
    ours = s.mult(a, b)
    assert (host(ours.data[0])[:, : top + 1] == m[:, : top + 1]).all()
    r = host(rt.rescale(ours.data[0], top))
    orr = o.rescale(om, top)
    assert (r[:, :top] == orr[:, :top]).all(), "reference launchers' rescale != oracle"
    s.rescale_one(ours)
    assert (host(ours.data[0])[:, :top] == r[:, :top]).all()


# ------------------------------------------------------------------------------------------------ the evaluator's other entries
# (crates/pc-gpu/src: ops.rs wsum / wsum_k / tensor_sum / tensor_multi, relin.rs wsum, ks.rs ew_many / submul_many,
# rescale.rs rescale_fwd / rescale_combine_to, bts/evalmod.rs wsum_multi / md_epilogue_to)


def _poly_ptr(t, env, c, part):
    """pointer to polynomial (c, part) of a [K][2][R][N] device tensor (rows at + r N words)"""
    return t.data_ptr() + ((c * 2 + part) * env.R * env.n) * 8


def test_ew_many_and_submul_many(env):
    rng = np.random.default_rng(120)
    K, nrows = 3, 9
    srcs = [env.cts(rng, K) for _ in range(3)]
    t = env.rows(rng, range(nrows))

    def mk_many():
        a, b, c = (dev(x) for x in srcs)
        out = torch.zeros_like(a)
        args = L.EwManyArgs()
        polys = [(cc, part) for cc in range(K) for part in range(2)]
        for j, (cc, part) in enumerate(polys):
            args.out[j] = _poly_ptr(out, env, cc, part)
            args.a[j] = _poly_ptr(a, env, cc, part)
            args.b[j] = _poly_ptr(b, env, cc, part) if j % 3 != 1 else None  # null b / c skipped
            args.c[j] = _poly_ptr(c, env, cc, part) if j % 2 == 0 else None
        args.pr, args.n, args.nrows = env.pc.data_ptr(), len(polys), nrows
        return args, [out], [a, b, c]

    same(run_both("ew_many", mk_many))

    def mk_submul():
        a, b = dev(srcs[0]), dev(srcs[1])
        td = dev(t)
        out = torch.zeros_like(a)
        args = L.SubMulManyArgs()
        polys = [(cc, part) for cc in range(K) for part in range(2)]
        for j, (cc, part) in enumerate(polys):
            args.out[j] = _poly_ptr(out, env, cc, part)
            args.a[j] = _poly_ptr(a, env, cc, part)
            args.b[j] = _poly_ptr(b, env, cc, part)
        args.t, args.pr, args.n, args.nrows = td.data_ptr(), env.pc.data_ptr(), len(polys), nrows
        return args, [out], [a, b, td]

    same(run_both("submul_many", mk_submul))


@pytest.mark.parametrize("nsrc", [1, 3, 8])
def test_weighted_sums(env, nsrc):
    rng = np.random.default_rng(130 + nsrc)
    K, n = 2, env.R
    srcs = [env.cts(rng, K) for _ in range(nsrc)]
    rowstride = env.R
    w = [[int(rng.integers(0, env.primes[r])) for r in range(rowstride)] for _ in range(nsrc)]
    ws = [[shoup(v, env.primes[r]) for r, v in enumerate(row)] for row in w]
    kraw = [int(rng.integers(0, 2 * env.primes[r])) for r in range(env.R)]  # raw: reduced once when >= p

    def base_args(keep):
        sd = [dev(x) for x in srcs]
        wd, wsd = dev(np.array(w, np.uint64).ravel()), dev(np.array(ws, np.uint64).ravel())
        out = torch.zeros_like(sd[0])
        keep += sd + [wd, wsd]
        a = L.WsumArgs()
        a.out = env.cref(out)
        for j in range(nsrc):
            a.src[j] = env.cref(sd[j])
        a.w, a.ws, a.pr, a.nsrc, a.rowstride, a.n, a.K = wd.data_ptr(), wsd.data_ptr(), env.pc.data_ptr(), nsrc, \
            rowstride, n, K
        return a, out

    def mk_wsum():
        keep = []
        a, out = base_args(keep)
        return a, [out], keep

    same(run_both("wsum", mk_wsum))

    def mk_wsum_k():
        keep = []
        a, out = base_args(keep)
        kd = dev(kraw)
        keep.append(kd)
        return L.WsumKArgs(a, kd.data_ptr()), [out], keep

    same(run_both("wsum_k", mk_wsum_k))

    wmulti = [[[int(rng.integers(0, env.primes[r])) for r in range(rowstride)] for _ in range(nsrc)] for _ in range(3)]

    def mk_multi():
        keep = []
        sd = [dev(x) for x in srcs]
        keep += sd
        a = L.WsumMultiArgs()
        outs = []
        for m in range(3):
            wm = wmulti[m]
            wd = dev(np.array(wm, np.uint64).ravel())
            wsd = dev(np.array([[shoup(v, env.primes[r]) for r, v in enumerate(row)] for row in wm], np.uint64).ravel())
            out = torch.zeros_like(sd[0])
            keep += [wd, wsd]
            outs.append(out)
            a.out[m], a.w[m], a.ws[m] = env.cref(out), wd.data_ptr(), wsd.data_ptr()
            a.n[m] = [env.R, 7, 10][m]
            if m == 1:
                kd = dev(kraw)
                keep.append(kd)
                a.k[m] = kd.data_ptr()
        for j in range(nsrc):
            a.src[j] = env.cref(sd[j])
        a.pr, a.nout, a.nsrc, a.rowstride, a.K, a.nmax = env.pc.data_ptr(), 3, nsrc, rowstride, K, env.R
        return a, outs, keep

    same(run_both("wsum_multi", mk_multi))


@pytest.mark.parametrize("acc", [0, 1, 3])
def test_tensor_sum_and_multi(env, acc):
    rng = np.random.default_rng(140 + acc)
    K, n, npairs = 2, env.R, 5
    A = [env.cts(rng, K) for _ in range(npairs)]
    Bv = [env.cts(rng, K) for _ in range(npairs)]
    out0, d20 = env.cts(rng, K), env.cts(rng, K)

    def mk_sum():
        ad, bd = [dev(x) for x in A], [dev(x) for x in Bv]
        out, d2 = dev(out0), dev(d20)
        a = L.TensorSumArgs()
        a.out, a.d2 = env.cref(out), env.cref(d2)
        for j in range(npairs):
            a.a[j], a.b[j] = env.cref(ad[j]), env.cref(bd[j])
        a.pr, a.npairs, a.acc, a.n, a.K = env.pc.data_ptr(), npairs, acc, n, K
        return a, [out, d2], ad + bd

    same(run_both("tensor_sum", mk_sum))

    def mk_multi():
        ad, bd = [dev(x) for x in A], [dev(x) for x in Bv]
        outs = [(dev(out0), dev(d20)) for _ in range(3)]
        a = L.TensorMultiArgs()
        for o in range(3):
            a.out[o], a.d2[o] = env.cref(outs[o][0]), env.cref(outs[o][1])
            for j in range(npairs):  # output o pairs (a[j], b[(j + o) % npairs])
                a.a[o][j], a.b[o][j] = env.cref(ad[j]), env.cref(bd[(j + o) % npairs])
        a.pr, a.nout, a.npairs, a.acc, a.n, a.K = env.pc.data_ptr(), 3, npairs, acc, n, K
        return a, [t for pair in outs for t in pair], ad + bd

    same(run_both("tensor_multi", mk_multi))


@pytest.mark.parametrize("sub", [0, 1])
def test_md_epilogue_to_and_combine_to(env, sub):
    rng = np.random.default_rng(150 + sub)
    K, n = 2, 9
    x, t, a0, d0 = env.cts(rng, K), env.cts(rng, K), env.cts(rng, K), env.cts(rng, K)
    binv = [int(rng.integers(1, p)) for p in env.primes]
    binvs = [shoup(v, p) for v, p in zip(binv, env.primes)]

    def mk_md():
        xd, td, ad, dd = dev(x), dev(t), dev(a0), dev(d0)
        bi, bis = dev(binv), dev(binvs)
        m = L.MdEpiArgs(env.cref(dd), env.cref(xd), env.cref(td), bi.data_ptr(), bis.data_ptr(), None,
                        env.pc.data_ptr(), 0, n, K, 0)
        return L.MdEpiToArgs(m, env.cref(ad), sub, 0), [dd], [xd, td, ad, bi, bis]

    same(run_both("md_epilogue_to", mk_md))

    def mk_comb():
        xd, td, od = dev(x), dev(t), dev(d0)
        al, als = dev(binv), dev(binvs)
        r = L.RescaleCombineArgs(env.cref(xd), env.cref(td), al.data_ptr(), als.data_ptr(), env.pc.data_ptr(), n, K)
        return L.RescaleCombineToArgs(r, env.cref(od)), [od, xd], [td, al, als]

    same(run_both("rescale_combine_to", mk_comb))


def test_rescale_fwd(env):
    """rescale_fwd (two dropped primes, pre-factors): the corrections and their forward NTT with the combine epilogue;
    rows 0..top-2 of x must agree (tmp is scratch)."""
    rng = np.random.default_rng(160)
    K, top = 2, 7
    q = env.primes
    a_, b_ = top, top - 1
    nrows = top - 1

    def qlql(xp, i):
        return (-pow(q[xp], -1, q[i])) % q[i]

    A = [((pow(q[b_], -1, q[i]) * qlql(a_, i)) % q[i]) if i < nrows else 0 for i in range(env.R)]
    B = [qlql(b_, i) if i < nrows else 0 for i in range(env.R)]
    al = [((pow(q[a_], -1, q[i]) * pow(q[b_], -1, q[i])) % q[i]) if i < nrows else 1 for i in range(env.R)]
    As, Bs, als = ([shoup(v, q[i]) for i, v in enumerate(arr)] for arr in (A, B, al))
    qam = [q[a_] % q[i] for i in range(env.R)]
    qbm = [q[b_] % q[i] for i in range(env.R)]
    x0 = env.cts(rng, K)
    ca, cb = int(rng.integers(2, q[a_])), int(rng.integers(2, q[b_]))
    roff = [(c * 2 + part) * env.R + i for c in range(K) for part in range(2) for i in range(nrows)]
    rprime = [i for c in range(K) for part in range(2) for i in range(nrows)]

    def mk():
        keep = [dev(v) for v in (A, B, As, Bs, qam, qbm, al, als)]
        xd, tmp = dev(x0), torch.zeros((K, 2, env.R, env.n), dtype=torch.int64, device="cuda")
        keep.append(tmp)
        rs = L.RescaleArgs(env.cref(xd), env.cref(tmp), *[v.data_ptr() for v in keep[:6]], env.pc.data_ptr(),
                           pow(q[a_], -1, q[b_]), qlql(a_, b_), ca, cb, top, nrows, K, 2)
        ntt = env.ntt_args(tmp, roff, rprime, keep, eout=xd.data_ptr(), ex=xd.data_ptr(), es=keep[6].data_ptr(),
                           ess=keep[7].data_ptr(), epi=3, xnum=1)
        return L.RescaleNttArgs(rs, ntt), [xd], keep

    got = run_both("rescale_fwd", mk)
    a, b = got["ours"][0].reshape(K, 2, env.R, env.n), got["ref"][0].reshape(K, 2, env.R, env.n)
    assert (a[:, :, :nrows] == b[:, :, :nrows]).all()
