"""The C ABI without a GPU: the library loads, exports every symbol include/pcb200.h declares, and its argument
structs and tables have the reference's sizes (crates/pc-kernels/kernels/args.cuh static asserts)."""
import ctypes as C
import os
import re

import pytest

from perseus_b200 import _lib as L
from perseus_b200 import fhe

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "pcb200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b((?:pc|pcb)_\w+)\s*\(", src, re.M)))


def test_library_exports_declared_symbols():
    lib = L.lib()
    names = declared_symbols()
    assert "pc_table_u64_barrett64" in names and "pcb_mult" in names and len(names) > 20
    for n in names:
        assert hasattr(lib, n), n


@pytest.mark.parametrize("name,size", sorted(L.SIZES.items()))
def test_struct_sizes(name, size):
    assert C.sizeof(getattr(L, name)) == size


def test_table_headers():
    t = L.kernel_table()
    assert (t.abi, t.word_bytes, t.mm, t.log_n) == (30, 8, 0, 16)
    for n in L.LAUNCHERS:
        assert getattr(t, n), n  # every entry is non-null (absent ones return -1)
    for ln in (14, 16):
        r = L.ring_table(ln)
        assert (r.abi, r.word_bytes, r.mm, r.log_n) == (7, 8, 0, ln)


def test_absent_entries_refuse():
    t = L.kernel_table()
    assert t.tfhe(None, None) == -1 and t.pcmm(None, None) == -1 and t.cts_fused(None, None) == -1
    assert t.small_int(None, None) == -2  # 32-bit words only, as the reference's 64-bit table answers
    for n in ("pt_dot", "ks_dot_regen", "ks_dot_key", "ntt_fwd"):  # a null argument pointer: refused by every entry
        assert getattr(t, n)(None, None) == -1, n


def test_plaintext_entries_refuse_out_of_range():
    """pt_dot K in [1, 8], mul_add_n nterm in [1, 8], mul_add sub in [0, 2] (args.cuh:184-200, :508-528): refused on
    the host (-1) before any launch; the pointers are fakes that no kernel sees."""
    t = L.kernel_table()
    n = 1 << 16
    a = L.PtDotArgs()
    a.rot = a.res = L.PolyRef(0x1000, 0, 0)
    a.pr, a.pts, a.rs = 0x2000, 0x3000, L.RowSet(1, 0, 1, 0)
    a.npts, a.bstep, a.gstep, a.ptw, a.enc = 1, 1, 1, n, 0xFFFFFFFF
    for k in (0, 9):
        a.K = k
        assert t.pt_dot(C.cast(C.pointer(a), C.c_void_p), None) == -1
    a.K, a.bstep = 1, 257  # 128-bit sums of at most 256 products
    assert t.pt_dot(C.cast(C.pointer(a), C.c_void_p), None) == -1
    m = L.MulAddNArgs()
    m.out, m.pr, m.n, m.K = L.PolyRef(0x1000, 0, 0), 0x2000, 1, 1
    for nt in (0, 9):
        m.nterm = nt
        assert t.mul_add_n(C.cast(C.pointer(m), C.c_void_p), None) == -1
    z = L.PolyRef(0x1000, 0, 0)
    ma = L.MulAddArgs(L.MulTableArgs(z, z, 0x3000, 0x2000, 1, 1), z, 3, 0)
    assert t.mul_add(C.cast(C.pointer(ma), C.c_void_p), None) == -1
    mt = L.MulTableArgs(L.PolyRef(0x1008, 0, 0), z, 0x3000, 0x2000, 1, 1)  # misaligned row base
    assert t.mul_table(C.cast(C.pointer(mt), C.c_void_p), None) == -1
    ac = L.AddConstArgs(z, None, 0x2000, 1, 1)
    assert t.add_const(C.cast(C.pointer(ac), C.c_void_p), None) == -1


def test_null_arguments_refused_without_launch():
    t = L.kernel_table()
    a = L.NttArgs()
    assert t.ntt_fwd(C.cast(C.pointer(a), C.c_void_p), None) == -1
    assert t.ntt_fwd(None, None) == -1


def test_misaligned_rows_refused_without_launch():
    """Rows move 16 bytes at a time: a row base off a 16-byte boundary is refused on the host (-1) before any
    launch. The pointers are fakes that no kernel ever sees: the refusal comes first."""
    t = L.kernel_table()
    a = L.NttArgs()
    a.base, a.roff, a.rprime, a.fw, a.fws, a.iw, a.iws, a.ninv, a.ninvs, a.pr = (0x1008,) + (0x2000,) * 9
    a.nrows, a.snum, a.xnum = 1, 1, 1
    assert t.ntt_fwd(C.cast(C.pointer(a), C.c_void_p), None) == -1
    assert t.ntt_inv(C.cast(C.pointer(a), C.c_void_p), None) == -1
    e = L.EwArgs()
    e.out.base, e.a.base, e.b.base, e.pr = 0x1000, 0x1008, 0x1000, 0x2000
    e.rs.nq, e.K, e.nparts = 1, 1, 1
    assert t.ew_add(C.cast(C.pointer(e), C.c_void_p), None) == -1


def test_ctx_bytes_config2():
    ch = fhe.config2_chain()
    q = (C.c_uint64 * 24)(*ch.q)
    p = (C.c_uint64 * 8)(*ch.p)
    prm = L.Params(16, 24, 8, 3, C.cast(q, L.u64p), C.cast(p, L.u64p), 64, 0)
    nb = L.lib().pcb_ctx_bytes(C.byref(prm), 16)
    assert nb > 0
    gib = nb / 2**30
    assert 5 < gib < 40, gib  # workspaces for 64 ciphertexts + 16 keys fit one B200 many times over


def test_ctx_bytes_regenerated_keys():
    """PCB_KEYS_REGEN keeps b and a seed per key: the arena shrinks by every key's `a` rows; other sources refused."""
    ch = fhe.config2_chain()
    q = (C.c_uint64 * 24)(*ch.q)
    p = (C.c_uint64 * 8)(*ch.p)
    dense = L.Params(16, 24, 8, 3, C.cast(q, L.u64p), C.cast(p, L.u64p), 4, fhe.KEY_SOURCES["dense"])
    regen = L.Params(16, 24, 8, 3, C.cast(q, L.u64p), C.cast(p, L.u64p), 4, fhe.KEY_SOURCES["regen"])
    nd, nr = L.lib().pcb_ctx_bytes(C.byref(dense), 16), L.lib().pcb_ctx_bytes(C.byref(regen), 16)
    a_rows = 16 * 3 * 32 * (1 << 16) * 8
    assert 0 < nr and nd - nr == a_rows, (nd, nr)
    bad = L.Params(16, 24, 8, 3, C.cast(q, L.u64p), C.cast(p, L.u64p), 4, 7)
    assert L.lib().pcb_ctx_bytes(C.byref(bad), 1) < 0
    assert "key_source" in L.lib().pcb_last_error().decode()


def test_ctx_bytes_rejects_bad_chains():
    q = (C.c_uint64 * 2)(97, 193)
    p = (C.c_uint64 * 1)(257)
    prm = L.Params(16, 2, 1, 1, C.cast(q, L.u64p), C.cast(p, L.u64p), 1, 0)
    assert L.lib().pcb_ctx_bytes(C.byref(prm), 1) < 0
    assert "NTT prime" in L.lib().pcb_last_error().decode()


def test_chain_primes():
    c1, c2 = fhe.config1_chain(), fhe.config2_chain()
    assert len(c1.q) == 8 and len(c1.p) == 1 and all(q.bit_length() == 50 for q in c1.q) and c1.p[0].bit_length() == 60
    assert len(c2.q) == 24 and len(c2.p) == 8 and all(x.bit_length() == 50 for x in c2.q + c2.p)
    assert len(set(c2.q + c2.p)) == 32
    assert all((x - 1) % (2 << 16) == 0 for x in c2.q + c2.p)


def test_regen_entries_refuse_out_of_range():
    """ks_dot_regen / ks_dot_key: K in [0, 4], packed `b` rows (the reference's 32-bit words) refused on the host."""
    t = L.kernel_table()
    k = L.KsArgs()
    k.c1, k.modup, k.rows, k.digit_of, k.pr, k.kb = 0x1000, 0x1000, 0x2000, 0x2000, 0x2000, 0x3000
    k.out0 = k.out1 = 0x4000
    k.ndig, k.nrows, k.nq = 2, 1, 1
    r = L.KsRegenArgs()
    r.ks, r.seed = k, 0x5000
    r.ks.K = 5
    assert t.ks_dot_regen(C.cast(C.pointer(r), C.c_void_p), None) == -1
    r.ks.K, r.key.kb, r.key.srows, r.key.bits = 1, 0x6000, 2, 28
    assert t.ks_dot_regen(C.cast(C.pointer(r), C.c_void_p), None) == -1
    a = L.KsKeyArgs()
    a.ks = k
    a.ks.K, a.ks.R, a.ks.autok = 1, 1, 0x7000
    a.key.kb, a.key.seed, a.key.srows, a.key.bits = 0x6000, 0x5000, 2, 28
    assert t.ks_dot_key(C.cast(C.pointer(a), C.c_void_p), None) == -1
    a.key.bits, a.ks.K = 0, 9
    assert t.ks_dot_key(C.cast(C.pointer(a), C.c_void_p), None) == -1
