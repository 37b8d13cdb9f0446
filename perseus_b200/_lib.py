"""ctypes binding of perseus_b200/libpcb200.so (the C ABI declared in include/pcb200.h).

The library is built in-tree (perseus_b200/build.py). Loading fails loudly when it is missing: there is no CPU
fallback for any op of this package.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpcb200.so")

vp = C.c_void_p
u64p = C.POINTER(C.c_uint64)


class PrimeConst(C.Structure):
    _fields_ = [("p", C.c_uint64), ("mu_lo", C.c_uint64), ("mu_hi", C.c_uint64), ("neal_mu", C.c_uint64),
                ("bits", C.c_uint32), ("word_bits", C.c_uint32), ("mont_pinv", C.c_uint64),
                ("mont_r2", C.c_uint64), ("split", C.c_uint64)]


class RowSet(C.Structure):
    _fields_ = [("nq", C.c_int32), ("np", C.c_int32), ("qmax", C.c_int32), ("pad", C.c_int32)]


class PolyRef(C.Structure):
    _fields_ = [("base", vp), ("ct_stride", C.c_uint64), ("part_stride", C.c_uint64)]


class NttArgs(C.Structure):
    _fields_ = [("base", vp), ("roff", vp), ("rprime", vp), ("fw", vp), ("fws", vp), ("iw", vp), ("iws", vp),
                ("ninv", vp), ("ninvs", vp), ("pr", vp), ("nrows", C.c_int32), ("chunk", C.c_int32), ("src", vp),
                ("soff", vp), ("eout", vp), ("ex", vp), ("es", vp), ("ess", vp), ("epi", C.c_int32),
                ("snum", C.c_int32), ("sstride", C.c_uint64), ("xnum", C.c_int32), ("lazy", C.c_int32),
                ("xstride", C.c_uint64), ("ed", vp)]


class BconvJob(C.Structure):
    _fields_ = [(f, C.c_uint32) for f in ("src_off", "dst_off", "nsrc", "ntgt", "pool_off", "exact", "prescaled", "split")]


class BconvArgs(C.Structure):
    _fields_ = [("src", vp), ("dst", vp), ("jobs", vp), ("pool", vp), ("pr", vp), ("njobs", C.c_int32),
                ("max_tgt", C.c_int32), ("kind", C.c_int32), ("pad", C.c_int32)]


class EwArgs(C.Structure):
    _fields_ = [("out", PolyRef), ("a", PolyRef), ("b", PolyRef), ("rs", RowSet), ("sc", vp), ("scs", vp),
                ("pr", vp), ("K", C.c_int32), ("nparts", C.c_int32), ("sub", C.c_int32), ("zero_p", C.c_int32)]


class KsArgs(C.Structure):
    _fields_ = [("c1", vp), ("modup", vp), ("c0", vp), ("out0", vp), ("out1", vp), ("kb", vp), ("ka", vp),
                ("autok", vp), ("rows", vp), ("digit_of", vp), ("pmod", vp), ("pmods", vp), ("pr", vp),
                ("ct_stride", C.c_uint64), ("mu_ct_stride", C.c_uint64), ("mu_digit_stride", C.c_uint64),
                ("out_ct_stride", C.c_uint64), ("out_rot_stride", C.c_uint64), ("key_digit_stride", C.c_uint64),
                ("K", C.c_int32), ("R", C.c_int32), ("ndig", C.c_int32), ("c0_mode", C.c_int32), ("nq", C.c_int32),
                ("nrows", C.c_int32)]


class EpiArgs(C.Structure):
    _fields_ = [("dst", vp), ("conv", vp), ("binv", vp), ("binvs", vp), ("k", vp), ("part_stride", C.c_uint64),
                ("dbl", C.c_int32), ("pad", C.c_int32), ("alpha", vp), ("alphas", vp)]


class KeyTab(C.Structure):
    _fields_ = [("kb", vp), ("seed", vp), ("row_words", C.c_uint64), ("bits", C.c_int32), ("q_top", C.c_int32),
                ("srows", C.c_int32), ("nregen", C.c_int32)]


class KsRegenArgs(C.Structure):
    _fields_ = [("ks", KsArgs), ("seed", vp), ("epi", EpiArgs), ("use_epi", C.c_int32), ("pad", C.c_int32),
                ("key", KeyTab), ("add", vp)]


class KsKeyArgs(C.Structure):
    _fields_ = [("ks", KsArgs), ("key", KeyTab)]


class CoeffArgs(C.Structure):
    _fields_ = [("scratch", vp), ("out", vp), ("fw", vp), ("fws", vp), ("pr", vp), ("overflow", vp),
                ("part_stride", C.c_uint64), ("scale", C.c_double), ("n", C.c_int32), ("L", C.c_int32),
                ("accumulate", C.c_int32), ("pad", C.c_int32), ("rows", vp * 32), ("ct", vp * 32)]


class PackSplitArgs(C.Structure):
    _fields_ = [("q", vp), ("p", vp), ("out", vp), ("q_stride", C.c_uint64), ("p_stride", C.c_uint64),
                ("out_stride", C.c_uint64), ("K", C.c_int32), ("sub", C.c_int32), ("nq", C.c_int32),
                ("nrows", C.c_int32)]


class PackDotArgs(C.Structure):
    _fields_ = [("dig", vp), ("kb", vp), ("ka", vp), ("c0", vp), ("out0", vp), ("out1", vp), ("rows", vp),
                ("pmod", vp), ("pmods", vp), ("pr", vp), ("dig_stride", C.c_uint64), ("ct_stride", C.c_uint64),
                ("out_ct_stride", C.c_uint64), ("K", C.c_int32), ("sub", C.c_int32), ("nq", C.c_int32),
                ("nrows", C.c_int32)]


class CtsArgs(C.Structure):
    _fields_ = [("x", vp), ("modup", vp), ("res", vp), ("kb", vp), ("ka", vp), ("kinv", vp), ("pts", vp), ("rows", vp),
                ("digit_of", vp), ("pmod", vp), ("pmods", vp), ("pr", vp), ("ct_stride", C.c_uint64),
                ("part_stride", C.c_uint64), ("mu_ct_stride", C.c_uint64), ("mu_digit_stride", C.c_uint64),
                ("key_digit_stride", C.c_uint64)] + [(n, C.c_int32) for n in (
                    "K", "B", "G", "npts", "ndig", "nq", "nlive", "ptw", "pt_prow")] + [
                ("enc", C.c_uint32), ("ngrp", C.c_int32), ("nrows", C.c_int32), ("kmax", C.c_int32),
                ("pair_cts", C.c_int32), ("x0", vp)]


class CtsRegenArgs(C.Structure):
    _fields_ = [("cts", CtsArgs), ("key", KeyTab)]


class KskExpandArgs(C.Structure):
    _fields_ = [("out", vp), ("seed", vp), ("prime_ids", vp), ("pr", vp), ("nmod", C.c_int32), ("dnum", C.c_int32),
                ("d0", C.c_int32), ("pad", C.c_int32)]


class TensorArgs(C.Structure):
    _fields_ = [("out", PolyRef), ("d2", PolyRef), ("a0", PolyRef), ("b0", PolyRef), ("a1", PolyRef),
                ("b1", PolyRef), ("coef", vp), ("coef_ct_stride", C.c_uint64), ("pr", vp), ("npairs", C.c_int32),
                ("acc", C.c_int32), ("n", C.c_int32), ("K", C.c_int32), ("dbl", C.c_int32), ("acc_d2", C.c_int32)]


class TensorYArgs(C.Structure):
    _fields_ = [("t", TensorArgs), ("y", PolyRef), ("c", vp), ("cs", vp), ("sub", C.c_int32), ("pad", C.c_int32)]


class MdEpiArgs(C.Structure):
    _fields_ = [("dst", PolyRef), ("x", PolyRef), ("t", PolyRef), ("binv", vp), ("binvs", vp), ("k", vp),
                ("pr", vp), ("dbl", C.c_int32), ("n", C.c_int32), ("K", C.c_int32), ("pad", C.c_int32)]


class RescaleArgs(C.Structure):
    _fields_ = [("x", PolyRef), ("tmp", PolyRef), ("A", vp), ("B", vp), ("As", vp), ("Bs", vp), ("qam", vp),
                ("qbm", vp), ("pr", vp), ("qinv_ab", C.c_uint64), ("C_ab", C.c_uint64), ("ca", C.c_uint64),
                ("cb", C.c_uint64), ("top", C.c_int32), ("nrows", C.c_int32), ("K", C.c_int32), ("ndrop", C.c_int32)]


class RescaleCombineArgs(C.Structure):
    _fields_ = [("x", PolyRef), ("tmp", PolyRef), ("alpha", vp), ("alphas", vp), ("pr", vp), ("n", C.c_int32),
                ("K", C.c_int32)]


class RescaleNttArgs(C.Structure):
    _fields_ = [("rs", RescaleArgs), ("ntt", NttArgs)]


class RescaleCombineToArgs(C.Structure):
    _fields_ = [("a", RescaleCombineArgs), ("out", PolyRef)]


class MdEpiToArgs(C.Structure):
    _fields_ = [("m", MdEpiArgs), ("a", PolyRef), ("sub", C.c_int32), ("pad", C.c_int32)]


class WsumArgs(C.Structure):
    _fields_ = [("out", PolyRef), ("src", PolyRef * 8), ("w", vp), ("ws", vp), ("pr", vp), ("nsrc", C.c_int32),
                ("rowstride", C.c_int32), ("n", C.c_int32), ("K", C.c_int32)]


class WsumKArgs(C.Structure):
    _fields_ = [("w", WsumArgs), ("k", vp)]


class WsumMultiArgs(C.Structure):
    _fields_ = [("out", PolyRef * 3), ("src", PolyRef * 8), ("w", vp * 3), ("ws", vp * 3), ("k", vp * 3), ("pr", vp),
                ("nout", C.c_int32), ("nsrc", C.c_int32), ("rowstride", C.c_int32), ("K", C.c_int32),
                ("n", C.c_int32 * 3), ("nmax", C.c_int32)]


EWM_MAX, TSUM_MAX, TMULTI_OUT, TMULTI_PAIRS = 48, 16, 4, 32


class EwManyArgs(C.Structure):
    _fields_ = [("out", vp * EWM_MAX), ("a", vp * EWM_MAX), ("b", vp * EWM_MAX), ("c", vp * EWM_MAX), ("pr", vp),
                ("n", C.c_int32), ("nrows", C.c_int32)]


class SubMulManyArgs(C.Structure):
    _fields_ = [("out", vp * EWM_MAX), ("a", vp * EWM_MAX), ("b", vp * EWM_MAX), ("t", vp), ("pr", vp),
                ("n", C.c_int32), ("nrows", C.c_int32)]


class TensorSumArgs(C.Structure):
    _fields_ = [("out", PolyRef), ("d2", PolyRef), ("a", PolyRef * TSUM_MAX), ("b", PolyRef * TSUM_MAX), ("pr", vp),
                ("npairs", C.c_int32), ("acc", C.c_int32), ("n", C.c_int32), ("K", C.c_int32)]


class TensorMultiArgs(C.Structure):
    _fields_ = [("out", PolyRef * TMULTI_OUT), ("d2", PolyRef * TMULTI_OUT), ("a", (PolyRef * TMULTI_PAIRS) * TMULTI_OUT),
                ("b", (PolyRef * TMULTI_PAIRS) * TMULTI_OUT), ("pr", vp), ("nout", C.c_int32), ("npairs", C.c_int32),
                ("acc", C.c_int32), ("n", C.c_int32), ("K", C.c_int32), ("pad", C.c_int32)]


class PtDotArgs(C.Structure):
    _fields_ = [("rot", PolyRef), ("res", PolyRef), ("rot_stride", C.c_uint64), ("res_stride", C.c_uint64),
                ("pts", vp), ("pr", vp), ("rs", RowSet), ("npts", C.c_int32), ("bstep", C.c_int32),
                ("gstep", C.c_int32), ("K", C.c_int32), ("ptw", C.c_int32), ("pt_prow", C.c_int32),
                ("enc", C.c_uint32), ("pad", C.c_int32)]


class AddConstArgs(C.Structure):
    _fields_ = [("x", PolyRef), ("k", vp), ("pr", vp), ("n", C.c_int32), ("K", C.c_int32)]


class MulTableArgs(C.Structure):
    _fields_ = [("out", PolyRef), ("in_", PolyRef), ("t", vp), ("pr", vp), ("n", C.c_int32), ("K", C.c_int32)]


class MulAddArgs(C.Structure):
    _fields_ = [("m", MulTableArgs), ("y", PolyRef), ("sub", C.c_int32), ("pad", C.c_int32)]


class MulAddNArgs(C.Structure):
    _fields_ = [("out", PolyRef), ("y", PolyRef), ("x", PolyRef * 8), ("t", vp * 8), ("pr", vp), ("n", C.c_int32),
                ("K", C.c_int32), ("nterm", C.c_int32), ("lazy", C.c_int32)]


class AutomorphArgs(C.Structure):
    _fields_ = [("out", PolyRef), ("in_", PolyRef), ("add", PolyRef), ("rs", RowSet), ("pr", vp), ("k", C.c_uint32),
                ("K", C.c_int32), ("nparts", C.c_int32), ("has_add", C.c_int32)]


class EncryptArgs(C.Structure):
    _fields_ = [("c0", vp), ("c1", vp), ("s", vp), ("e", vp), ("m", vp), ("seed", vp), ("pr", vp),
                ("nonce", C.c_uint32), ("nl", C.c_int32)]


class ModRaiseArgs(C.Structure):
    _fields_ = [("x", vp), ("pr", vp), ("ct_stride", C.c_uint64), ("part_stride", C.c_uint64),
                ("qhatinv", C.c_uint64 * 4), ("qhat", (C.c_uint64 * 64) * 4), ("K", C.c_int32), ("d", C.c_int32),
                ("r0", C.c_int32), ("r1", C.c_int32), ("nparts", C.c_int32), ("pad", C.c_int32)]


class SmallInt1Args(C.Structure):
    _fields_ = [("x", vp), ("pr", vp), ("ct_stride", C.c_uint64), ("part_stride", C.c_uint64), ("mc", C.c_uint64),
                ("sh", C.c_int32), ("nrows", C.c_int32), ("K", C.c_int32), ("nparts", C.c_int32)]


class KskUnpackArgs(C.Structure):
    _fields_ = [("out", vp), ("in_", vp), ("row_words", C.c_uint64), ("nrows", C.c_int32), ("bits", C.c_int32)]


class KskGenArgs(C.Structure):
    _fields_ = [("b", vp), ("a", vp), ("e", vp), ("s_new", vp), ("s_old", vp), ("seed", vp), ("ids", vp),
                ("digit_of", vp), ("pmod", vp), ("pmods", vp), ("pr", vp), ("row_words", C.c_uint64),
                ("nrows", C.c_int32), ("ndig", C.c_int32), ("nq", C.c_int32), ("bits", C.c_int32), ("sq", C.c_int32),
                ("pad", C.c_int32)]


LAUNCHERS = ["ntt_fwd", "ntt_inv", "bconv", "ew_add", "ew_scale", "ew_sub_mul", "ew_copy", "pt_dot", "ks_dot",
             "ks_dot_regen", "ksk_expand", "cts_fused", "tensor", "md_epilogue", "wsum", "add_const", "mul_table",
             "rescale_coef", "rescale_combine", "automorph", "encode", "encrypt", "ksk_gen", "ksk_unpack",
             "mod_raise", "small_int", "spru_extract", "spru_fft_pass", "spru_scatter", "cts_fused_regen",
             "ks_dot_key", "pcmm", "ccmm", "wsum_k", "rescale_combine_to", "md_epilogue_to", "small_int1",
             "coeff_sum", "mul_add", "rescale_fwd", "mul_add_n", "tensor_y", "wsum_multi", "bconv_wide", "tfhe",
             "tensor_sum", "tensor_multi", "tensor_seeded", "ew_many", "submul_many", "pack_split", "pack_dot"]
LAUNCH = C.CFUNCTYPE(C.c_int, vp, vp)


class KernelTable(C.Structure):
    _fields_ = [("abi", C.c_uint32), ("word_bytes", C.c_uint32), ("mm", C.c_uint32), ("log_n", C.c_uint32)] + [
        (n, LAUNCH) for n in LAUNCHERS]


RING_LAUNCHERS = ["ntt_fwd", "ntt_inv", "ntt_fwd_g", "ntt_inv_g", "bconv", "ew_add", "ew_scale", "ew_sub_mul", "ew_copy"]


class RingTable(C.Structure):
    _fields_ = [("abi", C.c_uint32), ("word_bytes", C.c_uint32), ("mm", C.c_uint32), ("log_n", C.c_uint32)] + [
        (n, LAUNCH) for n in RING_LAUNCHERS]


class Params(C.Structure):
    _fields_ = [("log_n", C.c_uint32), ("nq", C.c_int32), ("kp", C.c_int32), ("dnum", C.c_int32), ("q", u64p),
                ("p", u64p), ("k_max", C.c_int32), ("key_source", C.c_int32)]


SIZES = {"PrimeConst": 64, "RowSet": 16, "PolyRef": 24, "NttArgs": 176, "BconvJob": 32, "BconvArgs": 56,
         "EwArgs": 128, "KsArgs": 176, "EpiArgs": 72, "KeyTab": 40, "KsRegenArgs": 312, "KskExpandArgs": 48,
         "TensorArgs": 192, "MdEpiArgs": 120, "RescaleArgs": 152, "RescaleCombineArgs": 80, "AutomorphArgs": 112,
         "EncryptArgs": 64, "KskGenArgs": 120, "KskUnpackArgs": 32, "KsKeyArgs": 216, "PtDotArgs": 128, "AddConstArgs": 48, "MulTableArgs": 72,
         "MulAddArgs": 104, "MulAddNArgs": 328, "ModRaiseArgs": 2136, "TensorYArgs": 240, "CtsArgs": 200, "PackSplitArgs": 64, "CoeffArgs": 80 + 16 * 32, "PackDotArgs": 120, "CtsRegenArgs": 240, "SmallInt1Args": 56, "RescaleNttArgs": 328,
         "RescaleCombineToArgs": 104, "MdEpiToArgs": 152, "WsumArgs": 256, "WsumKArgs": 264, "WsumMultiArgs": 376,
         "EwManyArgs": 4 * 48 * 8 + 16, "SubMulManyArgs": 3 * 48 * 8 + 24, "TensorSumArgs": 2 * 24 + 2 * 16 * 24 + 24,
         "TensorMultiArgs": (2 * 4 + 2 * 4 * 32) * 24 + 32, "KernelTable": 16 + 52 * 8, "RingTable": 16 + 9 * 8}

_lib = None


class PcbError(RuntimeError):
    pass


def lib():
    """The loaded CUDA library (raises when it has not been built: no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise PcbError(f"{LIB_PATH} is missing: build it with `python perseus_b200/build.py` (no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    i32, i64, u32, u64, dbl = C.c_int32, C.c_int64, C.c_uint32, C.c_uint64, C.c_double
    sig = {
        "pc_table_u64_barrett64": (C.POINTER(KernelTable), []),
        "pc_ring_u64_14": (C.POINTER(RingTable), []),
        "pcb_kernel_table": (C.POINTER(KernelTable), [C.c_int32]),
        "pc_ring_u64_16": (C.POINTER(RingTable), []),
        "pcb_last_error": (C.c_char_p, []),
        "pcb_launch_count": (C.c_uint64, []),
        "pcb_device_timeouts": (C.c_uint32, []),
        "pcb_fp64_fma_loop": (C.c_int64, [vp, i32, vp]),
        "pcb_key_seed": (C.c_int, [vp, i32, vp]),
        "pcb_key_load": (C.c_int, [vp, i32, u64, vp, vp, vp]),
        "pcb_ct_compress": (C.c_int, [vp, vp, i32, i32, vp, vp]),
        "pcb_wire_sum64": (u64, [vp, C.c_size_t]),
        "pcb_wire_packed_words": (C.c_size_t, [C.c_size_t, i32]),
        "pcb_wire_packed_row_words": (C.c_size_t, [C.c_size_t, i32]),
        "pcb_wire_pack_bits": (C.c_int, [vp, C.c_size_t, i32, vp]),
        "pcb_wire_unpack_bits": (C.c_int, [vp, C.c_size_t, C.c_size_t, i32, vp]),
        "pcb_wire_pack_row": (C.c_int, [vp, C.c_size_t, i32, vp, C.c_size_t]),
        "pcb_wire_write_header": (i64, [C.c_char_p, vp, u64, vp, u64]),
        "pcb_wire_read_header": (i64, [vp, u64, C.c_char_p, C.POINTER(C.c_uint64)]),
        "pcb_wire_unpack_coeffs": (C.c_int, [vp, i32, vp, C.c_size_t, i32, vp]),
        "pcb_ctx_bytes": (i64, [C.POINTER(Params), i32]),
        "pcb_ctx_create": (C.c_int, [C.POINTER(Params), i32, vp, C.c_size_t, vp, C.POINTER(vp)]),
        "pcb_ctx_destroy": (None, [vp]),
        "pcb_ctx_rows": (C.c_int, [vp]),
        "pcb_ctx_tables": (C.c_int, [vp] + [C.POINTER(vp)] * 7),
        "pcb_keygen": (C.c_int, [vp, u64, u32, dbl, i32, u64p, vp]),
        "pcb_key_ptrs": (C.c_int, [vp, i32, C.POINTER(vp), C.POINTER(vp), C.POINTER(u64)]),
        "pcb_key_copy": (C.c_int, [vp, i32, vp, vp, vp]),
        "pcb_encrypt": (C.c_int, [vp, C.POINTER(dbl), i32, i32, dbl, i32, vp, vp]),
        "pcb_decrypt": (C.c_int, [vp, vp, i32, i32, dbl, C.POINTER(dbl), vp]),
        "pcb_encode": (C.c_int, [vp, C.POINTER(dbl), i32, i32, dbl, i32, u64p]),
        "pcb_pt_load": (C.c_int, [vp, u64p, i32, vp, vp]),
        "pcb_encode_ext": (C.c_int, [vp, C.POINTER(dbl), i32, i32, dbl, i32, u64p]),
        "pcb_pt_load_ext": (C.c_int, [vp, u64p, i32, vp, vp]),
        "pcb_add": (C.c_int, [vp, vp, vp, vp, i32, i32, vp]),
        "pcb_sum": (C.c_int, [vp, vp, i32, vp, i32, i32, vp]),
        "pcb_rotate_sum": (C.c_int, [vp, vp, vp, i32, vp, i32, i32, vp]),
        "pcb_rotate_and_sum_radix": (C.c_int, [vp, vp, C.c_int64, C.c_int64, i32, vp, i32, i32, vp]),
        "pcb_sub": (C.c_int, [vp, vp, vp, vp, i32, i32, vp]),
        "pcb_mult": (C.c_int, [vp, vp, vp, vp, i32, i32, vp]),
        "pcb_rescale": (C.c_int, [vp, vp, i32, i32, vp]),
        "pcb_rescale_static": (C.c_int, [vp, vp, i32, vp]),
        "pcb_rotate": (C.c_int, [vp, vp, i64, vp, i32, i32, vp]),
        "pcb_rotate_and_sum": (C.c_int, [vp, vp, i64, i64, vp, i32, i32, vp]),
        "pcb_rotate_hoisted": (C.c_int, [vp, vp, C.POINTER(i64), i32, C.POINTER(vp), i32, i32, vp]),
        "pcb_mult_pt": (C.c_int, [vp, vp, vp, vp, i32, i32, vp]),
        "pcb_add_pt": (C.c_int, [vp, vp, vp, vp, i32, i32, vp]),
        "pcb_mult_pt_add": (C.c_int, [vp, vp, vp, vp, vp, i32, i32, i32, vp]),
        "pcb_linear_transform": (C.c_int, [vp, vp, vp, i32, i32, C.c_int64, vp, vp, i32, i32, vp]),
        "pcb_linear_transform_multi": (C.c_int, [vp, vp, vp, i32, i32, i32, C.c_int64, vp, vp, i32, i32, vp]),
        "pcb_linear_transform_ext": (C.c_int, [vp, vp, vp, i32, i32, i32, C.c_int64, C.c_int64, vp, vp, i32, i32, vp]),
        "pcb_mult_pt_sum": (C.c_int, [vp, vp, vp, i32, vp, i32, i32, vp]),
        "pcb_keyswitch": (C.c_int, [vp, vp, vp, i32, i32, u32, vp, i32, i32, u64, vp]),
        "pcb_mod_raise": (C.c_int, [vp, vp, i32, i32, vp]),
        "pcb_ntt_batch": (C.c_int, [vp, vp, i32, i32, vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def check(rc, what=""):
    if rc != 0:
        msg = lib().pcb_last_error().decode(errors="replace")
        raise PcbError(f"{what} failed ({rc}): {msg}")
    return rc


def kernel_table(log_n=16):
    if log_n == 16:
        return lib().pc_table_u64_barrett64().contents
    t = lib().pcb_kernel_table(log_n)
    if not t:
        raise ValueError(f"no kernel table at log n {log_n}")
    return t.contents


def ring_table(log_n):
    return (lib().pc_ring_u64_14() if log_n == 14 else lib().pc_ring_u64_16()).contents
