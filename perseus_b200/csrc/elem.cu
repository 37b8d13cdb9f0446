// Element-wise kernels of the hot path: ew_* (row sets), tensor, md_epilogue, rescale_coef / rescale_combine,
// automorph. Semantics of crates/pc-kernels/kernels/args.cuh (EwArgs :143-157, TensorArgs :355-367, MdEpiArgs
// :438-447, RescaleArgs :525-572, AutomorphArgs :580-592); host twin crates/pc-host/src/{elem,rescale}.rs.
//
// All of these are HBM-bound streams: every thread moves 4 consecutive words (two 16-byte vector accesses per
// operand), grids are (N / 1024, rows, ciphertexts x parts) so one launch covers a whole batch.
#include "arith.cuh"
#include "kernels.h"

namespace pcb {
namespace elem {

constexpr int BX = 256;
constexpr int WPT = 4;  // words per thread

struct V4 {
    uint64_t v[4];
};
__device__ __forceinline__ V4 ld4(const uint64_t* p) {
    const ulonglong2 a = ((const ulonglong2*)p)[0], b = ((const ulonglong2*)p)[1];
    return V4{{a.x, a.y, b.x, b.y}};
}
__device__ __forceinline__ void st4(uint64_t* p, const uint64_t (&r)[4]) {
    ((ulonglong2*)p)[0] = make_ulonglong2(r[0], r[1]);
    ((ulonglong2*)p)[1] = make_ulonglong2(r[2], r[3]);
}

enum EwOp { EW_ADD = 0, EW_SCALE = 1, EW_SUB_MUL = 2, EW_COPY = 3 };

template <int LOGN, int OP>
__global__ void __launch_bounds__(BX) ew(PcbEwArgs a) {
    const int row = rs_row(a.rs, blockIdx.y);
    const int c = blockIdx.z / a.nparts, part = blockIdx.z % a.nparts;
    const size_t i = ((size_t)blockIdx.x * BX + threadIdx.x) * WPT;
    uint64_t* o = at_row_w(a.out, c, part, row, LOGN) + i;
    uint64_t r[4];
    if (OP == EW_COPY) {
        const V4 x = ld4(at_row(a.a, c, part, row, LOGN) + i);
#pragma unroll
        for (int w = 0; w < 4; ++w) r[w] = x.v[w];
        st4(o, r);
        return;
    }
    const uint64_t p = a.pr[row].p;
    if (OP == EW_SCALE && a.zero_p && (int)blockIdx.y >= a.rs.nq) {
#pragma unroll
        for (int w = 0; w < 4; ++w) r[w] = 0;
        st4(o, r);
        return;
    }
    const V4 x = ld4(at_row(a.a, c, part, row, LOGN) + i);
    if (OP == EW_SCALE) {
        const uint64_t s = ((const uint64_t*)a.sc)[row], ss = ((const uint64_t*)a.scs)[row];
#pragma unroll
        for (int w = 0; w < 4; ++w) r[w] = shoup(x.v[w], s, ss, p);
    } else {
        const V4 y = ld4(at_row(a.b, c, part, row, LOGN) + i);
        if (OP == EW_ADD) {
#pragma unroll
            for (int w = 0; w < 4; ++w) r[w] = a.sub ? sub_mod(x.v[w], y.v[w], p) : add_mod(x.v[w], y.v[w], p);
        } else {
            const uint64_t s = ((const uint64_t*)a.sc)[row], ss = ((const uint64_t*)a.scs)[row];
#pragma unroll
            for (int w = 0; w < 4; ++w) r[w] = shoup(sub_mod(x.v[w], y.v[w], p), s, ss, p);
        }
    }
    st4(o, r);
}

// Kernels that move 4 words per thread as two 16-byte accesses need every row to start on a 16-byte boundary: the
// base 16-byte aligned and both strides even (a null base is checked by the caller)
__host__ inline bool ok16(const PcbPolyRef& r) {
    return ((uintptr_t)r.base & 15) == 0 && (r.ct_stride & 1) == 0 && (r.part_stride & 1) == 0;
}

template <int LOGN, int OP>
int ew_launch(const PcbEwArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbEwArgs& a = *ap;
    const int rows = a.rs.nq + a.rs.np;
    if (a.K < 0 || a.nparts < 1 || a.rs.nq < 0 || a.rs.np < 0 || !a.out.base || !a.a.base) return PCB_BAD_ARGS;
    if (OP != EW_COPY && !a.pr) return PCB_BAD_ARGS;
    if ((OP == EW_ADD || OP == EW_SUB_MUL) && !a.b.base) return PCB_BAD_ARGS;
    if ((OP == EW_SCALE || OP == EW_SUB_MUL) && (!a.sc || !a.scs)) return PCB_BAD_ARGS;
    if (!ok16(a.out) || !ok16(a.a) || ((OP == EW_ADD || OP == EW_SUB_MUL) && !ok16(a.b))) return PCB_BAD_ARGS;
    if (rows == 0 || a.K == 0) return 0;
    ew<LOGN, OP><<<dim3((1 << LOGN) / (BX * WPT), rows, a.K * a.nparts), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ tensor
// (c0, c1, d2) = sum over up to two pairs (a, b) of (a0 b0, a0 b1 + a1 b0, a1 b1): lazy 128-bit sums, one reduction.
// Y (tensor_y, args.cuh:369-378): then (c0, c1) +/-= c[row] y, after the doubling (EvalMod's x y +/- c t in one pass).
template <int LOGN, bool Y>
__global__ void __launch_bounds__(BX) tensor(PcbTensorYArgs g) {
    const PcbTensorArgs& a = g.t;
    const int row = blockIdx.y, c = blockIdx.z;
    const PcbPrimeConst& pc = a.pr[row];
    const uint64_t p = pc.p;
    const size_t i = ((size_t)blockIdx.x * BX + threadIdx.x) * WPT;
    Acc s0[4], s1[4], s2[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) s0[w] = s1[w] = s2[w] = Acc{0, 0};
    for (int j = 0; j < a.npairs && j < 2; ++j) {
        const PcbPolyRef& x = j ? a.a1 : a.a0;
        const PcbPolyRef& y = j ? a.b1 : a.b0;
        const V4 x0 = ld4(at_row(x, c, 0, row, LOGN) + i), x1 = ld4(at_row(x, c, 1, row, LOGN) + i);
        const V4 y0 = ld4(at_row(y, c, 0, row, LOGN) + i), y1 = ld4(at_row(y, c, 1, row, LOGN) + i);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            mac(s0[w], x0.v[w], y0.v[w]);
            mac(s1[w], x0.v[w], y1.v[w]);
            mac(s1[w], x1.v[w], y0.v[w]);
            mac(s2[w], x1.v[w], y1.v[w]);
        }
    }
    uint64_t r0[4], r1[4], r2[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        r0[w] = reduce(s0[w], pc);
        r1[w] = reduce(s1[w], pc);
        r2[w] = reduce(s2[w], pc);
    }
    uint64_t* o0 = at_row_w(a.out, c, 0, row, LOGN) + i;
    uint64_t* o1 = at_row_w(a.out, c, 1, row, LOGN) + i;
    uint64_t* o2 = at_row_w(a.d2, c, 1, row, LOGN) + i;
    if (a.acc) {
        const V4 d0 = ld4(o0), d1 = ld4(o1);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            r0[w] = add_mod(r0[w], d0.v[w], p);
            r1[w] = add_mod(r1[w], d1.v[w], p);
        }
    }
    if (a.acc_d2) {
        const V4 d2 = ld4(o2);
#pragma unroll
        for (int w = 0; w < 4; ++w) r2[w] = add_mod(r2[w], d2.v[w], p);
    }
    if (a.dbl) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            r0[w] = add_mod(r0[w], r0[w], p);
            r1[w] = add_mod(r1[w], r1[w], p);
            r2[w] = add_mod(r2[w], r2[w], p);
        }
    }
    if (Y) {
        const uint64_t m = ((const uint64_t*)g.c)[row], ms = ((const uint64_t*)g.cs)[row];
        const V4 y0 = ld4(at_row(g.y, c, 0, row, LOGN) + i), y1 = ld4(at_row(g.y, c, 1, row, LOGN) + i);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const uint64_t u0 = shoup(y0.v[w], m, ms, p), u1 = shoup(y1.v[w], m, ms, p);
            r0[w] = g.sub ? sub_mod(r0[w], u0, p) : add_mod(r0[w], u0, p);
            r1[w] = g.sub ? sub_mod(r1[w], u1, p) : add_mod(r1[w], u1, p);
        }
    }
    st4(o0, r0);
    st4(o1, r1);
    st4(o2, r2);
    if (a.coef) st4((uint64_t*)a.coef + (size_t)c * a.coef_ct_stride + ((size_t)row << LOGN) + i, r2);
}

__host__ inline int tensor_check(const PcbTensorArgs& a) {
    if (a.npairs < 1 || a.npairs > 2 || a.n < 0 || a.K < 0 || !a.pr || !a.out.base || !a.d2.base || !a.a0.base ||
        !a.b0.base || (a.npairs == 2 && (!a.a1.base || !a.b1.base)))
        return PCB_BAD_ARGS;
    if (!ok16(a.out) || !ok16(a.d2) || !ok16(a.a0) || !ok16(a.b0) || (a.npairs == 2 && (!ok16(a.a1) || !ok16(a.b1))))
        return PCB_BAD_ARGS;
    return 0;
}

template <int LOGN>
int tensor_launch(const PcbTensorArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    if (const int rc = tensor_check(*ap)) return rc;
    if (ap->n == 0 || ap->K == 0) return 0;
    PcbTensorYArgs g;
    memset(&g, 0, sizeof g);
    g.t = *ap;
    tensor<LOGN, false><<<dim3((1 << LOGN) / (BX * WPT), ap->n, ap->K), BX, 0, s>>>(g);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int tensor_y_launch(const PcbTensorYArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    if (const int rc = tensor_check(ap->t)) return rc;
    if (!ap->c || !ap->cs || !ap->y.base || !ok16(ap->y)) return PCB_BAD_ARGS;
    if (ap->t.n == 0 || ap->t.K == 0) return 0;
    tensor<LOGN, true><<<dim3((1 << LOGN) / (BX * WPT), ap->t.n, ap->t.K), BX, 0, s>>>(*ap);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ md_epilogue
// parts 0, 1 of K cts over Q rows [0, n): dst = f (dst + (x - t) binv) [+ k on part 0]
template <int LOGN>
__global__ void __launch_bounds__(BX) md_epilogue(PcbMdEpiArgs a) {
    const int row = blockIdx.y, c = blockIdx.z >> 1, part = blockIdx.z & 1;
    const uint64_t p = a.pr[row].p;
    const size_t i = ((size_t)blockIdx.x * BX + threadIdx.x) * WPT;
    uint64_t* d = at_row_w(a.dst, c, part, row, LOGN) + i;
    const uint64_t bi = ((const uint64_t*)a.binv)[row], bis = ((const uint64_t*)a.binvs)[row];
    uint64_t kk = 0;
    const bool addk = a.k && part == 0;
    if (addk) {
        kk = ((const uint64_t*)a.k)[row];
        kk = kk >= p ? kk - p : kk;
    }
    const V4 x = ld4(at_row(a.x, c, part, row, LOGN) + i), t = ld4(at_row(a.t, c, part, row, LOGN) + i), dv = ld4(d);
    uint64_t r[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        r[w] = add_mod(dv.v[w], shoup(sub_mod(x.v[w], t.v[w], p), bi, bis, p), p);
        if (a.dbl) r[w] = add_mod(r[w], r[w], p);
        if (addk) r[w] = add_mod(r[w], kk, p);
    }
    st4(d, r);
}

template <int LOGN>
int md_epilogue_launch(const PcbMdEpiArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbMdEpiArgs& a = *ap;
    if (a.n < 0 || a.K < 0 || !a.pr || !a.dst.base || !a.x.base || !a.t.base || !a.binv || !a.binvs) return PCB_BAD_ARGS;
    if (!ok16(a.dst) || !ok16(a.x) || !ok16(a.t)) return PCB_BAD_ARGS;
    if (a.n == 0 || a.K == 0) return 0;
    md_epilogue<LOGN><<<dim3((1 << LOGN) / (BX * WPT), a.n, 2 * a.K), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ rescale
// Composite rescale by the top ndrop primes (crates/pc-kernels/kernels/args.cuh:530-552; crates/pc-host/src/
// rescale.rs:54-70), with lift(y, q) = the centred representative of y mod q (y > q / 2: y - q) reduced mod q_i:
//   ndrop 1: tmp_i = A_i lift(y_a)
//   ndrop 2: y' = qinv_ab y_b + C_ab lift(y_a) mod q_b, tmp_i = A_i lift(y_a) + B_i lift(y')
// y_a = x_top (times ca when ca != 1), y_b = x_(top-1) (times cb when cb != 1), coefficient form.
// two consecutive words per thread, one row per grid row (the top words are re-read per row from L2)
__device__ __forceinline__ uint64_t red_word(uint64_t y, const PcbPrimeConst& pq) {
    const uint64_t q = pq.p;
    return y < q ? y : (y < 2 * q ? y - q : reduce(Acc{y, 0}, pq));
}
// lift(y mod qo) mod the prime of pq; qom = qo mod that prime
__device__ __forceinline__ uint64_t lift_word(uint64_t y, uint64_t qo, uint64_t qom, const PcbPrimeConst& pq) {
    const uint64_t l = red_word(y, pq);
    return y > (qo >> 1) ? sub_mod(l, qom, pq.p) : l;
}

template <int LOGN>
__global__ void __launch_bounds__(BX) rescale_coef(PcbRescaleArgs a) {
    const int c = blockIdx.z >> 1, part = blockIdx.z & 1, row = blockIdx.y;
    const size_t i = ((size_t)blockIdx.x * BX + threadIdx.x) * 2;
    const PcbPrimeConst& pa = a.pr[a.top];
    const uint64_t qa = pa.p;
    const ulonglong2 yv = *(const ulonglong2*)(at_row(a.x, c, part, a.top, LOGN) + i);
    uint64_t ya[2] = {yv.x, yv.y}, yp[2] = {0, 0}, qb = 0;
    if (a.ca != 1) {
        ya[0] = mul_mod(ya[0], a.ca, pa);
        ya[1] = mul_mod(ya[1], a.ca, pa);
    }
    if (a.ndrop == 2) {
        const PcbPrimeConst& pb = a.pr[a.top - 1];
        qb = pb.p;
        const uint64_t qab = red_word(qa, pb);
        const ulonglong2 bv = *(const ulonglong2*)(at_row(a.x, c, part, a.top - 1, LOGN) + i);
        const uint64_t yb[2] = {bv.x, bv.y};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint64_t b = a.cb != 1 ? mul_mod(yb[h], a.cb, pb) : yb[h];
            yp[h] = add_mod(mul_mod(a.qinv_ab, b, pb), mul_mod(a.C_ab, lift_word(ya[h], qa, qab, pb), pb), qb);
        }
    }
    const PcbPrimeConst& pq = a.pr[row];
    const uint64_t q = pq.p;
    const uint64_t A = ((const uint64_t*)a.A)[row], As = ((const uint64_t*)a.As)[row];
    const uint64_t qm = ((const uint64_t*)a.qam)[row];
    uint64_t r[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        r[h] = shoup(lift_word(ya[h], qa, qm, pq), A, As, q);
        if (a.ndrop == 2) {
            const uint64_t B = ((const uint64_t*)a.B)[row], Bs = ((const uint64_t*)a.Bs)[row];
            const uint64_t qbm = ((const uint64_t*)a.qbm)[row];
            r[h] = add_mod(r[h], shoup(lift_word(yp[h], qb, qbm, pq), B, Bs, q), q);
        }
    }
    *(ulonglong2*)(at_row_w(a.tmp, c, part, row, LOGN) + i) = make_ulonglong2(r[0], r[1]);
}

template <int LOGN>
int rescale_coef_launch(const PcbRescaleArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbRescaleArgs& a = *ap;
    if (a.ndrop != 1 && a.ndrop != 2) return PCB_BAD_ARGS;
    if (a.top < a.ndrop || a.nrows < 0 || a.K < 0 || !a.pr || !a.x.base || !a.tmp.base || !a.A || !a.As || !a.qam)
        return PCB_BAD_ARGS;
    if (a.ndrop == 2 && (!a.B || !a.Bs || !a.qbm)) return PCB_BAD_ARGS;
    if (!ok16(a.x) || !ok16(a.tmp)) return PCB_BAD_ARGS;
    if (a.nrows == 0 || a.K == 0) return 0;
    rescale_coef<LOGN><<<dim3((1 << LOGN) / (BX * 2), a.nrows, 2 * a.K), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ ModRaise
// args.cuh:665-677: rows t in [r0, r1) of K ciphertexts (nparts parts), one output word per thread:
// x[t] = sum_{k < d} lift_k([x_k qhatinv_k]_{q_k}) qhat[k][t] mod q_t, lift_k = the centred representative mod q_k
template <int LOGN>
__global__ void __launch_bounds__(BX) mod_raise(PcbModRaiseArgs a) {
    const int c = blockIdx.z / a.nparts, part = blockIdx.z % a.nparts;
    const int t = a.r0 + blockIdx.y;
    const size_t i = (size_t)blockIdx.x * BX + threadIdx.x;
    uint64_t* x = (uint64_t*)a.x + (size_t)c * a.ct_stride + (size_t)part * a.part_stride;
    const PcbPrimeConst& pt = a.pr[t];
    const uint64_t qt = pt.p;
    uint64_t acc = 0;
    for (int k = 0; k < a.d; ++k) {
        const PcbPrimeConst& pk = a.pr[k];
        const uint64_t y = mul_mod(x[((size_t)k << LOGN) + i], a.qhatinv[k], pk);
        const uint64_t r = lift_word(y, pk.p, red_word(pk.p, pt), pt);
        acc = add_mod(acc, mul_mod(r, a.qhat[k][t], pt), qt);
    }
    x[((size_t)t << LOGN) + i] = acc;
}

template <int LOGN>
int mod_raise_launch(const PcbModRaiseArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbModRaiseArgs& a = *ap;
    if (!a.x || !a.pr || a.d < 1 || a.d > 4 || a.r0 < a.d || a.r1 > 64 || a.r1 < a.r0 || a.K < 0 || a.nparts < 1 ||
        a.nparts > 2)
        return PCB_BAD_ARGS;
    if (a.K == 0 || a.r1 == a.r0) return 0;
    mod_raise<LOGN><<<dim3((1 << LOGN) / BX, a.r1 - a.r0, a.K * a.nparts), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// args.cuh:892-907 (small_int1): the raise of a one-prime source with an exact scaling folded in. The centred
// value x of row 0 times the scale mc 2^-sh is rounded half up in 128-bit integers (|x| < 2^63, mc < 2^64: the
// product and the half fit), and its sign put back on the residue of every row.
template <int LOGN>
__global__ void __launch_bounds__(BX) small_int1(PcbSmallInt1Args a) {
    const size_t i = (size_t)blockIdx.x * BX + threadIdx.x;
    uint64_t* x = (uint64_t*)a.x + (size_t)blockIdx.z * a.ct_stride + (size_t)blockIdx.y * a.part_stride;
    const uint64_t q0 = a.pr[0].p;
    const uint64_t v = x[i];
    const bool neg = v > q0 / 2;
    const uint64_t mag = neg ? q0 - v : v;
    uint64_t lo = mag * a.mc, hi = __umul64hi(mag, a.mc);
    if (a.sh <= 64) {
        const uint64_t h = 1ull << (a.sh - 1);
        lo += h;
        hi += lo < h;
    } else {
        hi += 1ull << (a.sh - 65);
    }
    const uint64_t q = a.sh < 64 ? (lo >> a.sh) | (hi << (64 - a.sh)) : hi >> (a.sh - 64);
    for (int t = 0; t < a.nrows; ++t) {
        const PcbPrimeConst& pt = a.pr[t];
        const uint64_t r = reduce(Acc{q, 0}, pt);
        x[((size_t)t << LOGN) + i] = neg && r ? pt.p - r : r;
    }
}

template <int LOGN>
int small_int1_launch(const PcbSmallInt1Args* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbSmallInt1Args& a = *ap;
    if (!a.x || !a.pr || a.sh < 1 || a.sh > 127 || a.nrows < 1 || a.nrows > 64 || a.K < 0 || a.nparts < 1 ||
        a.nparts > 2)
        return PCB_BAD_ARGS;
    if (a.K == 0) return 0;
    small_int1<LOGN><<<dim3((1 << LOGN) / BX, a.nparts, a.K), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
__global__ void __launch_bounds__(BX) rescale_combine(PcbRescaleCombineArgs a) {
    const int row = blockIdx.y, c = blockIdx.z >> 1, part = blockIdx.z & 1;
    const uint64_t p = a.pr[row].p;
    const size_t i = ((size_t)blockIdx.x * BX + threadIdx.x) * WPT;
    uint64_t* d = at_row_w(a.x, c, part, row, LOGN) + i;
    const uint64_t al = ((const uint64_t*)a.alpha)[row], als = ((const uint64_t*)a.alphas)[row];
    const V4 x = ld4(d), t = ld4(at_row(a.tmp, c, part, row, LOGN) + i);
    uint64_t r[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) r[w] = add_mod(shoup(x.v[w], al, als, p), t.v[w], p);
    st4(d, r);
}

template <int LOGN>
int rescale_combine_launch(const PcbRescaleCombineArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbRescaleCombineArgs& a = *ap;
    if (a.n < 0 || a.K < 0 || !a.pr || !a.x.base || !a.tmp.base || !a.alpha || !a.alphas) return PCB_BAD_ARGS;
    if (!ok16(a.x) || !ok16(a.tmp)) return PCB_BAD_ARGS;
    if (a.n == 0 || a.K == 0) return 0;
    rescale_combine<LOGN><<<dim3((1 << LOGN) / (BX * WPT), a.n, 2 * a.K), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ automorph
// out[o] = in[automorph_slot(k, o)] (+ add[o]): aligned 32-slot runs of o map to aligned 32-slot runs of the source,
// so the gather stays sector-coalesced
template <int LOGN, bool ADD>
__global__ void __launch_bounds__(BX) automorph(PcbAutomorphArgs a) {
    const int row = rs_row(a.rs, blockIdx.y);
    const int c = blockIdx.z / a.nparts, part = blockIdx.z % a.nparts;
    const uint32_t o = blockIdx.x * BX + threadIdx.x;
    uint64_t v = at_row(a.in, c, part, row, LOGN)[automorph_slot<LOGN>(a.k, o)];
    if (ADD) v = add_mod(v, at_row(a.add, c, part, row, LOGN)[o], a.pr[row].p);
    at_row_w(a.out, c, part, row, LOGN)[o] = v;
}

template <int LOGN>
int automorph_launch(const PcbAutomorphArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbAutomorphArgs& a = *ap;
    if ((a.k & 1u) == 0 || a.K < 0 || a.nparts < 1 || !a.out.base || !a.in.base || (a.has_add && (!a.add.base || !a.pr)))
        return PCB_BAD_ARGS;
    const int rows = a.rs.nq + a.rs.np;
    if (rows == 0 || a.K == 0) return 0;
    const dim3 g((1 << LOGN) / BX, rows, a.K * a.nparts);
    if (a.has_add) automorph<LOGN, true><<<g, BX, 0, s>>>(a);
    else automorph<LOGN, false><<<g, BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ sum
// one pass over n inputs (each read once) instead of n - 1 pairwise adds; out may be one of the inputs
template <int LOGN>
__global__ void __launch_bounds__(BX) sum_cts(SumArgs a) {
    const int row = blockIdx.y, c = blockIdx.z >> 1, part = blockIdx.z & 1;
    const size_t off = (size_t)c * a.ct_stride + (size_t)part * a.part_stride + ((size_t)row << LOGN) +
                       ((size_t)blockIdx.x * BX + threadIdx.x) * WPT;
    const uint64_t p = a.pr[row].p;
    V4 acc = ld4(a.in[0] + off);
    for (int m = 1; m < a.n; ++m) {
        const V4 x = ld4(a.in[m] + off);
#pragma unroll
        for (int w = 0; w < 4; ++w) acc.v[w] = add_mod(acc.v[w], x.v[w], p);
    }
    uint64_t r[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) r[w] = acc.v[w];
    st4(a.out + off, r);
}

template <int LOGN>
int sum_launch(const SumArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const SumArgs& a = *ap;
    if (a.n < 1 || a.n > SUM_MAX || a.nrows < 0 || a.K < 0 || !a.out || !a.pr) return PCB_BAD_ARGS;
    if (((uintptr_t)a.out & 15) || (a.ct_stride & 1) || (a.part_stride & 1)) return PCB_BAD_ARGS;
    for (int m = 0; m < a.n; ++m)
        if (!a.in[m] || ((uintptr_t)a.in[m] & 15)) return PCB_BAD_ARGS;
    if (a.nrows == 0 || a.K == 0) return 0;
    sum_cts<LOGN><<<dim3((1 << LOGN) / (BX * WPT), a.nrows, 2 * a.K), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

#define PCB_INST(L)                                                                                  \
    template int sum_launch<L>(const SumArgs*, cudaStream_t);                                        \
    template int ew_launch<L, EW_ADD>(const PcbEwArgs*, cudaStream_t);                               \
    template int ew_launch<L, EW_SCALE>(const PcbEwArgs*, cudaStream_t);                             \
    template int ew_launch<L, EW_SUB_MUL>(const PcbEwArgs*, cudaStream_t);                           \
    template int ew_launch<L, EW_COPY>(const PcbEwArgs*, cudaStream_t);                              \
    template int tensor_launch<L>(const PcbTensorArgs*, cudaStream_t);                               \
    template int tensor_y_launch<L>(const PcbTensorYArgs*, cudaStream_t);                            \
    template int md_epilogue_launch<L>(const PcbMdEpiArgs*, cudaStream_t);                           \
    template int rescale_coef_launch<L>(const PcbRescaleArgs*, cudaStream_t);                        \
    template int mod_raise_launch<L>(const PcbModRaiseArgs*, cudaStream_t);                          \
    template int small_int1_launch<L>(const PcbSmallInt1Args*, cudaStream_t);                       \
    template int rescale_combine_launch<L>(const PcbRescaleCombineArgs*, cudaStream_t);              \
    template int automorph_launch<L>(const PcbAutomorphArgs*, cudaStream_t);
PCB_INST(14)
PCB_INST(16)

}  // namespace elem
}  // namespace pcb
