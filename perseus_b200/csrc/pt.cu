// Plaintext-operand kernels of the linear layers: pt_dot (the BSGS baby-step dot), mul_table (ct x pt), mul_add
// (y +- ct x pt in one pass), mul_add_n (a chain of ct x pt products summed in one pass) and add_const. Semantics
// of crates/pc-kernels/kernels/args.cuh (PtDotArgs :184-200, AddConstArgs / MulTableArgs / MulAddArgs /
// MulAddNArgs :491-528); host twin crates/pc-host/src/elem.rs:145-180. coeff_sum (the streamed-weight inner sum,
// CoeffArgs :909-927; caller crates/pc-gpu/src/encode_dev.rs) closes the file.
//
// All five are HBM streams over residue rows: no reuse inside a thread beyond the pt_dot sums, so the design is about
// bytes. Sums of products are kept in 128-bit accumulators and reduced once (the Barrett reduction of arith.cuh is
// exact for any 128-bit value), so every output is the canonical residue of the exact integer sum, whatever the
// summation order: the outputs equal the reference's word for word.
#include "arith.cuh"
#include "kernels.h"

namespace pcb {
namespace pt {

constexpr int BX = 256;  // element-wise kernels: 4 words per thread
constexpr int WPT = 4;
constexpr int DOT_BX = 128;  // pt_dot

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
// a read-only row of the plaintext table t ([row][N] words)
__device__ __forceinline__ V4 ld4_ro(const uint64_t* p) {
    const ulonglong2 a = __ldg((const ulonglong2*)p), b = __ldg((const ulonglong2*)p + 1);
    return V4{{a.x, a.y, b.x, b.y}};
}

__host__ inline bool ok16(const PcbPolyRef& r) {
    return ((uintptr_t)r.base & 15) == 0 && (r.ct_stride & 1) == 0 && (r.part_stride & 1) == 0;
}

// ------------------------------------------------------------------------------------------------ add_const
// part 0 += k[row]; k may equal p (args.cuh:491-498: the raw word is reduced once)
template <int LOGN>
__global__ void __launch_bounds__(BX) add_const(PcbAddConstArgs a) {
    const int row = blockIdx.y, c = blockIdx.z;
    const uint64_t p = a.pr[row].p;
    const uint64_t k0 = ((const uint64_t*)a.k)[row], k = k0 >= p ? k0 - p : k0;
    uint64_t* d = at_row_w(a.x, c, 0, row, LOGN) + ((size_t)blockIdx.x * BX + threadIdx.x) * WPT;
    const V4 x = ld4(d);
    uint64_t r[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) r[w] = add_mod(x.v[w], k, p);
    st4(d, r);
}

template <int LOGN>
int add_const_launch(const PcbAddConstArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbAddConstArgs& a = *ap;
    if (a.n < 0 || a.K < 0 || !a.x.base || !a.k || !a.pr || !ok16(a.x)) return PCB_BAD_ARGS;
    if (a.n == 0 || a.K == 0) return 0;
    add_const<LOGN><<<dim3((1 << LOGN) / (BX * WPT), a.n, a.K), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ mul_table / mul_add
// MODE 0: out = in t; 1: out = y + in t; 2: y - in t; 3: in t - y (the MulAddArgs sub codes 0, 1, 2 shifted by one)
template <int LOGN, int MODE>
__global__ void __launch_bounds__(BX) mul_table(PcbMulTableArgs m, PcbPolyRef y) {
    const int row = blockIdx.y, c = blockIdx.z >> 1, part = blockIdx.z & 1;
    const PcbPrimeConst& pc = m.pr[row];
    const size_t i = ((size_t)blockIdx.x * BX + threadIdx.x) * WPT;
    const V4 x = ld4(at_row(m.in, c, part, row, LOGN) + i);
    const V4 t = ld4_ro((const uint64_t*)m.t + ((size_t)row << LOGN) + i);
    uint64_t r[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) r[w] = mul_mod(x.v[w], t.v[w], pc);
    if (MODE != 0) {
        const V4 yv = ld4(at_row(y, c, part, row, LOGN) + i);
#pragma unroll
        for (int w = 0; w < 4; ++w)
            r[w] = MODE == 1 ? add_mod(yv.v[w], r[w], pc.p)
                 : MODE == 2 ? sub_mod(yv.v[w], r[w], pc.p)
                             : sub_mod(r[w], yv.v[w], pc.p);
    }
    st4(at_row_w(m.out, c, part, row, LOGN) + i, r);
}

__host__ inline bool mul_table_ok(const PcbMulTableArgs& m) {
    return m.n >= 0 && m.K >= 0 && m.out.base && m.in.base && m.t && m.pr && ok16(m.out) && ok16(m.in) &&
           ((uintptr_t)m.t & 15) == 0;
}

template <int LOGN>
int mul_table_launch(const PcbMulTableArgs* ap, cudaStream_t s) {
    if (!ap || !mul_table_ok(*ap)) return PCB_BAD_ARGS;
    if (ap->n == 0 || ap->K == 0) return 0;
    mul_table<LOGN, 0><<<dim3((1 << LOGN) / (BX * WPT), ap->n, 2 * ap->K), BX, 0, s>>>(*ap, PcbPolyRef{});
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int mul_add_launch(const PcbMulAddArgs* ap, cudaStream_t s) {
    if (!ap || !mul_table_ok(ap->m) || ap->sub < 0 || ap->sub > 2 || !ap->y.base || !ok16(ap->y)) return PCB_BAD_ARGS;
    const PcbMulTableArgs& m = ap->m;
    if (m.n == 0 || m.K == 0) return 0;
    const dim3 g((1 << LOGN) / (BX * WPT), m.n, 2 * m.K);
    if (ap->sub == 0) mul_table<LOGN, 1><<<g, BX, 0, s>>>(m, ap->y);
    else if (ap->sub == 1) mul_table<LOGN, 2><<<g, BX, 0, s>>>(m, ap->y);
    else mul_table<LOGN, 3><<<g, BX, 0, s>>>(m, ap->y);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ mul_add_n
// out = y + sum_j x_j t_j: the nterm <= 8 products summed in 128 bits (8 (2^62)^2 = 2^127) and reduced once. The
// reference's lazy = 0 reduces each product and adds mod p: for canonical operands both give the canonical residue
// of the same integer sum, so one code path serves both flags.
template <int LOGN>
__global__ void __launch_bounds__(BX) mul_add_n(PcbMulAddNArgs a) {
    const int row = blockIdx.y, c = blockIdx.z >> 1, part = blockIdx.z & 1;
    const PcbPrimeConst& pc = a.pr[row];
    const size_t i = ((size_t)blockIdx.x * BX + threadIdx.x) * WPT;
    Acc s[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) s[w] = Acc{0, 0};
    for (int j = 0; j < a.nterm; ++j) {
        const V4 x = ld4(at_row(a.x[j], c, part, row, LOGN) + i);
        const V4 t = ld4_ro((const uint64_t*)a.t[j] + ((size_t)row << LOGN) + i);
#pragma unroll
        for (int w = 0; w < 4; ++w) mac(s[w], x.v[w], t.v[w]);
    }
    uint64_t r[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) r[w] = reduce(s[w], pc);
    if (a.y.base) {
        const V4 yv = ld4(at_row(a.y, c, part, row, LOGN) + i);
#pragma unroll
        for (int w = 0; w < 4; ++w) r[w] = add_mod(yv.v[w], r[w], pc.p);
    }
    st4(at_row_w(a.out, c, part, row, LOGN) + i, r);
}

template <int LOGN>
int mul_add_n_launch(const PcbMulAddNArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbMulAddNArgs& a = *ap;
    if (a.nterm < 1 || a.nterm > 8 || a.n < 0 || a.K < 0 || !a.out.base || !a.pr || !ok16(a.out)) return PCB_BAD_ARGS;
    if (a.y.base && !ok16(a.y)) return PCB_BAD_ARGS;
    for (int j = 0; j < a.nterm; ++j)
        if (!a.x[j].base || !ok16(a.x[j]) || !a.t[j] || ((uintptr_t)a.t[j] & 15)) return PCB_BAD_ARGS;
    if (a.n == 0 || a.K == 0) return 0;
    mul_add_n<LOGN><<<dim3((1 << LOGN) / (BX * WPT), a.n, 2 * a.K), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ pt_dot
template <int W>
struct Words {
    uint64_t v[W];
};
template <int W>
__device__ __forceinline__ Words<W> ldw(const uint64_t* p) {
    Words<W> r;
    if constexpr (W == 1) {
        r.v[0] = p[0];
    } else {
#pragma unroll
        for (int h = 0; h < W / 2; ++h) {
            const ulonglong2 q = ((const ulonglong2*)p)[h];
            r.v[2 * h] = q.x;
            r.v[2 * h + 1] = q.y;
        }
    }
    return r;
}
template <int W>
__device__ __forceinline__ void stw(uint64_t* p, const uint64_t (&r)[W]) {
    if constexpr (W == 1) {
        p[0] = r[0];
    } else {
#pragma unroll
        for (int h = 0; h < W / 2; ++h) ((ulonglong2*)p)[h] = make_ulonglong2(r[2 * h], r[2 * h + 1]);
    }
}

// One block = DOT_BX x WPT consecutive words of one row for ONE giant step j. The giant step is the fastest-varying
// block index, so the gstep blocks that read the same baby-rotation slice run next to each other and all but the
// first find it in L2: HBM sees the rotations once, the plaintexts once and the results once. Per thread KMAX x 2
// parts x WPT 128-bit sums (KMAX WPT = 8 at most: 64 registers of sums).
template <int LOGN, int KMAX, int WPT_>
__global__ void __launch_bounds__(DOT_BX) pt_dot(PcbPtDotArgs a) {
    const int j = blockIdx.x % a.gstep;
    const uint32_t chunk = blockIdx.x / a.gstep;
    const int y = blockIdx.y;
    const int row = rs_row(a.rs, y);
    const size_t prow = y < a.rs.nq ? y : a.pt_prow + (y - a.rs.nq);
    const PcbPrimeConst& pc = a.pr[row];
    const uint32_t i0 = (chunk * DOT_BX + threadIdx.x) * WPT_;
    uint32_t pi[WPT_];
#pragma unroll
    for (int u = 0; u < WPT_; ++u) pi[u] = pt_index(i0 + u, a.enc);
    Acc s0[KMAX][WPT_], s1[KMAX][WPT_];
#pragma unroll
    for (int c = 0; c < KMAX; ++c)
#pragma unroll
        for (int u = 0; u < WPT_; ++u) s0[c][u] = s1[c][u] = Acc{0, 0};
    const uint64_t* rbase = (const uint64_t*)a.rot.base + ((size_t)row << LOGN) + i0;
    for (int b = 0; b < a.bstep; ++b) {
        const int d = a.bstep * j + b;
        if (d >= a.npts) break;
        const uint64_t* ptrow = (const uint64_t*)a.pts[d] + prow * (size_t)a.ptw;
        uint64_t w[WPT_];
#pragma unroll
        for (int u = 0; u < WPT_; ++u) w[u] = __ldg(ptrow + pi[u]);
#pragma unroll
        for (int c = 0; c < KMAX; ++c) {
            if (c < a.K) {
                const uint64_t* r0 = rbase + (size_t)c * a.rot.ct_stride + (size_t)b * a.rot_stride;
                const Words<WPT_> x0 = ldw<WPT_>(r0), x1 = ldw<WPT_>(r0 + a.rot.part_stride);
#pragma unroll
                for (int u = 0; u < WPT_; ++u) {
                    mac(s0[c][u], x0.v[u], w[u]);
                    mac(s1[c][u], x1.v[u], w[u]);
                }
            }
        }
    }
#pragma unroll
    for (int c = 0; c < KMAX; ++c) {
        if (c < a.K) {
            uint64_t* o = (uint64_t*)a.res.base + (size_t)c * a.res.ct_stride + (size_t)j * a.res_stride +
                          ((size_t)row << LOGN) + i0;
            uint64_t r0[WPT_], r1[WPT_];
#pragma unroll
            for (int u = 0; u < WPT_; ++u) {
                r0[u] = reduce(s0[c][u], pc);
                r1[u] = reduce(s1[c][u], pc);
            }
            stw<WPT_>(o, r0);
            stw<WPT_>(o + a.res.part_stride, r1);
        }
    }
}

template <int LOGN, int KMAX>
int pt_dot_go(const PcbPtDotArgs& a, cudaStream_t s) {
    constexpr int W = KMAX >= 8 ? 1 : KMAX >= 4 ? 2 : 4;
    const int rows = a.rs.nq + a.rs.np;
    const long long bx = (long long)((1 << LOGN) / (DOT_BX * W)) * a.gstep;
    if (bx > 0x7FFFFFFFll) return PCB_BAD_ARGS;
    pt_dot<LOGN, KMAX, W><<<dim3((unsigned)bx, rows), DOT_BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int pt_dot_launch(const PcbPtDotArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbPtDotArgs& a = *ap;
    // 128-bit sums of bstep products below 2^120 (primes up to 60 bits): at most 256 baby steps
    if (a.K < 1 || a.K > 8 || a.bstep < 0 || a.bstep > 256 || a.gstep < 0 || a.npts < 0 || a.ptw < 0 || a.pt_prow < 0)
        return PCB_BAD_ARGS;
    if (a.rs.nq < 0 || a.rs.np < 0 || (a.rs.np > 0 && a.rs.qmax < a.rs.nq)) return PCB_BAD_ARGS;
    if (!a.rot.base || !a.res.base || !a.pr || (a.npts > 0 && !a.pts)) return PCB_BAD_ARGS;
    // the vector paths move 2 or 4 words: row starts 16-byte aligned (K = 8 moves one word and needs no check)
    if (a.K < 5 && (!ok16(a.rot) || !ok16(a.res) || (a.rot_stride & 1) || (a.res_stride & 1))) return PCB_BAD_ARGS;
    if (a.rs.nq + a.rs.np == 0 || a.gstep == 0) return 0;
    return a.K <= 1 ? pt_dot_go<LOGN, 1>(a, s)
         : a.K <= 2 ? pt_dot_go<LOGN, 2>(a, s)
         : a.K <= 4 ? pt_dot_go<LOGN, 4>(a, s)
                    : pt_dot_go<LOGN, 8>(a, s);
}

// ------------------------------------------------------------------------------------------------ coeff_sum
// args.cuh:909-927: out (+)= sum_{r < n} ct_r pt_r over Q limbs 0..L-1, with pt_r[k] = round(rows_r[k] scale) mod p_l
// (round half to even; a value past the int64 range clamped to +-2^62 and counted once per limb in *overflow) taken
// to the NTT domain by the forward transform of the launcher table's twiddles. The plaintext is never stored as an
// object: its float32 row (the weight as streamed from the host) is expanded into the caller's scratch
// [term][limb][N], transformed in place, and consumed by one multiply-accumulate pass over all terms (128-bit sums,
// folded every 8 terms: 8 products below 2^124 and a residue stay below 2^128).
__device__ const uint32_t g_limb_ident[PCB_COEFF_MAXL] = {
    0,  1,  2,  3,  4,  5,  6,  7,  8,  9,  10, 11, 12, 13, 14, 15, 16, 17, 18, 19, 20, 21,
    22, 23, 24, 25, 26, 27, 28, 29, 30, 31, 32, 33, 34, 35, 36, 37, 38, 39, 40, 41, 42, 43,
    44, 45, 46, 47, 48, 49, 50, 51, 52, 53, 54, 55, 56, 57, 58, 59, 60, 61, 62, 63};

__device__ __forceinline__ uint64_t coeff_residue(float f, double scale, const PcbPrimeConst& pc,
                                                  unsigned long long* ovf) {
    const double x = (double)f * scale;
    long long m;
    if (fabs(x) < 9.2e18) {
        m = __double2ll_rn(x);
    } else {  // past the int64 range, or not a number
        m = x < 0 ? -(1ll << 62) : (1ll << 62);
        if (ovf) atomicAdd(ovf, 1ull);
    }
    const uint64_t mag = m < 0 ? (uint64_t)(-m) : (uint64_t)m;
    const uint64_t v = reduce(Acc{mag, 0}, pc);
    return m < 0 && v ? pc.p - v : v;
}

// grid (N / (BX WPT), L, n): scratch[r][l][k] = the residue of coefficient k of row r mod p_l
template <int LOGN>
__global__ void __launch_bounds__(BX) coeff_expand(PcbCoeffArgs a) {
    const int l = blockIdx.y, r = blockIdx.z;
    const PcbPrimeConst& pc = a.pr[l];
    const size_t i = ((size_t)blockIdx.x * BX + threadIdx.x) * WPT;
    const float4 f = *(const float4*)(a.rows[r] + i);
    const uint64_t w[4] = {coeff_residue(f.x, a.scale, pc, a.overflow), coeff_residue(f.y, a.scale, pc, a.overflow),
                           coeff_residue(f.z, a.scale, pc, a.overflow), coeff_residue(f.w, a.scale, pc, a.overflow)};
    st4((uint64_t*)a.scratch + (((size_t)r * a.L + l) << LOGN) + i, w);
}

// grid (N / (BX WPT), L, 2 parts): out[part][l] (+)= sum_r ct_r[part][l] pt_r[l]
template <int LOGN>
__global__ void __launch_bounds__(BX) coeff_mac(PcbCoeffArgs a) {
    const int l = blockIdx.y, part = blockIdx.z;
    const PcbPrimeConst& pc = a.pr[l];
    const uint64_t p = pc.p;
    const size_t i = ((size_t)blockIdx.x * BX + threadIdx.x) * WPT;
    const size_t row = (size_t)part * a.part_stride + ((size_t)l << LOGN) + i;
    Acc acc[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) acc[w] = Acc{0, 0};
    for (int r = 0; r < a.n; ++r) {
        const V4 x = ld4((const uint64_t*)a.ct[r] + row);
        const V4 y = ld4((const uint64_t*)a.scratch + (((size_t)r * a.L + l) << LOGN) + i);
#pragma unroll
        for (int w = 0; w < 4; ++w) mac(acc[w], x.v[w], y.v[w]);
        if ((r & 7) == 7) {
#pragma unroll
            for (int w = 0; w < 4; ++w) acc[w] = Acc{reduce(acc[w], pc), 0};
        }
    }
    uint64_t* o = (uint64_t*)a.out + row;
    uint64_t res[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) res[w] = reduce(acc[w], pc);
    if (a.accumulate) {
        const V4 d = ld4(o);
#pragma unroll
        for (int w = 0; w < 4; ++w) res[w] = add_mod(res[w], d.v[w], p);
    }
    st4(o, res);
}

template <int LOGN>
int coeff_sum_launch(const PcbCoeffArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbCoeffArgs& a = *ap;
    if (a.n < 1 || a.n > PCB_COEFF_MAXT || a.L < 1 || a.L > PCB_COEFF_MAXL || !a.scratch || !a.out || !a.fw || !a.fws ||
        !a.pr)
        return PCB_BAD_ARGS;
    const auto a16 = [](const void* q) { return ((uintptr_t)q & 15) == 0; };
    if (!a16(a.scratch) || !a16(a.out) || (a.part_stride & 1)) return PCB_BAD_ARGS;
    for (int r = 0; r < a.n; ++r)
        if (!a.rows[r] || !a.ct[r] || !a16(a.rows[r]) || !a16(a.ct[r])) return PCB_BAD_ARGS;
    const uint32_t* ident = nullptr;
    if (cudaGetSymbolAddress((void**)&ident, g_limb_ident) != cudaSuccess) return PCB_LAUNCH_RESULT();
    coeff_expand<LOGN><<<dim3((1 << LOGN) / (BX * WPT), a.L, a.n), BX, 0, s>>>(a);
    int rc = PCB_LAUNCH_RESULT();
    for (int r = 0; r < a.n && rc == 0; ++r) {
        PcbNttArgs na;
        memset(&na, 0, sizeof na);
        na.base = (uint64_t*)a.scratch + (((size_t)r * a.L) << LOGN);
        na.roff = ident;
        na.rprime = (const int32_t*)ident;
        na.fw = a.fw;
        na.fws = a.fws;
        na.pr = a.pr;
        na.nrows = a.L;
        na.snum = 1;
        na.xnum = 1;
        rc = ntt::fwd<LOGN>(&na, s);
    }
    if (rc) return rc;
    coeff_mac<LOGN><<<dim3((1 << LOGN) / (BX * WPT), a.L, 2), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

#define PCB_PT_INST(L)                                                      \
    template int coeff_sum_launch<L>(const PcbCoeffArgs*, cudaStream_t);   \
    template int add_const_launch<L>(const PcbAddConstArgs*, cudaStream_t); \
    template int mul_table_launch<L>(const PcbMulTableArgs*, cudaStream_t); \
    template int mul_add_launch<L>(const PcbMulAddArgs*, cudaStream_t);     \
    template int mul_add_n_launch<L>(const PcbMulAddNArgs*, cudaStream_t);  \
    template int pt_dot_launch<L>(const PcbPtDotArgs*, cudaStream_t);
PCB_PT_INST(14)
PCB_PT_INST(16)

}  // namespace pt
}  // namespace pcb
