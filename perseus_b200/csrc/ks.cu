// Key-switching kernels behind the launcher table: the batched fast base conversion (bconv) and the key inner
// product (ks_dot). Semantics: crates/pc-kernels/kernels/args.cuh:109-141 (BconvArgs) and :202-228 (KsArgs); host
// twins crates/pc-host/src/bconv.rs:13-108 and crates/pc-host/src/ks.rs:60-140.
//
// Both are multiply-accumulate streams over 64-bit residues, each output reduced once. Two accumulator forms:
//  - general (any prime < 2^62): a 128-bit accumulator fed by mad.lo.cc / madc.hi;
//  - narrow (every residue and constant < 2^52, the 50-bit chains): operands split at bit 26 into 26-bit halves, and
//    three 64-bit partial sums (hi x hi, the two cross products, lo x lo) fed by one 32 x 32 + 64 IMAD.WIDE each —
//    four integer multiply-adds per product and no carry chain; up to 2^12 products fit before any partial sum could
//    overflow. The table's launchers use the general form; the evaluator picks the narrow one when its chain allows.
// The conversion matrix of a job and its target primes' Barrett constants sit in shared memory; source words stay in
// registers across all targets.
#include "arith.cuh"
#include "keyregen.cuh"
#include "kernels.h"

namespace pcb {
namespace ks {

constexpr int BX = 128;
constexpr int MAX_SRC = 16;
constexpr int MAX_TGT = 64;
constexpr uint64_t LO26 = (1ull << 26) - 1;

// Three-part accumulator of 26-bit-split products: value = H 2^52 + M 2^26 + L
struct Acc3 {
    uint64_t h, m, l;
};
// 32 x 32 -> 64 multiply with a 64-bit addend in one instruction (mad.wide.u32)
__device__ __forceinline__ uint64_t madw(uint32_t x, uint32_t y, uint64_t acc) {
    uint64_t r;
    asm("mad.wide.u32 %0, %1, %2, %3;" : "=l"(r) : "r"(x), "r"(y), "l"(acc));
    return r;
}
__device__ __forceinline__ void mac3(Acc3& a, uint32_t x1, uint32_t x0, uint32_t y1, uint32_t y0) {
    a.h = madw(x1, y1, a.h);
    a.m = madw(x1, y0, a.m);
    a.m = madw(x0, y1, a.m);
    a.l = madw(x0, y0, a.l);
}
__device__ __forceinline__ Acc to_acc(const Acc3& a) {
    const uint64_t t = a.m << 26;
    uint64_t lo = a.l + t;
    uint64_t hi = (a.m >> 38) + (lo < t);
    const uint64_t u = a.h << 52;
    lo += u;
    hi += (a.h >> 12) + (lo < u);
    return Acc{lo, hi};
}

// ------------------------------------------------------------------------------------------------ bconv
// NS > 0: every job of the launch has exactly NS sources (the source loops unroll without guards); 0: any count.
template <int LOGN, bool NARROW, int NS>
__global__ void __launch_bounds__(BX) bconv(PcbBconvArgs a) {
    constexpr int S = NS > 0 ? NS : MAX_SRC;
    __shared__ uint64_t sM[MAX_SRC * MAX_TGT];
    __shared__ uint64_t sP[MAX_TGT], sM0[MAX_TGT], sM1[MAX_TGT];
    __shared__ uint32_t sRow[MAX_TGT];
    const PcbBconvJob j = a.jobs[blockIdx.y];
    const uint64_t* pool = (const uint64_t*)a.pool + j.pool_off;
    const int ns = NS > 0 ? NS : (int)j.nsrc, nt = (int)j.ntgt;
    // outside the kernel's job shape: nothing is written
    if (ns < 1 || ns > MAX_SRC || nt > MAX_TGT || (int)j.nsrc != ns) return;
    const uint64_t* srow = pool;
    const uint64_t* sprime = pool + ns;
    const uint64_t* pre = pool + 2 * ns;
    const uint64_t* trow = pool + 3 * ns;
    const uint64_t* tprime = pool + 3 * ns + nt;
    const uint64_t* M = pool + 3 * ns + 2 * nt;
    for (int e = threadIdx.x; e < ns * nt; e += BX) {
        const uint64_t v = M[e];
        // narrow: the two 26-bit halves packed as (hi << 32) | lo for one 8-byte shared load
        sM[e] = NARROW ? ((v >> 26) << 32) | (v & LO26) : v;
    }
    for (int t = threadIdx.x; t < nt; t += BX) {
        const PcbPrimeConst& pc = a.pr[tprime[t]];
        sP[t] = pc.p;
        sM0[t] = pc.mu_lo;
        sM1[t] = pc.mu_hi;
        sRow[t] = (uint32_t)trow[t];
    }
    __syncthreads();
    const size_t k = (size_t)blockIdx.x * BX + threadIdx.x;
    const uint64_t* src = (const uint64_t*)a.src + ((size_t)j.src_off << LOGN) + k;
    uint64_t* dst = (uint64_t*)a.dst + ((size_t)j.dst_off << LOGN) + k;
    uint64_t y[S];
#pragma unroll
    for (int i = 0; i < S; ++i) {
        if (NS > 0 || i < ns) {
            const uint64_t x = src[(size_t)srow[i] << LOGN];
            if (j.prescaled) {
                y[i] = x;
            } else {
                const PcbPrimeConst& q = a.pr[sprime[i]];
                y[i] = mul_mod(x, pre[i], q);
            }
        }
    }
    // exact jobs (HPS): u from the double estimate in source order (one fma per source), or the centred mean
    uint64_t u = 0;
    const uint64_t* bmod = nullptr;
    if (j.exact) {
        const uint64_t* rbw = M + ns * nt;  // u64 words are 8-byte aligned: the doubles start right after M
        if (j.exact == 2) {
            u = (uint64_t)(ns >> 1) + (uint64_t)((ns & 1) & (((uint32_t)k * 0x9E3779B1u) >> 31));
        } else {
            double v = 0.0;
#pragma unroll
            for (int i = 0; i < S; ++i)
                if (NS > 0 || i < ns) v = __fma_rn((double)y[i], __longlong_as_double((long long)rbw[i]), v);
            u = (uint64_t)floor(v + 0.5);
        }
        bmod = rbw + ns;
    }
    if constexpr (NARROW) {
        uint32_t y1[S], y0[S];
#pragma unroll
        for (int i = 0; i < S; ++i) {
            y1[i] = (uint32_t)(y[i] >> 26);
            y0[i] = (uint32_t)(y[i] & LO26);
        }
        for (int t = 0; t < nt; ++t) {
            Acc3 acc{0, 0, 0};
#pragma unroll
            for (int i = 0; i < S; ++i) {
                if (NS > 0 || i < ns) {
                    const uint64_t m = sM[i * nt + t];
                    mac3(acc, y1[i], y0[i], (uint32_t)(m >> 32), (uint32_t)m);
                }
            }
            const uint64_t p = sP[t];
            uint64_t r = reduce(to_acc(acc), p, sM0[t], sM1[t]);
            if (bmod) r = sub_mod(r, reduce(mul_wide(u, bmod[t]), p, sM0[t], sM1[t]), p);
            dst[(size_t)sRow[t] << LOGN] = r;
        }
    } else {
        for (int t = 0; t < nt; ++t) {
            Acc acc{0, 0};
#pragma unroll
            for (int i = 0; i < S; ++i)
                if (NS > 0 || i < ns) mac(acc, y[i], sM[i * nt + t]);
            const uint64_t p = sP[t];
            uint64_t r = reduce(acc, p, sM0[t], sM1[t]);
            if (bmod) r = sub_mod(r, reduce(mul_wide(u, bmod[t]), p, sM0[t], sM1[t]), p);
            dst[(size_t)sRow[t] << LOGN] = r;
        }
    }
}

// FP64 form for chains whose primes are all below 2^50: each product y_i M[i][t] mod t is mul_f with M centred and
// M / t taken as fl(M fl(1 / t)); sources enter as canonical doubles (|y M / t| < 2^49, so every product lies in
// [-0.625t, 0.625t]); the sum is reduced every 4 sources and made canonical once. The conversion matrix sits in shared
// memory as {M, M / t} pairs. Exact (HPS) jobs take their correction through the integer Barrett step.
// 128-coefficient spans per CTA: the shared tables are built once for all of them (2 and 8 measured the same)
constexpr int BCONV_F_SPAN = 4;
// NS > 0: every job has NS sources; NS < 0: at most -NS (a mixed launch of short digits); 0: any count up to MAX_SRC
template <int LOGN, int NS>
__global__ void __launch_bounds__(BX) bconv_f(PcbBconvArgs a) {
    constexpr int S = NS > 0 ? NS : NS < 0 ? -NS : MAX_SRC;
    __shared__ double2 sM[MAX_SRC * MAX_TGT];
    __shared__ double2 sP[MAX_TGT];  // {t, fl(1 / t)}
    __shared__ uint32_t sRow[MAX_TGT];
    const PcbBconvJob j = a.jobs[blockIdx.y];
    const uint64_t* pool = (const uint64_t*)a.pool + j.pool_off;
    const int ns = NS > 0 ? NS : (int)j.nsrc, nt = (int)j.ntgt;
    // outside the kernel's job shape: nothing is written
    if (ns < 1 || ns > S || nt > MAX_TGT || (int)j.nsrc != ns) return;
    const uint64_t* srow = pool;
    const uint64_t* sprime = pool + ns;
    const uint64_t* pre = pool + 2 * ns;
    const uint64_t* trow = pool + 3 * ns;
    const uint64_t* tprime = pool + 3 * ns + nt;
    const uint64_t* M = pool + 3 * ns + 2 * nt;
    for (int t = threadIdx.x; t < nt; t += BX) {
        const double tf = to_f(a.pr[tprime[t]].p);
        sP[t] = make_double2(tf, 1.0 / tf);
        sRow[t] = (uint32_t)trow[t];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < ns * nt; e += BX) {
        const uint64_t v = M[e], tp = a.pr[tprime[e % nt]].p;
        const double2 pt = sP[e % nt];
        const double w = v > tp / 2 ? -to_f(tp - v) : to_f(v);
        sM[e] = make_double2(w, __dmul_rn(w, pt.y));
    }
    __syncthreads();
    for (int rep = 0; rep < BCONV_F_SPAN; ++rep) {
    const size_t k = ((size_t)blockIdx.x * BCONV_F_SPAN + rep) * BX + threadIdx.x;
    const uint64_t* src = (const uint64_t*)a.src + ((size_t)j.src_off << LOGN) + k;
    uint64_t* dst = (uint64_t*)a.dst + ((size_t)j.dst_off << LOGN) + k;
    uint64_t y[S];
#pragma unroll
    for (int i = 0; i < S; ++i) {
        if (NS > 0 || i < ns) {
            const uint64_t x = src[(size_t)srow[i] << LOGN];
            y[i] = j.prescaled ? x : mul_mod(x, pre[i], a.pr[sprime[i]]);
        }
    }
    uint64_t u = 0;
    const uint64_t* bmod = nullptr;
    if (j.exact) {
        const uint64_t* rbw = M + ns * nt;
        if (j.exact == 2) {
            u = (uint64_t)(ns >> 1) + (uint64_t)((ns & 1) & (((uint32_t)k * 0x9E3779B1u) >> 31));
        } else {
            double v = 0.0;
#pragma unroll
            for (int i = 0; i < S; ++i)
                if (NS > 0 || i < ns) v = __fma_rn((double)y[i], __longlong_as_double((long long)rbw[i]), v);
            u = (uint64_t)floor(v + 0.5);
        }
        bmod = rbw + ns;
    }
    double yf[S];
#pragma unroll
    for (int i = 0; i < S; ++i)
        if (NS > 0 || i < ns) yf[i] = to_f(y[i]);
    for (int t = 0; t < nt; ++t) {
        const double2 pt = sP[t];
        double acc = 0.0;
#pragma unroll
        for (int i = 0; i < S; ++i) {
            if (NS > 0 || i < ns) {
                const double2 m = sM[i * nt + t];
                acc = __dadd_rn(acc, mul_f(yf[i], m.x, m.y, pt.x));
                if ((i & 3) == 3 && i + 1 < ns) acc = red_f(acc, pt.x, pt.y);
            }
        }
        uint64_t r = canon_f(acc, pt.x, pt.y);
        if (bmod) {
            const PcbPrimeConst& pc = a.pr[tprime[t]];
            r = sub_mod(r, reduce(mul_wide(u, bmod[t]), pc), pc.p);
        }
        dst[(size_t)sRow[t] << LOGN] = r;
    }
    }
}

template <int LOGN>
void bconv_dispatch_f(const PcbBconvArgs& a, int ns_all, dim3 g, cudaStream_t s) {
    switch (ns_all) {
        case 1: bconv_f<LOGN, 1><<<g, BX, 0, s>>>(a); break;
        case 2: bconv_f<LOGN, 2><<<g, BX, 0, s>>>(a); break;
        case 3: bconv_f<LOGN, 3><<<g, BX, 0, s>>>(a); break;
        case 4: bconv_f<LOGN, 4><<<g, BX, 0, s>>>(a); break;
        case 5: bconv_f<LOGN, 5><<<g, BX, 0, s>>>(a); break;
        case 6: bconv_f<LOGN, 6><<<g, BX, 0, s>>>(a); break;
        case 7: bconv_f<LOGN, 7><<<g, BX, 0, s>>>(a); break;
        case 8: bconv_f<LOGN, 8><<<g, BX, 0, s>>>(a); break;
        default:
            if (ns_all < 0 && ns_all >= -8) bconv_f<LOGN, -8><<<g, BX, 0, s>>>(a);
            else bconv_f<LOGN, 0><<<g, BX, 0, s>>>(a);
    }
}

template <int LOGN, bool NARROW>
void bconv_dispatch(const PcbBconvArgs& a, int ns_all, dim3 g, cudaStream_t s) {
    switch (ns_all) {
        case 1: bconv<LOGN, NARROW, 1><<<g, BX, 0, s>>>(a); break;
        case 2: bconv<LOGN, NARROW, 2><<<g, BX, 0, s>>>(a); break;
        case 4: bconv<LOGN, NARROW, 4><<<g, BX, 0, s>>>(a); break;
        case 8: bconv<LOGN, NARROW, 8><<<g, BX, 0, s>>>(a); break;
        default: bconv<LOGN, NARROW, 0><<<g, BX, 0, s>>>(a);
    }
}

// ns_all: the source count every job of the launch shares (unrolled kernels: FP64 1 .. 8, integer 1, 2, 4, 8); when
// they differ, minus the largest (FP64: up to 8 sources get an 8-wide kernel) or 0
template <int LOGN>
int bconv_run(const PcbBconvArgs* ap, bool narrow, bool f64, int ns_all, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbBconvArgs& a = *ap;
    if (a.njobs < 0 || a.max_tgt < 0 || a.max_tgt > MAX_TGT || !a.src || !a.dst || !a.jobs || !a.pool || !a.pr)
        return PCB_BAD_ARGS;
    if (a.njobs == 0) return 0;
    const dim3 g((1 << LOGN) / BX, a.njobs);
    if (f64) bconv_dispatch_f<LOGN>(a, ns_all, dim3((1 << LOGN) / (BX * BCONV_F_SPAN), a.njobs), s);
    else if (narrow) bconv_dispatch<LOGN, true>(a, ns_all, g, s);
    else bconv_dispatch<LOGN, false>(a, ns_all, g, s);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int bconv_launch(const PcbBconvArgs* ap, cudaStream_t s) {
    return bconv_run<LOGN>(ap, false, false, 0, s);
}

// ------------------------------------------------------------------------------------------------ ks_dot
// s1 = sum_d D_d a_d, s0 = C0 + sum_d D_d b_d for K <= KMAX ciphertexts x R keys; D_d[t] is c1 itself on digit d's
// own rows, else the ModUp output; each key word is read once per launch and reused by all K ciphertexts.
template <int LOGN>
__device__ __forceinline__ void ks_store(const PcbKsArgs& a, int c, int r, uint32_t t, size_t roff, uint32_t o,
                                         uint64_t r0, uint64_t r1, uint64_t p, uint64_t pm, uint64_t pms) {
    const uint64_t* c0 = (const uint64_t*)a.c0;
    if ((a.c0_mode & 3) == 1) {
        if ((int)t < a.nq) r0 = add_mod(r0, shoup(c0[(size_t)c * a.ct_stride + roff], pm, pms, p), p);
    } else if ((a.c0_mode & 3) == 2) {
        r0 = add_mod(r0, c0[(size_t)c * a.ct_stride + roff], p);
    }
    const size_t ob = (size_t)c * a.out_ct_stride + (size_t)r * a.out_rot_stride + ((size_t)t << LOGN) + o;
    if (a.c0_mode & PCB_KS_ACC) {
        r0 = add_mod(r0, ((const uint64_t*)a.out0)[ob], p);
        r1 = add_mod(r1, ((const uint64_t*)a.out1)[ob], p);
    }
    ((uint64_t*)a.out0)[ob] = r0;
    ((uint64_t*)a.out1)[ob] = r1;
}

template <int LOGN, int KMAX, bool NARROW>
__global__ void __launch_bounds__(BX) ks_dot(PcbKsArgs a) {
    const uint32_t t = a.rows[blockIdx.y];
    const PcbPrimeConst& pc = a.pr[t];
    const uint64_t p = pc.p;
    const uint32_t idx = blockIdx.x * BX + threadIdx.x;
    const int dt = (int)t < a.nq ? a.digit_of[t] : -1;
    const size_t roff = ((size_t)t << LOGN) + idx;
    const uint64_t* c1 = (const uint64_t*)a.c1;
    const uint64_t* mu = (const uint64_t*)a.modup;
    uint64_t pm = 0, pms = 0;
    if ((a.c0_mode & 3) == 1 && (int)t < a.nq) {
        pm = ((const uint64_t*)a.pmod)[t];
        pms = ((const uint64_t*)a.pmods)[t];
    }
    for (int r = 0; r < a.R; ++r) {
        const uint64_t* kb = (const uint64_t*)a.kb[r] + roff;
        const uint64_t* ka = (const uint64_t*)a.ka[r] + roff;
        const uint32_t k = a.autok[r];
        const uint32_t o = k == 1 ? idx : automorph_slot<LOGN>(k, idx);
        if (NARROW) {
            Acc3 s0[KMAX], s1[KMAX];
#pragma unroll
            for (int c = 0; c < KMAX; ++c) s0[c] = s1[c] = Acc3{0, 0, 0};
            for (int d = 0; d < a.ndig; ++d) {
                const uint64_t b = __ldcs(kb + (size_t)d * a.key_digit_stride);
                const uint64_t av = __ldcs(ka + (size_t)d * a.key_digit_stride);
                uint64_t x[KMAX];
#pragma unroll
                for (int c = 0; c < KMAX; ++c)
                    if (c < a.K)
                        x[c] = d == dt ? c1[(size_t)c * a.ct_stride + roff]
                                       : mu[(size_t)c * a.mu_ct_stride + (size_t)d * a.mu_digit_stride + roff];
                const uint32_t b1 = (uint32_t)(b >> 26), b0 = (uint32_t)(b & LO26);
                const uint32_t a1 = (uint32_t)(av >> 26), a0 = (uint32_t)(av & LO26);
#pragma unroll
                for (int c = 0; c < KMAX; ++c) {
                    if (c < a.K) {
                        const uint32_t x1 = (uint32_t)(x[c] >> 26), x0 = (uint32_t)(x[c] & LO26);
                        mac3(s0[c], x1, x0, b1, b0);
                        mac3(s1[c], x1, x0, a1, a0);
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < KMAX; ++c)
                if (c < a.K)
                    ks_store<LOGN>(a, c, r, t, roff, o, reduce(to_acc(s0[c]), pc), reduce(to_acc(s1[c]), pc), p, pm, pms);
        } else {
            Acc s0[KMAX], s1[KMAX];
#pragma unroll
            for (int c = 0; c < KMAX; ++c) s0[c] = s1[c] = Acc{0, 0};
            for (int d = 0; d < a.ndig; ++d) {
                const uint64_t b = __ldcs(kb + (size_t)d * a.key_digit_stride);
                const uint64_t av = __ldcs(ka + (size_t)d * a.key_digit_stride);
#pragma unroll
                for (int c = 0; c < KMAX; ++c) {
                    if (c < a.K) {
                        const uint64_t x = d == dt ? c1[(size_t)c * a.ct_stride + roff]
                                                   : mu[(size_t)c * a.mu_ct_stride + (size_t)d * a.mu_digit_stride + roff];
                        mac(s0[c], x, b);
                        mac(s1[c], x, av);
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < KMAX; ++c)
                if (c < a.K) ks_store<LOGN>(a, c, r, t, roff, o, reduce(s0[c], pc), reduce(s1[c], pc), p, pm, pms);
        }
    }
}

template <int LOGN>
int ks_dot_run(const PcbKsArgs* ap, bool narrow, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbKsArgs& a = *ap;
    if (a.K < 0 || a.K > 8 || a.R < 0 || a.ndig < 1 || a.ndig > 16 || a.nrows < 0 || (a.c0_mode & 3) == 3 ||
        (a.c0_mode & ~(3 | PCB_KS_ACC)) || !a.c1 || !a.out0 || !a.out1 || !a.kb || !a.ka || !a.autok || !a.rows ||
        !a.digit_of || !a.pr)
        return PCB_BAD_ARGS;
    if ((a.c0_mode & 3) && !a.c0) return PCB_BAD_ARGS;
    if ((a.c0_mode & 3) == 1 && (!a.pmod || !a.pmods)) return PCB_BAD_ARGS;
    if (a.ndig > 1 && !a.modup) return PCB_BAD_ARGS;
    if (narrow && a.K > 4) return PCB_BAD_ARGS;  // the narrow accumulators hold four ciphertexts per thread
    if (a.K == 0 || a.R == 0 || a.nrows == 0) return 0;
    const dim3 g((1 << LOGN) / BX, a.nrows);
    if (narrow) {
        if (a.K <= 1) ks_dot<LOGN, 1, true><<<g, BX, 0, s>>>(a);
        else if (a.K <= 2) ks_dot<LOGN, 2, true><<<g, BX, 0, s>>>(a);
        else ks_dot<LOGN, 4, true><<<g, BX, 0, s>>>(a);
    } else {
        if (a.K <= 1) ks_dot<LOGN, 1, false><<<g, BX, 0, s>>>(a);
        else if (a.K <= 2) ks_dot<LOGN, 2, false><<<g, BX, 0, s>>>(a);
        else if (a.K <= 4) ks_dot<LOGN, 4, false><<<g, BX, 0, s>>>(a);
        else ks_dot<LOGN, 8, false><<<g, BX, 0, s>>>(a);
    }
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int ks_dot_launch(const PcbKsArgs* ap, cudaStream_t s) {
    return ks_dot_run<LOGN>(ap, false, s);
}

// ------------------------------------------------------------------------------------------------ dot over a batch
// The evaluator's inner product: one key (R = 1), any number K of ciphertexts. Each thread reads its slot's key
// words of every digit once and then walks the K ciphertexts, so a batch streams the key once (ks_dot re-reads it
// for every group of <= 8). The inputs (c1, the ModUp digits, c0) must not alias the outputs. ND > 0: exactly ND
// live digits (unrolled); 0: a.ndig <= 16. RG: the key's `a` is regenerated from `seed` into shared memory
// (keyregen.cuh: the CTA's BX slots, every digit) instead of read from a.ka.
template <int LOGN, int ND, bool NARROW, bool RG>
__global__ void __launch_bounds__(BX) dot_all(PcbKsArgs a, const uint32_t* seed) {
    extern __shared__ __align__(16) uint64_t rg_sm[];
    constexpr int D = ND > 0 ? ND : 16;
    const int nd = ND > 0 ? ND : a.ndig;
    const uint32_t t = a.rows[blockIdx.y];
    const PcbPrimeConst& pc = a.pr[t];
    const uint64_t p = pc.p;
    const uint32_t idx = blockIdx.x * BX + threadIdx.x;
    const int dt = (int)t < a.nq ? a.digit_of[t] : -1;
    const size_t roff = ((size_t)t << LOGN) + idx;
    const uint64_t* c1 = (const uint64_t*)a.c1;
    const uint64_t* mu = (const uint64_t*)a.modup;
    uint64_t pm = 0, pms = 0;
    if ((a.c0_mode & 3) == 1 && (int)t < a.nq) {
        pm = ((const uint64_t*)a.pmod)[t];
        pms = ((const uint64_t*)a.pmods)[t];
    }
    const uint64_t* kb = (const uint64_t*)a.kb[0] + roff;
    const uint64_t* ka = RG ? nullptr : (const uint64_t*)a.ka[0] + roff;
    constexpr int NSEG = BX / keyregen::SEG;
    if constexpr (RG) {
        const uint32_t tile0 = blockIdx.x * BX;
        keyregen::stage<LOGN>(&seed, 1, nd, NSEG, [tile0](int, int j) { return tile0 + (uint32_t)j * keyregen::SEG; },
                              pc, rg_sm);
    }
    uint64_t bv[D], av[D];
#pragma unroll
    for (int d = 0; d < D; ++d) {
        if (ND > 0 || d < nd) {
            bv[d] = __ldcs(kb + (size_t)d * a.key_digit_stride);
            av[d] = RG ? keyregen::at(rg_sm, nd, NSEG, 0, d, threadIdx.x / keyregen::SEG, idx)
                       : __ldcs(ka + (size_t)d * a.key_digit_stride);
        }
    }
    const uint32_t k = a.autok[0];
    const uint32_t o = k == 1 ? idx : automorph_slot<LOGN>(k, idx);
    if (NARROW) {
        uint32_t b1[D], b0[D], a1[D], a0[D];
#pragma unroll
        for (int d = 0; d < D; ++d) {
            b1[d] = (uint32_t)(bv[d] >> 26);
            b0[d] = (uint32_t)(bv[d] & LO26);
            a1[d] = (uint32_t)(av[d] >> 26);
            a0[d] = (uint32_t)(av[d] & LO26);
        }
#pragma unroll 2
        for (int c = 0; c < a.K; ++c) {
            Acc3 s0{0, 0, 0}, s1{0, 0, 0};
#pragma unroll
            for (int d = 0; d < D; ++d) {
                if (ND > 0 || d < nd) {
                    const uint64_t x = d == dt ? __ldg(c1 + (size_t)c * a.ct_stride + roff)
                                               : __ldg(mu + (size_t)c * a.mu_ct_stride + (size_t)d * a.mu_digit_stride + roff);
                    const uint32_t x1 = (uint32_t)(x >> 26), x0 = (uint32_t)(x & LO26);
                    mac3(s0, x1, x0, b1[d], b0[d]);
                    mac3(s1, x1, x0, a1[d], a0[d]);
                }
            }
            ks_store<LOGN>(a, c, 0, t, roff, o, reduce(to_acc(s0), pc), reduce(to_acc(s1), pc), p, pm, pms);
        }
    } else {
#pragma unroll 2
        for (int c = 0; c < a.K; ++c) {
            Acc s0{0, 0}, s1{0, 0};
#pragma unroll
            for (int d = 0; d < D; ++d) {
                if (ND > 0 || d < nd) {
                    const uint64_t x = d == dt ? __ldg(c1 + (size_t)c * a.ct_stride + roff)
                                               : __ldg(mu + (size_t)c * a.mu_ct_stride + (size_t)d * a.mu_digit_stride + roff);
                    mac(s0, x, bv[d]);
                    mac(s1, x, av[d]);
                }
            }
            ks_store<LOGN>(a, c, 0, t, roff, o, reduce(s0, pc), reduce(s1, pc), p, pm, pms);
        }
    }
}

// FP64 form of dot_all for primes below 2^50: a digit product x b mod p is mul_f with b centred and its quotient
// b / p taken as fl(b fl(1 / p)) (relative error <= 2^-52: |x b / p| < 2^49, so q is within 0.63 of it and each
// product lies in [-0.63p, 0.63p]); sums are reduced every 4 digits and made canonical once per output word. Each
// thread takes two adjacent words (16-byte loads; the launcher checks the alignment) of every ciphertext.
template <int LOGN, int ND, bool RG>
__global__ void __launch_bounds__(BX) dot_all_f(PcbKsArgs a, const uint32_t* seed) {
    extern __shared__ __align__(16) uint64_t rg_sm[];
    constexpr int D = ND > 0 ? ND : 16;
    const int nd = ND > 0 ? ND : a.ndig;
    const uint32_t t = a.rows[blockIdx.y];
    const uint64_t p = a.pr[t].p;
    const double pf = to_f(p), pinv = 1.0 / pf;
    const uint32_t idx = 2 * (blockIdx.x * BX + threadIdx.x);  // words idx, idx + 1
    const int dt = (int)t < a.nq ? a.digit_of[t] : -1;
    const size_t roff = ((size_t)t << LOGN) + idx;
    const uint64_t* c1 = (const uint64_t*)a.c1;
    const uint64_t* mu = (const uint64_t*)a.modup;
    uint64_t pm = 0, pms = 0;
    if ((a.c0_mode & 3) == 1 && (int)t < a.nq) {
        pm = ((const uint64_t*)a.pmod)[t];
        pms = ((const uint64_t*)a.pmods)[t];
    }
    const uint64_t* kb = (const uint64_t*)a.kb[0] + roff;
    const uint64_t* ka = RG ? nullptr : (const uint64_t*)a.ka[0] + roff;
    constexpr int NSEG = 2 * BX / keyregen::SEG;
    if constexpr (RG) {  // the CTA's 2 BX slots of every digit
        const uint32_t tile0 = 2 * blockIdx.x * BX;
        keyregen::stage<LOGN>(&seed, 1, nd, NSEG, [tile0](int, int j) { return tile0 + (uint32_t)j * keyregen::SEG; },
                              a.pr[t], rg_sm);
    }
    double bw[D][2], bq[D][2], aw[D][2], aq[D][2];
#pragma unroll
    for (int d = 0; d < D; ++d) {
        if (ND > 0 || d < nd) {
            const ulonglong2 b = __ldcs((const ulonglong2*)(kb + (size_t)d * a.key_digit_stride));
            const ulonglong2 av =
                RG ? *(const ulonglong2*)&rg_sm[((size_t)d * NSEG + (2 * threadIdx.x) / keyregen::SEG) * keyregen::SEG +
                                               ((2 * threadIdx.x) & (keyregen::SEG - 1))]
                   : __ldcs((const ulonglong2*)(ka + (size_t)d * a.key_digit_stride));
            const uint64_t bb[2] = {b.x, b.y}, aa[2] = {av.x, av.y};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                bw[d][h] = bb[h] > p / 2 ? -to_f(p - bb[h]) : to_f(bb[h]);
                aw[d][h] = aa[h] > p / 2 ? -to_f(p - aa[h]) : to_f(aa[h]);
                bq[d][h] = __dmul_rn(bw[d][h], pinv);
                aq[d][h] = __dmul_rn(aw[d][h], pinv);
            }
        }
    }
    const uint32_t k = a.autok[0];
    const uint32_t o0 = k == 1 ? idx : automorph_slot<LOGN>(k, idx);
    const uint32_t o1 = k == 1 ? idx + 1 : automorph_slot<LOGN>(k, idx + 1);
#pragma unroll 2
    for (int c = 0; c < a.K; ++c) {
        double s0[2] = {0.0, 0.0}, s1[2] = {0.0, 0.0};
#pragma unroll
        for (int d = 0; d < D; ++d) {
            if (ND > 0 || d < nd) {
                const ulonglong2 w = __ldg((const ulonglong2*)(d == dt ? c1 + (size_t)c * a.ct_stride + roff
                                                                        : mu + (size_t)c * a.mu_ct_stride +
                                                                              (size_t)d * a.mu_digit_stride + roff));
                const double x[2] = {to_f(w.x), to_f(w.y)};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    s0[h] = __dadd_rn(s0[h], mul_f(x[h], bw[d][h], bq[d][h], pf));
                    s1[h] = __dadd_rn(s1[h], mul_f(x[h], aw[d][h], aq[d][h], pf));
                    if ((d & 3) == 3) {
                        s0[h] = red_f(s0[h], pf, pinv);
                        s1[h] = red_f(s1[h], pf, pinv);
                    }
                }
            }
        }
        ks_store<LOGN>(a, c, 0, t, roff, o0, canon_f(s0[0], pf, pinv), canon_f(s1[0], pf, pinv), p, pm, pms);
        ks_store<LOGN>(a, c, 0, t, roff + 1, o1, canon_f(s0[1], pf, pinv), canon_f(s1[1], pf, pinv), p, pm, pms);
    }
}

// Several keys against the same ModUp digits (the steps of a hoisted rotation): each digit word is read once and
// multiplied by every key of the group, so the digits stream once per group instead of once per key. One word per
// thread; the keys stay in registers as centred doubles (their quotients by p are formed per use, as in dot_all_f).
// 6 CTAs per SM (at most 85 registers, 24 warps): the config-2 step took 100.0 ms, against 101.0 at 5 CTAs
// (102 registers) and 101.5-102.5 with the compiler's choice of 116
// RG: every key's `a` is regenerated from kg.seed[r] into shared memory (the CTA's BX slots, RK keys x ND digits).
template <int LOGN, int ND, int RK, bool RG>
__global__ void __launch_bounds__(BX, 6) dot_keys_f(PcbKsArgs a, KeyGroup kg) {
    extern __shared__ __align__(16) uint64_t rg_sm[];
    const uint32_t t = a.rows[blockIdx.y];
    const uint64_t p = a.pr[t].p;
    const double pf = to_f(p), pinv = 1.0 / pf;
    const uint32_t idx = blockIdx.x * BX + threadIdx.x;
    const int dt = (int)t < a.nq ? a.digit_of[t] : -1;
    const size_t roff = ((size_t)t << LOGN) + idx;
    const uint64_t* c1 = (const uint64_t*)a.c1;
    const uint64_t* mu = (const uint64_t*)a.modup;
    uint64_t pm = 0, pms = 0;
    if ((a.c0_mode & 3) == 1 && (int)t < a.nq) {
        pm = ((const uint64_t*)a.pmod)[t];
        pms = ((const uint64_t*)a.pmods)[t];
    }
    constexpr int NSEG = BX / keyregen::SEG;
    if constexpr (RG) {
        const uint32_t tile0 = blockIdx.x * BX;
        keyregen::stage<LOGN>(kg.seed, RK, ND, NSEG, [tile0](int, int j) { return tile0 + (uint32_t)j * keyregen::SEG; },
                              a.pr[t], rg_sm);
    }
    double bw[RK][ND], aw[RK][ND];
    uint32_t o[RK];
#pragma unroll
    for (int r = 0; r < RK; ++r) {
#pragma unroll
        for (int d = 0; d < ND; ++d) {
            const uint64_t b = __ldcs(kg.kb[r] + roff + (size_t)d * a.key_digit_stride);
            const uint64_t av = RG ? keyregen::at(rg_sm, ND, NSEG, r, d, threadIdx.x / keyregen::SEG, idx)
                                   : __ldcs(kg.ka[r] + roff + (size_t)d * a.key_digit_stride);
            bw[r][d] = b > p / 2 ? -to_f(p - b) : to_f(b);
            aw[r][d] = av > p / 2 ? -to_f(p - av) : to_f(av);
        }
        o[r] = kg.autok[r] == 1 ? idx : automorph_slot<LOGN>(kg.autok[r], idx);
    }
    for (int c = 0; c < a.K; ++c) {
        double x[ND];
#pragma unroll
        for (int d = 0; d < ND; ++d)
            x[d] = to_f(d == dt ? __ldg(c1 + (size_t)c * a.ct_stride + roff)
                                : __ldg(mu + (size_t)c * a.mu_ct_stride + (size_t)d * a.mu_digit_stride + roff));
#pragma unroll
        for (int r = 0; r < RK; ++r) {
            double s0 = 0.0, s1 = 0.0;
#pragma unroll
            for (int d = 0; d < ND; ++d) {
                s0 = __dadd_rn(s0, mul_f(x[d], bw[r][d], __dmul_rn(bw[r][d], pinv), pf));
                s1 = __dadd_rn(s1, mul_f(x[d], aw[r][d], __dmul_rn(aw[r][d], pinv), pf));
                if ((d & 3) == 3 && d + 1 < ND) {
                    s0 = red_f(s0, pf, pinv);
                    s1 = red_f(s1, pf, pinv);
                }
            }
            ks_store<LOGN>(a, c, r, t, roff, o[r], canon_f(s0, pf, pinv), canon_f(s1, pf, pinv), p, pm, pms);
        }
    }
}

// The inner products of a rotate_sum group (crates/pc-gpu/src/rotate.rs:690-775) in gather form, summed in
// registers: for every output slot o of row t and ciphertext c,
//   out0[o] = sum_r ( P c0[i_r] (Q rows) + sum_d x_d[i_r] b_{r,d}[i_r] ),  out1[o] = sum_r sum_d x_d[i_r] a_{r,d}[i_r]
// with i_r = automorph_slot(g_r, o), the slot the rotation by key r moves to o (the scatter form writes the same
// sums at automorph_slot(g_r^-1, i)). One launch writes the group's extended batch once, where a chain of
// accumulate-mode launches reads and rewrites it once per key; the digit words the keys gather from the same row
// are re-read from L2 (a row of K ciphertexts' digits is a few tens of MB).
struct SumRow {
    uint32_t t;
    size_t row;
    int dt;
    uint64_t p, pm, pms;
    double pf, pinv;
    bool addc0;
};

// CB ciphertexts from cb: per key, its 2 ND words and the CB x ND digit words are all loaded before any product (no
// predicate between them), so each key costs one memory latency instead of one per ciphertext
// rg: the keys' staged `a` segments (keyregen.cuh, nseg 4, this thread's segment j = its warp), or null (dense)
template <int LOGN, int ND, int CB>
__device__ __forceinline__ void dot_sum_chunk(const PcbKsArgs& a, const KeySum& ks, const SumRow& w,
                                              const uint32_t* src, uint32_t o, int cb, const uint64_t* rg) {
    const uint64_t* c1 = (const uint64_t*)a.c1;
    const uint64_t* mu = (const uint64_t*)a.modup;
    double s0[CB], s1[CB];
#pragma unroll
    for (int u = 0; u < CB; ++u) s0[u] = s1[u] = 0.0;
    for (int r = 0; r < ks.n; ++r) {
        const size_t off = w.row + src[r];
        uint64_t kbv[ND], kav[ND], xw[CB][ND];
#pragma unroll
        for (int d = 0; d < ND; ++d) {
            kbv[d] = __ldg(ks.kb[r] + off + (size_t)d * a.key_digit_stride);
            kav[d] = rg ? keyregen::at(rg, ND, BX / keyregen::SEG, r, d, threadIdx.x / keyregen::SEG, src[r])
                        : __ldg(ks.ka[r] + off + (size_t)d * a.key_digit_stride);
        }
#pragma unroll
        for (int u = 0; u < CB; ++u)
#pragma unroll
            for (int d = 0; d < ND; ++d)
                xw[u][d] = __ldg(d == w.dt ? c1 + (size_t)(cb + u) * a.ct_stride + off
                                           : mu + (size_t)(cb + u) * a.mu_ct_stride + (size_t)d * a.mu_digit_stride + off);
#pragma unroll
        for (int d = 0; d < ND; ++d) {
            const double bw = kbv[d] > w.p / 2 ? -to_f(w.p - kbv[d]) : to_f(kbv[d]);
            const double aw = kav[d] > w.p / 2 ? -to_f(w.p - kav[d]) : to_f(kav[d]);
            const double bq = __dmul_rn(bw, w.pinv), aq = __dmul_rn(aw, w.pinv);
#pragma unroll
            for (int u = 0; u < CB; ++u) {
                const double x = to_f(xw[u][d]);
                s0[u] = __dadd_rn(s0[u], mul_f(x, bw, bq, w.pf));
                s1[u] = __dadd_rn(s1[u], mul_f(x, aw, aq, w.pf));
            }
        }
        // at most ND <= 4 products since the last reduction: |s| < 9 p < 2^53
#pragma unroll
        for (int u = 0; u < CB; ++u) {
            s0[u] = red_f(s0[u], w.pf, w.pinv);
            s1[u] = red_f(s1[u], w.pf, w.pinv);
        }
    }
    const uint64_t* c0 = (const uint64_t*)a.c0;
#pragma unroll
    for (int u = 0; u < CB; ++u) {
        const int c = cb + u;
        uint64_t r0 = canon_f(s0[u], w.pf, w.pinv), r1 = canon_f(s1[u], w.pf, w.pinv);
        if (w.addc0)
            for (int r = 0; r < ks.n; ++r)
                r0 = add_mod(r0, shoup(__ldg(c0 + (size_t)c * a.ct_stride + w.row + src[r]), w.pm, w.pms, w.p), w.p);
        const size_t ob = (size_t)c * a.out_ct_stride + w.row + o;
        if (a.c0_mode & PCB_KS_ACC) {
            r0 = add_mod(r0, ((const uint64_t*)a.out0)[ob], w.p);
            r1 = add_mod(r1, ((const uint64_t*)a.out1)[ob], w.p);
        }
        ((uint64_t*)a.out0)[ob] = r0;
        ((uint64_t*)a.out1)[ob] = r1;
    }
}

// Ciphertexts in chunks of CB (then one at a time for the rest); with PCB_KS_ACC the previous batch is added
// RG: the keys' `a` regenerated into shared memory: per key, the 4 aligned 32-slot source segments that the CTA's
// 4 warps of output slots gather from
template <int LOGN, int ND, int CB, bool RG>
__global__ void __launch_bounds__(BX, 4) dot_sum_f(PcbKsArgs a, KeySum ks) {
    extern __shared__ __align__(16) uint64_t rg_sm[];
    SumRow w;
    w.t = a.rows[blockIdx.y];
    w.p = a.pr[w.t].p;
    w.pf = to_f(w.p);
    w.pinv = 1.0 / w.pf;
    w.dt = (int)w.t < a.nq ? a.digit_of[w.t] : -1;
    w.row = (size_t)w.t << LOGN;
    w.addc0 = (a.c0_mode & 3) == 1 && (int)w.t < a.nq;
    w.pm = w.pms = 0;
    if (w.addc0) {
        w.pm = ((const uint64_t*)a.pmod)[w.t];
        w.pms = ((const uint64_t*)a.pmods)[w.t];
    }
    const uint32_t o = blockIdx.x * BX + threadIdx.x;
    if constexpr (RG) {
        const uint32_t tile0 = blockIdx.x * BX;
        const uint32_t* g = ks.g;
        keyregen::stage<LOGN>(ks.seed, ks.n, ND, BX / keyregen::SEG,
                              [tile0, g](int r, int j) {
                                  return automorph_slot<LOGN>(g[r], tile0 + (uint32_t)j * keyregen::SEG) &
                                         ~(uint32_t)(keyregen::SEG - 1);
                              },
                              a.pr[w.t], rg_sm);
    }
    const uint64_t* rg = RG ? rg_sm : nullptr;
    uint32_t src[SUM_KEYS_MAX];
#pragma unroll
    for (int r = 0; r < SUM_KEYS_MAX; ++r) src[r] = r < ks.n ? automorph_slot<LOGN>(ks.g[r], o) : 0;
    int cb = 0;
    for (; cb + CB <= a.K; cb += CB) dot_sum_chunk<LOGN, ND, CB>(a, ks, w, src, o, cb, rg);
    for (; cb < a.K; ++cb) dot_sum_chunk<LOGN, ND, 1>(a, ks, w, src, o, cb, rg);
}

// One ciphertext (K = 1): the keys split over the CTA's 4 warps for the same 32 output slots (warp w takes keys w,
// w + 4), each warp's partial sum canonical in shared memory, warp 0 adding them up: four warps' loads in flight per
// slot where the one-thread-per-slot form walks the keys one after another.
constexpr int SUM1_WARPS = 4;
// RG: every key's `a` regenerated into shared memory (per key the one aligned 32-slot segment the 32 outputs gather
// from), staged by all four warps before the products
template <int LOGN, int ND, bool RG>
__global__ void __launch_bounds__(32 * SUM1_WARPS) dot_sum1_f(PcbKsArgs a, KeySum ks) {
    __shared__ uint64_t part[2][SUM1_WARPS][32];
    extern __shared__ __align__(16) uint64_t rg_sm[];
    const uint32_t t = a.rows[blockIdx.y];
    const uint64_t p = a.pr[t].p;
    const double pf = to_f(p), pinv = 1.0 / pf;
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    const uint32_t o = blockIdx.x * 32 + lane;
    const int dt = (int)t < a.nq ? a.digit_of[t] : -1;
    const size_t row = (size_t)t << LOGN;
    const uint64_t* c1 = (const uint64_t*)a.c1;
    const uint64_t* mu = (const uint64_t*)a.modup;
    const uint64_t* c0 = (const uint64_t*)a.c0;
    const bool addc0 = (a.c0_mode & 3) == 1 && (int)t < a.nq;
    uint64_t pm = 0, pms = 0;
    if (addc0) {
        pm = ((const uint64_t*)a.pmod)[t];
        pms = ((const uint64_t*)a.pmods)[t];
    }
    if constexpr (RG) {
        const uint32_t tile0 = blockIdx.x * 32;
        const uint32_t* g = ks.g;
        keyregen::stage<LOGN>(ks.seed, ks.n, ND, 1,
                              [tile0, g](int r, int) {
                                  return automorph_slot<LOGN>(g[r], tile0) & ~(uint32_t)(keyregen::SEG - 1);
                              },
                              a.pr[t], rg_sm);
    }
    double s0 = 0.0, s1 = 0.0;
    uint64_t cs = 0;  // this warp's keys' P sigma(c0) terms
    for (int r = wp; r < ks.n; r += SUM1_WARPS) {
        const uint32_t src = automorph_slot<LOGN>(ks.g[r], o);
        const size_t off = row + src;
        uint64_t kbv[ND], kav[ND], xw[ND];
#pragma unroll
        for (int d = 0; d < ND; ++d) {
            kbv[d] = __ldg(ks.kb[r] + off + (size_t)d * a.key_digit_stride);
            kav[d] = RG ? keyregen::at(rg_sm, ND, 1, r, d, 0, src) : __ldg(ks.ka[r] + off + (size_t)d * a.key_digit_stride);
            xw[d] = __ldg(d == dt ? c1 + off : mu + (size_t)d * a.mu_digit_stride + off);
        }
        const uint64_t cw = addc0 ? __ldg(c0 + off) : 0;
#pragma unroll
        for (int d = 0; d < ND; ++d) {
            const double bw = kbv[d] > p / 2 ? -to_f(p - kbv[d]) : to_f(kbv[d]);
            const double aw = kav[d] > p / 2 ? -to_f(p - kav[d]) : to_f(kav[d]);
            const double x = to_f(xw[d]);
            s0 = __dadd_rn(s0, mul_f(x, bw, __dmul_rn(bw, pinv), pf));
            s1 = __dadd_rn(s1, mul_f(x, aw, __dmul_rn(aw, pinv), pf));
        }
        // at most ND <= 4 products since the last reduction: |s| < 9 p < 2^53
        s0 = red_f(s0, pf, pinv);
        s1 = red_f(s1, pf, pinv);
        if (addc0) cs = add_mod(cs, shoup(cw, pm, pms, p), p);
    }
    part[0][wp][lane] = add_mod(canon_f(s0, pf, pinv), cs, p);
    part[1][wp][lane] = canon_f(s1, pf, pinv);
    __syncthreads();
    if (wp == 0) {
        uint64_t r0 = part[0][0][lane], r1 = part[1][0][lane];
#pragma unroll
        for (int w = 1; w < SUM1_WARPS; ++w) {
            r0 = add_mod(r0, part[0][w][lane], p);
            r1 = add_mod(r1, part[1][w][lane], p);
        }
        const size_t ob = row + o;
        if (a.c0_mode & PCB_KS_ACC) {
            r0 = add_mod(r0, ((const uint64_t*)a.out0)[ob], p);
            r1 = add_mod(r1, ((const uint64_t*)a.out1)[ob], p);
        }
        ((uint64_t*)a.out0)[ob] = r0;
        ((uint64_t*)a.out1)[ob] = r1;
    }
}

template <int LOGN, int ND, bool RG>
void dot_keys_dispatch(const PcbKsArgs& a, const KeyGroup& kg, dim3 g, cudaStream_t s) {
    const size_t sm = RG ? (size_t)kg.n * ND * BX * sizeof(uint64_t) : 0;
    switch (kg.n) {
        case 1: dot_keys_f<LOGN, ND, 1, RG><<<g, BX, sm, s>>>(a, kg); break;
        case 2: dot_keys_f<LOGN, ND, 2, RG><<<g, BX, sm, s>>>(a, kg); break;
        case 3: dot_keys_f<LOGN, ND, 3, RG><<<g, BX, sm, s>>>(a, kg); break;
        default: dot_keys_f<LOGN, ND, 4, RG><<<g, BX, sm, s>>>(a, kg);
    }
}

// every key of a group or sum is either dense (ka set) or regenerated (seed set), the same for all
template <class G>
int key_source_of(const G& kg) {
    bool dense = false, regen = false;
    for (int r = 0; r < kg.n; ++r) {
        if (!kg.kb[r] || (!kg.ka[r] == !kg.seed[r])) return -1;
        (kg.seed[r] ? regen : dense) = true;
    }
    return dense && regen ? -1 : regen ? 1 : 0;
}

template <int LOGN>
int dot_keys_run(const PcbKsArgs* ap, const KeyGroup& kg, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbKsArgs& a = *ap;
    if (kg.n < 1 || kg.n > KEYS_MAX || a.K < 0 || a.ndig < 1 || a.ndig > 4 || a.nrows < 0 || (a.c0_mode & 3) == 3 ||
        (a.c0_mode & ~(3 | PCB_KS_ACC)) || !a.c1 || !a.out0 || !a.out1 || !a.rows || !a.digit_of || !a.pr)
        return PCB_BAD_ARGS;
    const int src = key_source_of(kg);
    if (src < 0) return PCB_BAD_ARGS;
    for (int r = 0; r < kg.n; ++r)
        if (!(kg.autok[r] & 1)) return PCB_BAD_ARGS;
    if ((a.c0_mode & 3) && !a.c0) return PCB_BAD_ARGS;
    if ((a.c0_mode & 3) == 1 && (!a.pmod || !a.pmods)) return PCB_BAD_ARGS;
    if (a.ndig > 1 && !a.modup) return PCB_BAD_ARGS;
    if (a.K == 0 || a.nrows == 0) return 0;
    const dim3 g((1 << LOGN) / BX, a.nrows);
    if (src) {
        switch (a.ndig) {
            case 1: dot_keys_dispatch<LOGN, 1, true>(a, kg, g, s); break;
            case 2: dot_keys_dispatch<LOGN, 2, true>(a, kg, g, s); break;
            case 3: dot_keys_dispatch<LOGN, 3, true>(a, kg, g, s); break;
            default: dot_keys_dispatch<LOGN, 4, true>(a, kg, g, s);
        }
    } else {
        switch (a.ndig) {
            case 1: dot_keys_dispatch<LOGN, 1, false>(a, kg, g, s); break;
            case 2: dot_keys_dispatch<LOGN, 2, false>(a, kg, g, s); break;
            case 3: dot_keys_dispatch<LOGN, 3, false>(a, kg, g, s); break;
            default: dot_keys_dispatch<LOGN, 4, false>(a, kg, g, s);
        }
    }
    return PCB_LAUNCH_RESULT();
}

template <int LOGN, bool RG>
void dot_sum_dispatch(const PcbKsArgs& a, const KeySum& ks, cudaStream_t s) {
    if (a.K == 1) {
        const dim3 g1((1 << LOGN) / 32, a.nrows);
        const size_t sm = RG ? (size_t)ks.n * a.ndig * keyregen::SEG * sizeof(uint64_t) : 0;
        switch (a.ndig) {
            case 1: dot_sum1_f<LOGN, 1, RG><<<g1, 32 * SUM1_WARPS, sm, s>>>(a, ks); break;
            case 2: dot_sum1_f<LOGN, 2, RG><<<g1, 32 * SUM1_WARPS, sm, s>>>(a, ks); break;
            case 3: dot_sum1_f<LOGN, 3, RG><<<g1, 32 * SUM1_WARPS, sm, s>>>(a, ks); break;
            default: dot_sum1_f<LOGN, 4, RG><<<g1, 32 * SUM1_WARPS, sm, s>>>(a, ks);
        }
        return;
    }
    const dim3 g((1 << LOGN) / BX, a.nrows);
    const size_t sm = RG ? (size_t)ks.n * a.ndig * BX * sizeof(uint64_t) : 0;
    switch (a.ndig) {
        case 1: dot_sum_f<LOGN, 1, 4, RG><<<g, BX, sm, s>>>(a, ks); break;
        case 2: dot_sum_f<LOGN, 2, 4, RG><<<g, BX, sm, s>>>(a, ks); break;
        case 3: dot_sum_f<LOGN, 3, 4, RG><<<g, BX, sm, s>>>(a, ks); break;
        default: dot_sum_f<LOGN, 4, 4, RG><<<g, BX, sm, s>>>(a, ks);
    }
}

template <int LOGN>
int dot_sum_run(const PcbKsArgs* ap, const KeySum& ks, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbKsArgs& a = *ap;
    if (ks.n < 1 || ks.n > SUM_KEYS_MAX || a.K < 0 || a.ndig < 1 || a.ndig > 4 || a.nrows < 0 ||
        (a.c0_mode & 3) == 2 || (a.c0_mode & 3) == 3 || (a.c0_mode & ~(3 | PCB_KS_ACC)) || !a.c1 || !a.out0 ||
        !a.out1 || !a.rows || !a.digit_of || !a.pr)
        return PCB_BAD_ARGS;
    const int src = key_source_of(ks);
    if (src < 0) return PCB_BAD_ARGS;
    for (int r = 0; r < ks.n; ++r)
        if (!(ks.g[r] & 1)) return PCB_BAD_ARGS;
    if ((a.c0_mode & 3) == 1 && (!a.c0 || !a.pmod || !a.pmods)) return PCB_BAD_ARGS;
    if (a.ndig > 1 && !a.modup) return PCB_BAD_ARGS;
    if (a.K == 0 || a.nrows == 0) return 0;
    if (src) dot_sum_dispatch<LOGN, true>(a, ks, s);
    else dot_sum_dispatch<LOGN, false>(a, ks, s);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN, bool NARROW, bool RG>
void dot_dispatch(const PcbKsArgs& a, const uint32_t* seed, dim3 g, cudaStream_t s) {
    const size_t sm = RG ? (size_t)a.ndig * BX * sizeof(uint64_t) : 0;
    switch (a.ndig) {
        case 1: dot_all<LOGN, 1, NARROW, RG><<<g, BX, sm, s>>>(a, seed); break;
        case 2: dot_all<LOGN, 2, NARROW, RG><<<g, BX, sm, s>>>(a, seed); break;
        case 3: dot_all<LOGN, 3, NARROW, RG><<<g, BX, sm, s>>>(a, seed); break;
        case 4: dot_all<LOGN, 4, NARROW, RG><<<g, BX, sm, s>>>(a, seed); break;
        case 8: dot_all<LOGN, 8, NARROW, RG><<<g, BX, sm, s>>>(a, seed); break;
        default: dot_all<LOGN, 0, NARROW, RG><<<g, BX, sm, s>>>(a, seed);
    }
}

// Plain launches: programmatic dependent launch of bconv_f and dot_all_f (tables and keys staged before the wait)
// measured slower here (108.8 -> 111.3 ms per config-2 step)
template <int LOGN, bool RG>
void dot_dispatch_f(const PcbKsArgs& a, const uint32_t* seed, dim3 g, cudaStream_t s) {
    const size_t sm = RG ? (size_t)a.ndig * 2 * BX * sizeof(uint64_t) : 0;
    switch (a.ndig) {
        case 1: dot_all_f<LOGN, 1, RG><<<g, BX, sm, s>>>(a, seed); break;
        case 2: dot_all_f<LOGN, 2, RG><<<g, BX, sm, s>>>(a, seed); break;
        case 3: dot_all_f<LOGN, 3, RG><<<g, BX, sm, s>>>(a, seed); break;
        case 4: dot_all_f<LOGN, 4, RG><<<g, BX, sm, s>>>(a, seed); break;
        default: dot_all_f<LOGN, 0, RG><<<g, BX, sm, s>>>(a, seed);
    }
}

template <int LOGN>
int dot_all_run(const PcbKsArgs* ap, bool narrow, bool f64, const uint32_t* seed, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbKsArgs& a = *ap;
    if (a.K < 0 || a.R != 1 || a.ndig < 1 || a.ndig > 16 || a.nrows < 0 || (a.c0_mode & 3) == 3 ||
        (a.c0_mode & ~(3 | PCB_KS_ACC)) || !a.c1 || !a.out0 || !a.out1 || !a.kb || (!a.ka && !seed) || !a.autok ||
        !a.rows || !a.digit_of || !a.pr)
        return PCB_BAD_ARGS;
    if ((a.c0_mode & 3) && !a.c0) return PCB_BAD_ARGS;
    if ((a.c0_mode & 3) == 1 && (!a.pmod || !a.pmods)) return PCB_BAD_ARGS;
    if (a.ndig > 1 && !a.modup) return PCB_BAD_ARGS;
    if (a.K == 0 || a.nrows == 0) return 0;
    const dim3 g((1 << LOGN) / BX, a.nrows);
    if (f64) {  // two words per thread, 16-byte loads: row bases 16-byte aligned, strides even
        // (kb / ka are device arrays of key pointers, not readable here: the evaluator's keys are arena rows,
        // 256-byte aligned)
        const bool odd = (a.ct_stride | a.mu_ct_stride | a.mu_digit_stride | a.key_digit_stride) & 1;
        const uintptr_t bases = (uintptr_t)a.c1 | (uintptr_t)a.modup;
        if (odd || (bases & 15)) return PCB_BAD_ARGS;
        const dim3 gf((1 << LOGN) / (2 * BX), a.nrows);
        seed ? dot_dispatch_f<LOGN, true>(a, seed, gf, s) : dot_dispatch_f<LOGN, false>(a, nullptr, gf, s);
    } else if (narrow) {
        seed ? dot_dispatch<LOGN, true, true>(a, seed, g, s) : dot_dispatch<LOGN, true, false>(a, nullptr, g, s);
    } else {
        seed ? dot_dispatch<LOGN, false, true>(a, seed, g, s) : dot_dispatch<LOGN, false, false>(a, nullptr, g, s);
    }
    return PCB_LAUNCH_RESULT();
}

template int dot_sum_run<14>(const PcbKsArgs*, const KeySum&, cudaStream_t);
template int dot_sum_run<16>(const PcbKsArgs*, const KeySum&, cudaStream_t);
template int dot_keys_run<14>(const PcbKsArgs*, const KeyGroup&, cudaStream_t);
template int dot_keys_run<16>(const PcbKsArgs*, const KeyGroup&, cudaStream_t);
template int dot_all_run<14>(const PcbKsArgs*, bool, bool, const uint32_t*, cudaStream_t);
template int dot_all_run<16>(const PcbKsArgs*, bool, bool, const uint32_t*, cudaStream_t);
template int bconv_launch<14>(const PcbBconvArgs*, cudaStream_t);
template int bconv_launch<16>(const PcbBconvArgs*, cudaStream_t);
template int bconv_run<14>(const PcbBconvArgs*, bool, bool, int, cudaStream_t);
template int bconv_run<16>(const PcbBconvArgs*, bool, bool, int, cudaStream_t);
template int ks_dot_launch<14>(const PcbKsArgs*, cudaStream_t);
template int ks_dot_launch<16>(const PcbKsArgs*, cudaStream_t);
template int ks_dot_run<14>(const PcbKsArgs*, bool, cudaStream_t);
template int ks_dot_run<16>(const PcbKsArgs*, bool, cudaStream_t);

}  // namespace ks
}  // namespace pcb
