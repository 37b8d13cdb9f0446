// Negacyclic NTT / INTT of 64-bit RNS rows on sm_100a.
//
// Transform (crates/pc-kernels/kernels/args.cuh:67-107; host twin crates/pc-host/src/ntt.rs:85-130): OpenFHE order,
// Cooley-Tukey forward to bit-reversed output with twiddles w[m + i] = psi^brev(m + i), Gentleman-Sande inverse with
// psi^-brev and N^-1 (or a per-row factor) folded into its last pass. Canonical words in and out.
//
// B200 design. A row of N = 2^LOGN words is viewed as R = N / 256 "columns" x 256: stages 0 .. A-1 (A = LOGN - 8,
// butterfly spans >= 256 words) run in the column pass, the last 8 stages (spans 128 .. 1) in the row pass over
// 256-word blocks. Each pass keeps 16 (or 8) words per thread in registers and does two register rounds of 4 (or 3)
// stages around one shared-memory exchange, so a pass reads and writes HBM once. Launches go in chunks of rows,
// both passes of a chunk back to back, so the intermediate state stays in the 126 MB L2.
//
// Two arithmetics, one kernel body (template flag F):
//  - integer (any p < 2^62): Harvey-lazy butterflies (words in [0, 4p) forward, [0, 2p) inverse) with Shoup
//    twiddles w' = floor(w 2^64 / p); 64-bit products are emulated on the 32-bit integer multiplier.
//  - FP64 (every prime of the launch below 2^50): words are integer-valued doubles, signed and lazy (|x| < 4p), and
//    a product y w mod p is six FP64 operations, exact (mul_f). The B200 retires 64 FP64 FMAs per clock per SM;
//    this butterfly measured 2.4x the integer one. Twiddles are pairs {w, fl(w / p)} with w centred (|w| <= p/2);
//    the intermediate between the passes is stored as raw doubles.
//    The row pass of this path runs one fixed 256-point transform on every block: block b's stage-l twiddles are
//    w8[2^l + j] gamma_b^(2^(7-l)) (w8: the OpenFHE twiddles of psi^(N/256); gamma_b = psi^c_b with
//    c_b = 1 - 2^(LOGN-8) + 2 brev(b)), which equals the fixed transform of the block pre-multiplied word-wise by
//    gamma_b^k. The column pass applies that twist as it stores (one product per word, coalesced table reads) and
//    the row pass reads its 255 twiddles from shared memory instead of N scattered global ones; the inverse runs the
//    fixed inverse transform, then the inverse twist. Tables per prime: Pack<LOGN>.
#include <type_traits>

#include "arith.cuh"

namespace pcb {
namespace ntt {

constexpr int THREADS = 256;
#ifndef NTT_MIN_BLOCKS
#define NTT_MIN_BLOCKS 3  // at most 80 registers per thread: 24 warps per SM (measured faster than 4 CTAs with spills)
#endif
// CTAs per SM of the FP64 passes (column passes, row passes); 4 fit in 64 registers without spills but measured
// slower on the config-2 step (160.4 and 164.6 ms against 159.8 ms at 3 and 3)
#ifndef NTT_COLS_BLOCKS_F
#define NTT_COLS_BLOCKS_F 3
#endif
#ifndef NTT_ROWS_BLOCKS_F
#define NTT_ROWS_BLOCKS_F 3
#endif

// ------------------------------------------------------------------------------------------------ integer butterflies
__device__ __forceinline__ void ct_bfly(uint64_t& x, uint64_t& y, uint64_t w, uint64_t ws, uint64_t p, uint64_t p2) {
    uint64_t u = x >= p2 ? x - p2 : x;
    const uint64_t v = shoup_lazy(y, w, ws, p);
    x = u + v;
    y = u + p2 - v;
}
__device__ __forceinline__ void gs_bfly(uint64_t& x, uint64_t& y, uint64_t w, uint64_t ws, uint64_t p, uint64_t p2) {
    const uint64_t u = x, v = y;
    uint64_t s = u + v;
    x = s >= p2 ? s - p2 : s;
    y = shoup_lazy(u + p2 - v, w, ws, p);
}
__device__ __forceinline__ uint64_t canon4(uint64_t x, uint64_t p) {
    const uint64_t p2 = 2 * p;
    x = x >= p2 ? x - p2 : x;
    return x >= p ? x - p : x;
}

// ------------------------------------------------------------------------------------------------ arithmetic policy
// Mod<F>: the per-row constants; Word<F>: the register word. Forward words grow by 0.75p per FP64 stage, so each
// round of <= 4 stages starts reduced (|x| <= p); inverse sums double per stage, so even stages reduce them.
struct IntMod {
    uint64_t p, p2;
};
struct FpMod {
    double p, pinv;
};
template <bool F> using Mod = std::conditional_t<F, FpMod, IntMod>;
template <bool F> using Word = std::conditional_t<F, double, uint64_t>;

template <bool F>
__device__ __forceinline__ Word<F> from_u64(uint64_t x) {
    if constexpr (F) return to_f(x);
    else return x;
}
// the intermediate between the passes, kept in the row's own words
template <bool F>
__device__ __forceinline__ Word<F> load_mid(const uint64_t* a) {
    if constexpr (F) return __longlong_as_double((long long)*a);
    else return *a;
}
template <bool F>
__device__ __forceinline__ void store_mid(uint64_t* a, Word<F> x) {
    if constexpr (F) *a = (uint64_t)__double_as_longlong(x);
    else *a = x;
}
// a twiddle: {w, w'} (integer, Shoup companion) or {w, fl(w / p)} (FP64)
template <bool F> using Tw = std::conditional_t<F, double2, ulonglong2>;
__device__ __forceinline__ void ct(uint64_t& x, uint64_t& y, ulonglong2 t, const IntMod& m) {
    ct_bfly(x, y, t.x, t.y, m.p, m.p2);
}
__device__ __forceinline__ void ct(double& x, double& y, double2 t, const FpMod& m) {
    const double v = mul_f(y, t.x, t.y, m.p), u = x;
    x = __dadd_rn(u, v);
    y = __dsub_rn(u, v);
}
__device__ __forceinline__ void gs(uint64_t& x, uint64_t& y, ulonglong2 t, const IntMod& m, bool) {
    gs_bfly(x, y, t.x, t.y, m.p, m.p2);
}
__device__ __forceinline__ void gs(double& x, double& y, double2 t, const FpMod& m, bool reduce) {
    const double s = __dadd_rn(x, y), d = __dsub_rn(x, y);
    x = reduce ? red_f(s, m.p, m.pinv) : s;
    y = mul_f(d, t.x, t.y, m.p);
}
__device__ __forceinline__ ulonglong2 tw_int(const uint64_t* w, const uint64_t* ws, int idx) {
    return make_ulonglong2(__ldg(w + idx), __ldg(ws + idx));
}

// FP64 twiddle pack of one prime (forward and inverse each), in doubles: R + 256 pairs {w, fl(w / p)} — the column
// stages' twiddles (pair indices 0 .. R-1) and the fixed 256-point transform's (R .. R+255) — then the N twist factors
// gamma_b^k (forward) or gamma_b^-k (inverse) at TWIST_D + b 256 + k as single centred doubles: their quotients by p
// are formed as fl(w fl(1 / p)) at use (relative error <= 2^-52; the product y w with |y| < 4p then stays within
// [-p, p], see mul_f), which halves the table each column pass re-reads per row.
template <int LOGN>
struct Pack {
    static constexpr int R = 1 << (LOGN - 8), ROW = R;
    static constexpr int TWIST_D = 2 * (R + 256), SIZE_D = TWIST_D + (1 << LOGN);
};
// the row's pack: pairs (double2 view) and the twist factors
template <int LOGN>
__device__ __forceinline__ const double2* pack_pairs(const void* tw, int pid) {
    return (const double2*)((const double*)tw + (size_t)pid * Pack<LOGN>::SIZE_D);
}
template <int LOGN>
__device__ __forceinline__ const double* pack_twist(const void* tw, int pid) {
    return (const double*)tw + (size_t)pid * Pack<LOGN>::SIZE_D + Pack<LOGN>::TWIST_D;
}
// Shared-memory slot of fixed twiddle t. Stages whose twiddle varies with the thread (4 .. 7 forward, 0 .. 3
// inverse) read region [2^e, 2^(e+1)) at offset u 2^(e-4) + j; stored as [j][u], 16 threads read consecutive slots.
// The per-row constants: FP64 takes fl(1 / p) from entry 0 of the row's pack ({1, fl(1 / p)}: twiddle index 0 is
// psi^0 and no stage uses it), which spares every thread a division before its first butterfly
template <int LOGN, bool F>
__device__ __forceinline__ Mod<F> mod_of(uint64_t p, const void* tw, int pid) {
    if constexpr (F) {
        return FpMod{to_f(p), __ldg(&pack_pairs<LOGN>(tw, pid)->y)};
    } else {
        return IntMod{p, 2 * p};
    }
}
__device__ __forceinline__ int tw_slot(int t) {
    if (t < 16) return t;
    const int e = 31 - __clz(t), off = t - (1 << e), sh = e - 4;
    return (1 << e) + ((off & ((1 << sh) - 1)) << 4) + (off >> sh);
}
__device__ __forceinline__ void round_end(uint64_t&, const IntMod&) {}
__device__ __forceinline__ void round_end(double& x, const FpMod& m) { x = red_f(x, m.p, m.pinv); }
// the canonical word, kept in the register word's bits (so the epilogue reuses the registers)
__device__ __forceinline__ void canon(uint64_t& x, const IntMod& m) { x = canon4(x, m.p); }
__device__ __forceinline__ void canon(double& x, const FpMod& m) {
    x = __longlong_as_double((long long)canon_f(x, m.p, m.pinv));
}
__device__ __forceinline__ uint64_t bits(uint64_t x) { return x; }
__device__ __forceinline__ uint64_t bits(double x) { return (uint64_t)__double_as_longlong(x); }

// Shared-memory exchange of a 256-word block: one pad word after every 16, so both the strided (u + 16 k) and the
// contiguous (16 u + k) views of a half-warp hit 16 distinct 8-byte bank pairs.
constexpr int BLKPAD = 256 + 16;
__device__ __forceinline__ int pad(int e) { return e + (e >> 4); }

struct RowInfo {
    uint64_t* row;
    int pid;
};

// Rows of a launch: row i at base + roff[i] * N, prime id rprime[i]
template <int LOGN>
__device__ __forceinline__ RowInfo row_of(const PcbNttArgs& a, int i) {
    return RowInfo{(uint64_t*)a.base + ((size_t)a.roff[i] << LOGN), a.rprime[i]};
}

// The first pass's input word: the row itself, or the sum mod p of snum source rows (ABI 11 out-of-place)
template <int LOGN>
__device__ __forceinline__ uint64_t load_in(const PcbNttArgs& a, int i, const uint64_t* row, size_t off, uint64_t p) {
    if (a.soff == nullptr) return row[off];
    const uint64_t* s = (const uint64_t*)a.src + ((size_t)a.soff[i] << LOGN) + off;
    uint64_t v = s[0];
    for (int m = 1; m < a.snum; ++m) v = add_mod(v, s[(size_t)m * a.sstride], p);
    return v;
}

// ------------------------------------------------------------------------------------------------ forward
// Column pass: stages 0 .. A-1 on COLS columns; thread (cc, g) holds rows g + E k (round 1), then E g + k (round 2)
template <int LOGN, bool F>
__global__ void __launch_bounds__(THREADS, F ? NTT_COLS_BLOCKS_F : NTT_MIN_BLOCKS) fwd_cols(PcbNttArgs a, int row0) {
    using T = Word<F>;
    constexpr int A = LOGN - 8, R = 1 << A, H = A / 2, E = 1 << H, COLS = 256 / E;
    __shared__ T sm[R * COLS];
    __shared__ Tw<F> stw[R];  // the column stages use twiddles 1 .. R-1 only
    const int i = row0 + blockIdx.y;
    const RowInfo ri = row_of<LOGN>(a, i);
    const uint64_t p = a.pr[ri.pid].p;
    const Mod<F> md = mod_of<LOGN, F>(p, a.fw, ri.pid);
    const int cc = threadIdx.x % COLS, g = threadIdx.x / COLS;
    const int col = blockIdx.x * COLS + cc;
    const double* twist = nullptr;
    if constexpr (F) {
        const double2* pk = pack_pairs<LOGN>(a.fw, ri.pid);
        for (int t = threadIdx.x; t < R; t += THREADS) stw[t] = pk[t];
        twist = pack_twist<LOGN>(a.fw, ri.pid);
    } else {
        const uint64_t* fw = (const uint64_t*)a.fw + ((size_t)ri.pid << LOGN);
        const uint64_t* fws = (const uint64_t*)a.fws + ((size_t)ri.pid << LOGN);
        for (int t = threadIdx.x; t < R; t += THREADS) stw[t] = make_ulonglong2(fw[t], fws[t]);
    }
    pdl_wait();
    pdl_release();
    T x[E];
#pragma unroll
    for (int k = 0; k < E; ++k) x[k] = from_u64<F>(load_in<LOGN>(a, i, ri.row, (size_t)(g + E * k) * 256 + col, p));
    __syncthreads();
    // round 1: stages 0 .. H-1, rows g + E k: butterfly partners differ in k by E/2, E/4, ..
#pragma unroll
    for (int s = 0; s < H; ++s) {
        const int half = E >> (s + 1);
#pragma unroll
        for (int k = 0; k < E; ++k) {
            if (k & half) continue;
            ct(x[k], x[k + half], stw[(1 << s) + (k >> (H - s))], md);
        }
    }
#pragma unroll
    for (int k = 0; k < E; ++k) {
        round_end(x[k], md);
        sm[(g + E * k) * COLS + cc] = x[k];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < E; ++k) x[k] = sm[(E * g + k) * COLS + cc];
    // round 2: stages H .. A-1, rows E g + k
#pragma unroll
    for (int s = H; s < A; ++s) {
        const int half = E >> (s - H + 1);
#pragma unroll
        for (int k = 0; k < E; ++k) {
            if (k & half) continue;
            ct(x[k], x[k + half], stw[(1 << s) + (g << (s - H)) + (k >> (A - s))], md);
        }
    }
#pragma unroll
    for (int k = 0; k < E; ++k) {
        const size_t w = (size_t)(E * g + k) * 256 + col;  // block E g + k, word col: twist gamma_b^col
        if constexpr (F) {
            const double t = __ldg(twist + w);
            x[k] = mul_f(x[k], t, __dmul_rn(t, md.pinv), md.p);
        }
        store_mid<F>(ri.row + w, x[k]);
    }
}

// A forward epilogue word (args.cuh:82-87) of the transformed word o, the summed source xs and the previous output d:
// 1: (xs - o) s, 2: d + (xs - o) s, 3: xs s + o
__device__ __forceinline__ uint64_t epi_word(int epi, uint64_t xs, uint64_t o, uint64_t d, uint64_t sc, uint64_t scs,
                                             uint64_t p) {
    if (epi == 1) return shoup(sub_mod(xs, o, p), sc, scs, p);
    if (epi == 2) return add_mod(d, shoup(sub_mod(xs, o, p), sc, scs, p), p);
    return add_mod(shoup(xs, sc, scs, p), o, p);
}

// Row pass: the last 8 stages over 256-word blocks, 16 blocks per CTA, 16 threads per block; thread u holds words
// u + 16 k (round 1) then 16 u + k (round 2, 16 consecutive words: vector stores and the epilogue)
template <int LOGN, bool F, int EPI>
__global__ void __launch_bounds__(THREADS, F ? NTT_ROWS_BLOCKS_F : NTT_MIN_BLOCKS) fwd_rows(PcbNttArgs a, int row0) {
    using T = Word<F>;
    constexpr int A = LOGN - 8;
    __shared__ T sm[16 * BLKPAD];
    __shared__ double2 sw[F ? 256 : 1];  // FP64: the fixed transform's twiddles, slots tw_slot(t)
    const int i = row0 + blockIdx.y;
    const RowInfo ri = row_of<LOGN>(a, i);
    const uint64_t p = a.pr[ri.pid].p;
    const Mod<F> md = mod_of<LOGN, F>(p, a.fw, ri.pid);
    const uint64_t* fw = (const uint64_t*)a.fw + ((size_t)ri.pid << LOGN);
    const uint64_t* fws = (const uint64_t*)a.fws + ((size_t)ri.pid << LOGN);
    if constexpr (F) sw[tw_slot(threadIdx.x)] = pack_pairs<LOGN>(a.fw, ri.pid)[Pack<LOGN>::ROW + threadIdx.x];
    const int lb = threadIdx.x / 16, u = threadIdx.x % 16;
    const int b = blockIdx.x * 16 + lb;  // 256-word block of the row
    uint64_t* blk = ri.row + (size_t)b * 256;
    pdl_wait();
    pdl_release();
    if constexpr (EPI != 0) {
        // the epilogue's rows (this thread's 16 words = one 128-byte line of each) are read only after the
        // butterflies: start moving them into L2 now
        const size_t r = ((size_t)a.roff[i] << LOGN) + (size_t)b * 256 + 16 * u;
        for (int j = 0; j < a.xnum; ++j) prefetch_l2((const uint64_t*)a.ex + r + (size_t)j * a.xstride);
        if (EPI == 2) prefetch_l2(a.ed ? (const uint64_t*)a.ed + r : (const uint64_t*)a.eout + r);
    }
    T x[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = load_mid<F>(blk + u + 16 * k);
    if constexpr (F) __syncthreads();
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        const int half = 16 >> (l + 1);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (k & half) continue;
            if constexpr (F) ct(x[k], x[k + half], sw[(1 << l) + (k >> (4 - l))], md);
            else ct(x[k], x[k + half], tw_int(fw, fws, (1 << (A + l)) + (b << l) + (k >> (4 - l))), md);
        }
    }
    T* s = sm + lb * BLKPAD;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        round_end(x[k], md);
        s[pad(u + 16 * k)] = x[k];
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = s[pad(16 * u + k)];
#pragma unroll
    for (int l = 4; l < 8; ++l) {
        const int half = 16 >> (l - 3);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (k & half) continue;
            if constexpr (F) ct(x[k], x[k + half], sw[(1 << l) + ((k >> (8 - l)) << 4) + u], md);
            else
                ct(x[k], x[k + half],
                   tw_int(fw, fws, (1 << (A + l)) + (b << l) + (u << (l - 4)) + (k >> (8 - l))), md);
        }
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) canon(x[k], md);
    const size_t w0 = (size_t)b * 256 + 16 * u;  // word offset in the row
    if constexpr (EPI == 0) {
        ulonglong2* op = (ulonglong2*)(blk + 16 * u);
#pragma unroll
        for (int k = 0; k < 8; ++k) op[k] = make_ulonglong2(bits(x[2 * k]), bits(x[2 * k + 1]));
        return;
    }
    // forward epilogues (args.cuh:82-87): x = sum of xnum rows of ex, s = es[prime id]
    // 16-byte accesses: the launcher checks that ex, eout, ed and the row strides keep 16-byte alignment
    const size_t r = ((size_t)a.roff[i] << LOGN) + w0;
    const uint64_t sc = ((const uint64_t*)a.es)[ri.pid], scs = ((const uint64_t*)a.ess)[ri.pid];
    const ulonglong2* ex = (const ulonglong2*)((const uint64_t*)a.ex + r);
    ulonglong2* eo = (ulonglong2*)((uint64_t*)a.eout + r);
    const ulonglong2* ed = a.ed ? (const ulonglong2*)((const uint64_t*)a.ed + r) : eo;
    const size_t xs2 = a.xstride / 2;
    // the words go back to this thread's own exchange slots (read only by it since the exchange) so the epilogue
    // runs as a rolled loop instead of holding all 16 words and their operands in registers
    uint64_t* own = (uint64_t*)s;
#pragma unroll
    for (int k = 0; k < 16; ++k) own[pad(16 * u + k)] = bits(x[k]);
    // the loads of a group of 4 word pairs are all issued before any of them is used (one memory latency per group,
    // not per pair; the rows were prefetched into L2 at the start); groups of 8 spill under the 80-register cap
    constexpr int G = 4;
#pragma unroll 1
    for (int k0 = 0; k0 < 8; k0 += G) {
        ulonglong2 xs[G], d[G];
#pragma unroll
        for (int k = 0; k < G; ++k) {
            xs[k] = ex[k0 + k];
            d[k] = EPI == 2 ? ed[k0 + k] : make_ulonglong2(0, 0);
        }
        for (int j = 1; j < a.xnum; ++j) {
#pragma unroll
            for (int k = 0; k < G; ++k) {
                const ulonglong2 t = ex[k0 + k + (size_t)j * xs2];
                xs[k] = make_ulonglong2(add_mod(xs[k].x, t.x, p), add_mod(xs[k].y, t.y, p));
            }
        }
#pragma unroll
        for (int k = 0; k < G; ++k) {
            const int kk = k0 + k;
            eo[kk] = make_ulonglong2(epi_word(EPI, xs[k].x, own[pad(16 * u + 2 * kk)], d[k].x, sc, scs, p),
                                     epi_word(EPI, xs[k].y, own[pad(16 * u + 2 * kk + 1)], d[k].y, sc, scs, p));
        }
    }
}

// ------------------------------------------------------------------------------------------------ inverse
// Row pass first (GS spans 1 .. 128 inside 256-word blocks); thread u holds 16 u + k (round 1), then u + 16 k
template <int LOGN, bool F>
__global__ void __launch_bounds__(THREADS, F ? NTT_ROWS_BLOCKS_F : NTT_MIN_BLOCKS) inv_rows(PcbNttArgs a, int row0) {
    using T = Word<F>;
    constexpr int N = 1 << LOGN;
    __shared__ T sm[16 * BLKPAD];
    __shared__ double2 sw[F ? 256 : 1];  // FP64: the fixed inverse transform's twiddles, slots tw_slot(t)
    const int i = row0 + blockIdx.y;
    const RowInfo ri = row_of<LOGN>(a, i);
    const uint64_t p = a.pr[ri.pid].p;
    const Mod<F> md = mod_of<LOGN, F>(p, a.iw, ri.pid);
    const uint64_t* iw = (const uint64_t*)a.iw + ((size_t)ri.pid << LOGN);
    const uint64_t* iws = (const uint64_t*)a.iws + ((size_t)ri.pid << LOGN);
    const double* twist = nullptr;
    if constexpr (F) {
        sw[tw_slot(threadIdx.x)] = pack_pairs<LOGN>(a.iw, ri.pid)[Pack<LOGN>::ROW + threadIdx.x];
        twist = pack_twist<LOGN>(a.iw, ri.pid);
    }
    const int lb = threadIdx.x / 16, u = threadIdx.x % 16;
    const int b = blockIdx.x * 16 + lb;
    uint64_t* blk = ri.row + (size_t)b * 256;
    pdl_wait();
    pdl_release();
    T x[16];
    if (a.soff == nullptr) {  // 16 consecutive words: 16-byte loads
        const ulonglong2* v = (const ulonglong2*)(blk + 16 * u);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const ulonglong2 t = v[k];
            x[2 * k] = from_u64<F>(t.x);
            x[2 * k + 1] = from_u64<F>(t.y);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) x[k] = from_u64<F>(load_in<LOGN>(a, i, ri.row, (size_t)b * 256 + 16 * u + k, p));
    }
    if constexpr (F) __syncthreads();
    // spans h = 1, 2, 4, 8: group index j / (2h), m = N / (2h)
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        const int h = 1 << l;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (k & h) continue;
            if constexpr (F) gs(x[k], x[k + h], sw[(1 << (7 - l)) + ((k >> (l + 1)) << 4) + u], md, (l & 1) == 0);
            else gs(x[k], x[k + h], tw_int(iw, iws, N / (2 * h) + ((b * 256 + 16 * u + k) >> (l + 1))), md, false);
        }
    }
    T* s = sm + lb * BLKPAD;
#pragma unroll
    for (int k = 0; k < 16; ++k) s[pad(16 * u + k)] = x[k];
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = s[pad(u + 16 * k)];
    // spans h = 16 .. 128: partners differ in k by h / 16
#pragma unroll
    for (int l = 4; l < 8; ++l) {
        const int hk = 1 << (l - 4);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (k & hk) continue;
            if constexpr (F) gs(x[k], x[k + hk], sw[(1 << (7 - l)) + (k >> (l - 3))], md, (l & 1) == 0);
            else gs(x[k], x[k + hk], tw_int(iw, iws, (N >> (l + 1)) + ((b * 256 + u + 16 * k) >> (l + 1))), md, false);
        }
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        if constexpr (F) {  // the inverse twist gamma_b^-k of word u + 16 k
            const double t = __ldg(twist + (size_t)b * 256 + u + 16 * k);
            x[k] = mul_f(x[k], t, __dmul_rn(t, md.pinv), md.p);
        }
        store_mid<F>(blk + u + 16 * k, x[k]);
    }
}

// Column pass: spans 256 .. N/2, then the row's last-pass factor (N^-1, or es[i] with ess[i])
template <int LOGN, bool F>
__global__ void __launch_bounds__(THREADS, F ? NTT_COLS_BLOCKS_F : NTT_MIN_BLOCKS) inv_cols(PcbNttArgs a, int row0) {
    using T = Word<F>;
    constexpr int A = LOGN - 8, R = 1 << A, H = A / 2, E = 1 << H, COLS = 256 / E;
    __shared__ T sm[R * COLS];
    __shared__ Tw<F> stw[R];  // the column stages use twiddles 1 .. R-1 only
    const int i = row0 + blockIdx.y;
    const RowInfo ri = row_of<LOGN>(a, i);
    const uint64_t p = a.pr[ri.pid].p;
    const Mod<F> md = mod_of<LOGN, F>(p, a.iw, ri.pid);
    const int cc = threadIdx.x % COLS, g = threadIdx.x / COLS;
    const int col = blockIdx.x * COLS + cc;
    if constexpr (F) {
        const double2* pk = pack_pairs<LOGN>(a.iw, ri.pid);
        for (int t = threadIdx.x; t < R; t += THREADS) stw[t] = pk[t];
    } else {
        const uint64_t* iw = (const uint64_t*)a.iw + ((size_t)ri.pid << LOGN);
        const uint64_t* iws = (const uint64_t*)a.iws + ((size_t)ri.pid << LOGN);
        for (int t = threadIdx.x; t < R; t += THREADS) stw[t] = make_ulonglong2(iw[t], iws[t]);
    }
    pdl_wait();
    pdl_release();
    T x[E];
    // round 1: row spans 1 .. E/2 (word spans 256 ..) on rows E g + k
#pragma unroll
    for (int k = 0; k < E; ++k) x[k] = load_mid<F>(ri.row + (size_t)(E * g + k) * 256 + col);
    __syncthreads();
#pragma unroll
    for (int l = 0; l < H; ++l) {
        const int hk = 1 << l;
#pragma unroll
        for (int k = 0; k < E; ++k) {
            if (k & hk) continue;
            gs(x[k], x[k + hk], stw[(R >> (l + 1)) + ((E * g + k) >> (l + 1))], md, (l & 1) == 0);
        }
    }
#pragma unroll
    for (int k = 0; k < E; ++k) sm[(E * g + k) * COLS + cc] = x[k];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < E; ++k) x[k] = sm[(g + E * k) * COLS + cc];
    // round 2: row spans E .. R/2 on rows g + E k: partners differ in k by span / E
#pragma unroll
    for (int l = H; l < A; ++l) {
        const int hk = 1 << (l - H);
#pragma unroll
        for (int k = 0; k < E; ++k) {
            if (k & hk) continue;
            gs(x[k], x[k + hk], stw[(R >> (l + 1)) + ((g + E * k) >> (l + 1))], md, (l & 1) == 0);
        }
    }
    uint64_t ni, nis;
    if (a.es) {
        ni = ((const uint64_t*)a.es)[i];
        nis = ((const uint64_t*)a.ess)[i];
    } else {
        ni = ((const uint64_t*)a.ninv)[ri.pid];
        nis = ((const uint64_t*)a.ninvs)[ri.pid];
    }
    if constexpr (F) {
        // the row's factor as a centred double, its quotient by p as fl(nc fl(1 / p)) (relative error 2^-52: the
        // product lies in [-p, p], made canonical right after)
        const double nc = ni > p / 2 ? -to_f(p - ni) : to_f(ni), np = __dmul_rn(nc, md.pinv);
#pragma unroll
        for (int k = 0; k < E; ++k)
            ri.row[(size_t)(g + E * k) * 256 + col] = canon_f(mul_f(x[k], nc, np, md.p), md.p, md.pinv);
    } else {
#pragma unroll
        for (int k = 0; k < E; ++k) ri.row[(size_t)(g + E * k) * 256 + col] = shoup(x[k], ni, nis, p);
    }
}

#include "ntt_pipe.cuh"

// ------------------------------------------------------------------------------------------------ launchers
// Rows per chunk: both passes of a chunk run back to back so the intermediate state is read back from L2. The count
// is a whole number of waves (the column pass's CTAs of the chunk fill every SM's NTT_MIN_BLOCKS slots exactly, so
// no SM idles in a last partial wave) within ~56 MiB of rows, else ~48 MiB. B200, N = 2^16: 111 rows (4 waves of
// 148 x 3 CTAs); measured 1.6 % faster on the config-2 step than 96 rows.
template <int LOGN>
__host__ int chunk_rows(const PcbNttArgs& a) {
    if (a.chunk > 0) return a.chunk;
    constexpr int COLS = 256 / (1 << ((LOGN - 8) / 2)), CTAS_ROW = 256 / COLS;
    const int cap = (int)((56u << 20) >> (LOGN + 3));
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) ==
                                                  cudaSuccess && sms > 0) {
        const int slots = sms * NTT_MIN_BLOCKS;
        int g = slots, b = CTAS_ROW;
        while (b) {
            const int t = g % b;
            g = b;
            b = t;
        }
        const int r0 = slots / g;  // the fewest rows whose CTAs make whole waves
        if (r0 <= cap) return cap / r0 * r0;
    }
    const int per = (int)((48u << 20) >> (LOGN + 3));
    return per < 1 ? 1 : per;
}

// The row passes move 16 bytes at a time: rows (and the epilogue's rows) must start on 16-byte boundaries
__host__ inline bool misaligned(const void* p) { return ((uintptr_t)p & 15) != 0; }

// The row pass specialized on the launch's epilogue
template <int LOGN, bool F>
__host__ void launch_rows(const PcbNttArgs& a, dim3 grid, cudaStream_t s, int r0);

// fwd_rows_md's dynamic shared memory exceeds the default 48 KiB: raised once per device on its first launch
template <int LOGN>
__host__ void md_smem_once() {
    constexpr int MAXDEV = 64;
    static bool done[MAXDEV] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAXDEV) dev = 0;
    if (!done[dev]) {
        cudaFuncSetAttribute(fwd_rows_md<LOGN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MD_SMEM);
        done[dev] = true;
    }
}

template <int LOGN, bool F>
__host__ void launch_rows(const PcbNttArgs& a, dim3 grid, cudaStream_t s, int r0) {
    if constexpr (F && LOGN == 16) {
        if (a.epi == 1 && a.xnum == 1) {  // ModDown: the epilogue's tile staged by a bulk copy (ntt_pipe.cuh)
            md_smem_once<LOGN>();
            launch_pdl_smem(fwd_rows_md<LOGN>, grid, dim3(THREADS), MD_SMEM, s, a, r0);
            return;
        }
    }
    switch (a.epi) {
        case 0: launch_pdl(fwd_rows<LOGN, F, 0>, grid, dim3(THREADS), s, a, r0); break;
        case 1: launch_pdl(fwd_rows<LOGN, F, 1>, grid, dim3(THREADS), s, a, r0); break;
        case 2: launch_pdl(fwd_rows<LOGN, F, 2>, grid, dim3(THREADS), s, a, r0); break;
        default: launch_pdl(fwd_rows<LOGN, F, 3>, grid, dim3(THREADS), s, a, r0);
    }
}

// The pipelined FP64 inverse row pass (ntt_pipe.cuh): N = 2^16, the source read from at most one row, bulk copies
// starting on 16-byte boundaries (the row bases, and the out-of-place source when there is one)
template <int LOGN>
__host__ bool pipelined(const PcbNttArgs& a, bool f64) {
    return f64 && LOGN == 16 && !misaligned(a.base) && (a.soff == nullptr || (a.snum <= 1 && !misaligned(a.src)));
}

// Their dynamic shared memory exceeds the default 48 KiB: raised once per kernel and device (on the first launch,
// which should come before any stream capture); a persistent grid of PIPE_CTAS_PER_SM CTAs per SM, at most one per tile
template <auto KERN>
__host__ int pipe_grid(int tiles) {
    constexpr int MAXDEV = 64;
    static int sms[MAXDEV] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAXDEV) dev = 0;
    if (sms[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
        cudaFuncSetAttribute(KERN, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PIPE_SMEM);
        sms[dev] = n;
    }
    const int g = sms[dev] * PIPE_CTAS_PER_SM;
    return tiles < g ? tiles : g;
}

template <int LOGN>
int fwd_run(const PcbNttArgs* ap, bool f64, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbNttArgs a = *ap;
    if (a.nrows < 0 || a.epi < 0 || a.epi > 3 || !a.base || !a.roff || !a.rprime || !a.fw || !a.fws || !a.pr)
        return PCB_BAD_ARGS;
    if (a.epi != 0 && (!a.eout || !a.ex || !a.es || !a.ess)) return PCB_BAD_ARGS;
    if (misaligned(a.base) || (a.epi != 0 && (misaligned(a.eout) || misaligned(a.ex) || misaligned(a.ed) ||
                                              (a.xnum > 1 && (a.xstride & 1)))))
        return PCB_BAD_ARGS;
    if (a.soff && (!a.src || a.snum < 1)) return PCB_BAD_ARGS;
    if (a.nrows == 0) return 0;
    constexpr int A = LOGN - 8, COLS = 256 / (1 << (A / 2));
    const int ch = chunk_rows<LOGN>(a);
    for (int r0 = 0; r0 < a.nrows; r0 += ch) {
        const int n = a.nrows - r0 < ch ? a.nrows - r0 : ch;
        if (f64) {
            launch_pdl(fwd_cols<LOGN, true>, dim3(256 / COLS, n), dim3(THREADS), s, a, r0);
            launch_rows<LOGN, true>(a, dim3((1 << A) / 16, n), s, r0);
        } else {
            launch_pdl(fwd_cols<LOGN, false>, dim3(256 / COLS, n), dim3(THREADS), s, a, r0);
            launch_rows<LOGN, false>(a, dim3((1 << A) / 16, n), s, r0);
        }
    }
    return PCB_LAUNCHED(2u * (unsigned)((a.nrows + ch - 1) / ch));
}

template <int LOGN>
int inv_run(const PcbNttArgs* ap, bool f64, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbNttArgs a = *ap;
    if (a.nrows < 0 || a.epi != 0 || !a.base || !a.roff || !a.rprime || !a.iw || !a.iws || !a.pr) return PCB_BAD_ARGS;
    if (misaligned(a.base)) return PCB_BAD_ARGS;
    if (!a.es && (!a.ninv || !a.ninvs)) return PCB_BAD_ARGS;
    if (a.es && !a.ess) return PCB_BAD_ARGS;
    if (a.soff && (!a.src || a.snum < 1)) return PCB_BAD_ARGS;
    if (a.nrows == 0) return 0;
    constexpr int A = LOGN - 8, COLS = 256 / (1 << (A / 2));
    const int ch = chunk_rows<LOGN>(a);
    const bool pipe = pipelined<LOGN>(a, f64);
    for (int r0 = 0; r0 < a.nrows; r0 += ch) {
        const int n = a.nrows - r0 < ch ? a.nrows - r0 : ch;
        if (pipe) {
            if constexpr (LOGN == 16) {
                const int tiles = n * (256 / 16);
                launch_pdl_smem(inv_rows_p<LOGN>, dim3(pipe_grid<inv_rows_p<LOGN>>(tiles)), dim3(THREADS), PIPE_SMEM, s,
                                a, r0, n);
                launch_pdl(inv_cols<LOGN, true>, dim3(256 / COLS, n), dim3(THREADS), s, a, r0);
            }
        } else if (f64) {
            launch_pdl(inv_rows<LOGN, true>, dim3((1 << A) / 16, n), dim3(THREADS), s, a, r0);
            launch_pdl(inv_cols<LOGN, true>, dim3(256 / COLS, n), dim3(THREADS), s, a, r0);
        } else {
            launch_pdl(inv_rows<LOGN, false>, dim3((1 << A) / 16, n), dim3(THREADS), s, a, r0);
            launch_pdl(inv_cols<LOGN, false>, dim3(256 / COLS, n), dim3(THREADS), s, a, r0);
        }
    }
    return PCB_LAUNCHED(2u * (unsigned)((a.nrows + ch - 1) / ch));
}

// The table entries take the reference's integer twiddle tables (w, Shoup w')
template <int LOGN>
int fwd(const PcbNttArgs* ap, cudaStream_t s) {
    return fwd_run<LOGN>(ap, false, s);
}
template <int LOGN>
int inv(const PcbNttArgs* ap, cudaStream_t s) {
    return inv_run<LOGN>(ap, false, s);
}

// waits of the pipelined passes that ran out on the current device (0 unless a bulk copy never completed)
__host__ unsigned int device_timeouts() {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof v) != cudaSuccess) return ~0u;
    return v;
}

template int fwd<14>(const PcbNttArgs*, cudaStream_t);
template int fwd<16>(const PcbNttArgs*, cudaStream_t);
template int inv<14>(const PcbNttArgs*, cudaStream_t);
template int inv<16>(const PcbNttArgs*, cudaStream_t);
template int fwd_run<14>(const PcbNttArgs*, bool, cudaStream_t);
template int fwd_run<16>(const PcbNttArgs*, bool, cudaStream_t);
template int inv_run<14>(const PcbNttArgs*, bool, cudaStream_t);
template int inv_run<16>(const PcbNttArgs*, bool, cudaStream_t);

}  // namespace ntt
}  // namespace pcb

// Waits of the pipelined transforms that ran out on the current device since the library was loaded (0 in normal
// operation; each stopped one CTA, whose rows were then left untransformed).
extern "C" uint32_t pcb_device_timeouts(void) { return pcb::ntt::device_timeouts(); }
