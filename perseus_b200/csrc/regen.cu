// Key inner products with the switching key's `a` regenerated in the kernel (the reference's Regen key source): the
// key is stored as `b` and an 8-word seed, half the bytes of a dense key, and `a` comes back from the frozen u64
// expander lane (chacha.cuh) for (seed, digit, the row's prime). Semantics of crates/pc-kernels/kernels/args.cuh
// (KsRegenArgs :285-304, KeyTab :273-283, KsKeyArgs :764-768) and crates/pc-kernels/kernels/ks.cuh (ks_dot_regen
// :130-215, ks_dot_key :218-300).
//
// Each thread owns 4 consecutive slots of one row: per digit it computes the ChaCha block of its 8-slot group and
// keeps its half, loads `b` and the K ciphertexts' digit words 16 bytes at a time, and sums the products in 128 bits
// with one reduction at the end, so the outputs are the canonical residues of the exact sums (any prime below 2^62).
#include "chacha.cuh"
#include "kernels.h"

namespace pcb {
namespace regen {

constexpr int BX = 128;

struct W4 {
    uint64_t v[4];
};
__device__ __forceinline__ W4 ld4(const uint64_t* p) {
    const ulonglong2 a = __ldg((const ulonglong2*)p), b = __ldg((const ulonglong2*)p + 1);
    return W4{{a.x, a.y, b.x, b.y}};
}
// key rows reached through device pointer tables, whose alignment the host cannot check: 16-byte loads when the row
// start allows them, else 8-byte ones
__device__ __forceinline__ W4 ld4k(const uint64_t* p) {
    if (((uintptr_t)p & 15) == 0) return ld4(p);
    return W4{{__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3)}};
}
__device__ __forceinline__ void st4(uint64_t* p, const uint64_t (&r)[4]) {
    ((ulonglong2*)p)[0] = make_ulonglong2(r[0], r[1]);
    ((ulonglong2*)p)[1] = make_ulonglong2(r[2], r[3]);
}

// the key's slot of prime id t: Q ids at their index up to q_top, special ids after them; q_top < 0: the prime id
__device__ __forceinline__ int slot_of(const PcbKeyTab& T, int t, int nq) {
    return (t < nq || T.q_top < 0) ? t : T.q_top + 1 + (t - nq);
}

// ------------------------------------------------------------------------------------------------ ks_dot_regen
// TAB: the `b` rows come from key 0 of G.key (dense rows in the key's slot order) instead of ks.kb[0]
template <int LOGN, int KMAX, bool EPI, bool TAB>
__global__ void __launch_bounds__(BX) ks_dot_regen(PcbKsRegenArgs G) {
    const PcbKsArgs& A = G.ks;
    const uint32_t t = A.rows[blockIdx.y];
    const PcbPrimeConst& pc = A.pr[t];
    const uint64_t p = pc.p;
    const uint32_t gtid = blockIdx.x * BX + threadIdx.x;
    const uint32_t base = gtid * 4;
    const int dt = (int)t < A.nq ? A.digit_of[t] : -1;
    const size_t roff = ((size_t)t << LOGN) + base;
    const uint64_t* c1 = (const uint64_t*)A.c1;
    const uint64_t* mu = (const uint64_t*)A.modup;
    const uint64_t* kb;
    size_t brow0, bstride;  // word offset of digit 0's row (from the row base) and the digits' stride
    if constexpr (TAB) {
        kb = (const uint64_t*)G.key.kb[0];
        brow0 = (size_t)slot_of(G.key, (int)t, A.nq) * G.key.row_words;
        bstride = (size_t)G.key.srows * G.key.row_words;
    } else {
        kb = (const uint64_t*)A.kb[0];
        brow0 = (size_t)t << LOGN;
        bstride = A.key_digit_stride;
    }
    Acc s0[KMAX][4], s1[KMAX][4];
#pragma unroll
    for (int c = 0; c < KMAX; ++c)
#pragma unroll
        for (int w = 0; w < 4; ++w) s0[c][w] = s1[c][w] = Acc{0, 0};
    for (int d = 0; d < A.ndig; ++d) {
        uint64_t a4[4];
        keys::expand4<LOGN>(G.seed, gtid >> 1, gtid & 1, (uint32_t)d, keys::TAG_KSKA, pc, a4);
        const W4 b4 = ld4k(kb + brow0 + (size_t)d * bstride + base);
#pragma unroll
        for (int c = 0; c < KMAX; ++c) {
            if (c < A.K) {
                const W4 x4 = d == dt ? ld4(c1 + (size_t)c * A.ct_stride + roff)
                                      : ld4(mu + (size_t)c * A.mu_ct_stride + (size_t)d * A.mu_digit_stride + roff);
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    mac(s0[c][w], x4.v[w], b4.v[w]);
                    mac(s1[c][w], x4.v[w], a4[w]);
                }
            }
        }
    }
    const PcbEpiArgs& E = G.epi;
#pragma unroll
    for (int c = 0; c < KMAX; ++c) {
        if (c < A.K) {
            uint64_t r0[4], r1[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                r0[w] = reduce(s0[c][w], pc);
                r1[w] = reduce(s1[c][w], pc);
            }
            const size_t ob = (size_t)c * A.out_ct_stride + ((size_t)t << LOGN) + base;
            if constexpr (EPI) {
                // dst = f (alpha dst + (dot - conv) binv) [+ k on part 0] [+ add] (args.cuh:258-271, :285-304)
                const uint64_t bi = ((const uint64_t*)E.binv)[t], bis = ((const uint64_t*)E.binvs)[t];
                const uint64_t* kp = (const uint64_t*)E.k;
                const uint64_t kk = kp ? (kp[t] >= p ? kp[t] - p : kp[t]) : 0;
                const uint64_t* al = (const uint64_t*)E.alpha;
                const uint64_t ai = al ? al[t] : 0, ais = al ? ((const uint64_t*)E.alphas)[t] : 0;
#pragma unroll
                for (int part = 0; part < 2; ++part) {
                    uint64_t* dp = (uint64_t*)E.dst + ob + part * E.part_stride;
                    const W4 cv = ld4((const uint64_t*)E.conv + ob + part * E.part_stride);
                    const W4 dv = ld4(dp);
                    W4 av{};
                    if (G.add) av = ld4((const uint64_t*)G.add + ob + part * E.part_stride);
                    uint64_t r[4];
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        const uint64_t x = part ? r1[w] : r0[w];
                        const uint64_t dd = al ? shoup(dv.v[w], ai, ais, p) : dv.v[w];
                        uint64_t v = add_mod(dd, shoup(sub_mod(x, cv.v[w], p), bi, bis, p), p);
                        if (E.dbl) v = add_mod(v, v, p);
                        if (part == 0) v = add_mod(v, kk, p);
                        if (G.add) v = add_mod(v, av.v[w], p);
                        r[w] = v;
                    }
                    st4(dp, r);
                }
            } else {
                st4((uint64_t*)A.out0 + ob, r0);
                st4((uint64_t*)A.out1 + ob, r1);
            }
        }
    }
}

__host__ inline bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <int LOGN, bool EPI, bool TAB>
void regen_go(const PcbKsRegenArgs& a, cudaStream_t s) {
    const dim3 g((1 << LOGN) / (4 * BX), a.ks.nrows);
    switch (a.ks.K) {
        case 1: ks_dot_regen<LOGN, 1, EPI, TAB><<<g, BX, 0, s>>>(a); break;
        case 2: ks_dot_regen<LOGN, 2, EPI, TAB><<<g, BX, 0, s>>>(a); break;
        default: ks_dot_regen<LOGN, 4, EPI, TAB><<<g, BX, 0, s>>>(a);
    }
}

template <int LOGN>
int ks_dot_regen_launch(const PcbKsRegenArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbKsRegenArgs& a = *ap;
    const PcbKsArgs& k = a.ks;
    const bool tab = a.key.kb != nullptr;
    if (k.K < 0 || k.K > 4 || k.ndig < 1 || k.ndig > 16 || k.nrows < 0 || !k.c1 || !k.rows || !k.digit_of || !k.pr ||
        !a.seed || (k.ndig > 1 && !k.modup))
        return PCB_BAD_ARGS;
    // key.kb / ks.kb are device arrays of device pointers: only the table pointers themselves are checked here
    if (tab ? (a.key.bits != 0 || a.key.srows < 1) : !k.kb) return PCB_BAD_ARGS;
    if (a.use_epi ? (!a.epi.dst || !a.epi.conv || !a.epi.binv || !a.epi.binvs || (a.epi.alpha && !a.epi.alphas) ||
                     !al16(a.epi.dst) || !al16(a.epi.conv) || (a.epi.part_stride & 1) || (a.add && !al16(a.add)))
                  : (!k.out0 || !k.out1 || !al16(k.out0) || !al16(k.out1)))
        return PCB_BAD_ARGS;
    if (!al16(k.c1) || (k.modup && !al16(k.modup)) || (k.ct_stride & 1) || (k.mu_ct_stride & 1) ||
        (k.mu_digit_stride & 1) || (k.out_ct_stride & 1))
        return PCB_BAD_ARGS;
    if (k.K == 0 || k.nrows == 0) return 0;
    if (a.use_epi) tab ? regen_go<LOGN, true, true>(a, s) : regen_go<LOGN, true, false>(a, s);
    else tab ? regen_go<LOGN, false, true>(a, s) : regen_go<LOGN, false, false>(a, s);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ ks_dot_key
template <int LOGN, int KMAX>
__global__ void __launch_bounds__(BX) ks_dot_key(PcbKsKeyArgs G) {
    const PcbKsArgs& A = G.ks;
    const PcbKeyTab& T = G.key;
    const uint32_t t = A.rows[blockIdx.y];
    const PcbPrimeConst& pc = A.pr[t];
    const uint64_t p = pc.p;
    const uint32_t gtid = blockIdx.x * BX + threadIdx.x;
    const uint32_t base = gtid * 4;
    const int dt = (int)t < A.nq ? A.digit_of[t] : -1;
    const size_t roff = ((size_t)t << LOGN) + base;
    const uint64_t* c1 = (const uint64_t*)A.c1;
    const uint64_t* mu = (const uint64_t*)A.modup;
    const uint64_t* c0 = (const uint64_t*)A.c0;
    const size_t brow0 = (size_t)slot_of(T, (int)t, A.nq) * T.row_words, bstride = (size_t)T.srows * T.row_words;
    uint64_t pm = 0, pms = 0;
    if ((A.c0_mode & 3) == 1 && (int)t < A.nq) {
        pm = ((const uint64_t*)A.pmod)[t];
        pms = ((const uint64_t*)A.pmods)[t];
    }
    for (int r = 0; r < A.R; ++r) {
        Acc s0[KMAX][4], s1[KMAX][4];
#pragma unroll
        for (int c = 0; c < KMAX; ++c)
#pragma unroll
            for (int w = 0; w < 4; ++w) s0[c][w] = s1[c][w] = Acc{0, 0};
        const uint64_t* kb = (const uint64_t*)T.kb[r];
        for (int d = 0; d < A.ndig; ++d) {
            uint64_t a4[4];
            if (d < T.nregen) {
                keys::expand4<LOGN>(T.seed[r], gtid >> 1, gtid & 1, (uint32_t)d, keys::TAG_KSKA, pc, a4);
            } else {  // the resident dense `a` (prime-id rows)
                const W4 av = ld4k((const uint64_t*)A.ka[r] + (size_t)d * A.key_digit_stride + roff);
#pragma unroll
                for (int w = 0; w < 4; ++w) a4[w] = av.v[w];
            }
            const W4 b4 = ld4k(kb + brow0 + (size_t)d * bstride + base);
#pragma unroll
            for (int c = 0; c < KMAX; ++c) {
                if (c < A.K) {
                    const W4 x4 = d == dt ? ld4(c1 + (size_t)c * A.ct_stride + roff)
                                          : ld4(mu + (size_t)c * A.mu_ct_stride + (size_t)d * A.mu_digit_stride + roff);
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        mac(s0[c][w], x4.v[w], b4.v[w]);
                        mac(s1[c][w], x4.v[w], a4[w]);
                    }
                }
            }
        }
        const uint32_t k = A.autok[r];
#pragma unroll
        for (int c = 0; c < KMAX; ++c) {
            if (c < A.K) {
                W4 c04{};
                if (A.c0_mode & 3) c04 = ld4(c0 + (size_t)c * A.ct_stride + roff);
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    uint64_t r0 = reduce(s0[c][w], pc), r1 = reduce(s1[c][w], pc);
                    if ((A.c0_mode & 3) == 1) {
                        if ((int)t < A.nq) r0 = add_mod(r0, shoup(c04.v[w], pm, pms, p), p);
                    } else if ((A.c0_mode & 3) == 2) {
                        r0 = add_mod(r0, c04.v[w], p);
                    }
                    const uint32_t i = base + w;
                    const uint32_t o = k == 1 ? i : automorph_slot<LOGN>(k, i);
                    const size_t ob = (size_t)c * A.out_ct_stride + (size_t)r * A.out_rot_stride + ((size_t)t << LOGN) + o;
                    if (A.c0_mode & PCB_KS_ACC) {
                        r0 = add_mod(r0, ((const uint64_t*)A.out0)[ob], p);
                        r1 = add_mod(r1, ((const uint64_t*)A.out1)[ob], p);
                    }
                    ((uint64_t*)A.out0)[ob] = r0;
                    ((uint64_t*)A.out1)[ob] = r1;
                }
            }
        }
    }
}

template <int LOGN>
int ks_dot_key_launch(const PcbKsKeyArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbKsKeyArgs& a = *ap;
    const PcbKsArgs& k = a.ks;
    const PcbKeyTab& T = a.key;
    if (k.K < 0 || k.K > 4 || k.R < 0 || k.ndig < 1 || k.ndig > 16 || k.nrows < 0 || (k.c0_mode & 3) == 3 ||
        (k.c0_mode & ~(3 | PCB_KS_ACC)) || !k.c1 || !k.out0 || !k.out1 || !k.autok || !k.rows || !k.digit_of || !k.pr ||
        (k.ndig > 1 && !k.modup))
        return PCB_BAD_ARGS;
    if (!T.kb || !T.seed || T.bits != 0 || T.srows < 1 || T.nregen < 0) return PCB_BAD_ARGS;
    if ((k.c0_mode & 3) && !k.c0) return PCB_BAD_ARGS;
    if ((k.c0_mode & 3) == 1 && (!k.pmod || !k.pmods)) return PCB_BAD_ARGS;
    if (T.nregen < k.ndig && !k.ka) return PCB_BAD_ARGS;
    if (!al16(k.c1) || (k.modup && !al16(k.modup)) || (k.c0 && !al16(k.c0)) || (k.ct_stride & 1) ||
        (k.mu_ct_stride & 1) || (k.mu_digit_stride & 1))
        return PCB_BAD_ARGS;
    if (k.K == 0 || k.R == 0 || k.nrows == 0) return 0;
    const dim3 g((1 << LOGN) / (4 * BX), k.nrows);
    switch (k.K) {
        case 1: ks_dot_key<LOGN, 1><<<g, BX, 0, s>>>(a); break;
        case 2: ks_dot_key<LOGN, 2><<<g, BX, 0, s>>>(a); break;
        default: ks_dot_key<LOGN, 4><<<g, BX, 0, s>>>(a);
    }
    return PCB_LAUNCH_RESULT();
}

template int ks_dot_regen_launch<14>(const PcbKsRegenArgs*, cudaStream_t);
template int ks_dot_regen_launch<16>(const PcbKsRegenArgs*, cudaStream_t);
template int ks_dot_key_launch<14>(const PcbKsKeyArgs*, cudaStream_t);
template int ks_dot_key_launch<16>(const PcbKsKeyArgs*, cudaStream_t);

}  // namespace regen
}  // namespace pcb
