// The launcher-table entries whose switching keys come with `a` regenerated in the kernel: ks_dot_regen (the
// relinearization inner product, with its fused ModDown epilogue) and ks_dot_key (ks_dot over keys read through a
// key table). Semantics: crates/pc-kernels/kernels/args.cuh (KsRegenArgs :285-304, EpiArgs :258-271, KeyTab
// :273-283, KsKeyArgs :764-768); any prime below 2^62.
//
// Design (shared with the evaluator's FP64 inner products, keyregen.cuh): a CTA owns a tile of 2 BX consecutive slots
// of one row. For each key it first regenerates that key's `a` over the tile for every regenerated digit into shared
// memory — whole ChaCha12 blocks of 8 slots spread over the CTA's threads — and then each thread takes two adjacent
// slots (16-byte loads of the ciphertexts' digit words) and walks the ciphertexts one at a time: 128-bit sums of the
// digit products for its two slots, one reduction each, the epilogue or the scattered store. The key's `b` words are
// re-read per ciphertext from L1 (the tile's rows are a few KB), so only four accumulators are live per thread.
#include "keyregen.cuh"
#include "kernels.h"

namespace pcb {
namespace regen {

constexpr int BX = 128;
constexpr int TILE = 2 * BX;                     // slots per CTA
constexpr int NSEG = TILE / keyregen::SEG;       // staged segments per digit
constexpr int MAX_DIG = 16;

// two adjacent words at p: one 16-byte load when p allows it (key rows reached through device pointer tables, whose
// alignment the host cannot check), else two 8-byte loads
__device__ __forceinline__ ulonglong2 ld2(const uint64_t* p) {
    if (((uintptr_t)p & 15) == 0) return __ldg((const ulonglong2*)p);
    return make_ulonglong2(__ldg(p), __ldg(p + 1));
}

// Where a key's words of one row live: `b` at bsrc + d bstride, dense `a` (digits >= nreg) at asrc + d astride,
// regenerated `a` (digits < nreg) from seed.
struct KeyRow {
    const uint64_t* bsrc;
    size_t bstride;
    const uint64_t* asrc;
    size_t astride;
    const uint32_t* seed;
    int nreg;
};

// sums over the digits of ciphertext c at slots (i, i + 1) of row t: s0 = sum x_d b_d, s1 = sum x_d a_d
__device__ __forceinline__ void digit_sums(const PcbKsArgs& A, const KeyRow& K, const uint64_t* sm, int c, int dt,
                                           size_t roff, uint32_t tslot, Acc (&s0)[2], Acc (&s1)[2]) {
    const uint64_t* c1 = (const uint64_t*)A.c1;
    const uint64_t* mu = (const uint64_t*)A.modup;
    s0[0] = s0[1] = s1[0] = s1[1] = Acc{0, 0};
    for (int d = 0; d < A.ndig; ++d) {
        const ulonglong2 x = __ldg((const ulonglong2*)(d == dt ? c1 + (size_t)c * A.ct_stride + roff
                                                               : mu + (size_t)c * A.mu_ct_stride +
                                                                     (size_t)d * A.mu_digit_stride + roff));
        const ulonglong2 b = ld2(K.bsrc + (size_t)d * K.bstride);
        const ulonglong2 a = d < K.nreg ? *(const ulonglong2*)&sm[(size_t)d * TILE + tslot]
                                        : ld2(K.asrc + (size_t)d * K.astride);
        mac(s0[0], x.x, b.x);
        mac(s0[1], x.y, b.y);
        mac(s1[0], x.x, a.x);
        mac(s1[1], x.y, a.y);
    }
}

// ------------------------------------------------------------------------------------------------ ks_dot_regen
// TAB: `b` from key 0 of G.key (dense rows in the key's slot order, row_words apart), else ks.kb[0] (prime-id rows)
template <int LOGN, bool EPI, bool TAB>
__global__ void __launch_bounds__(BX) ks_dot_regen(PcbKsRegenArgs G) {
    extern __shared__ __align__(16) uint64_t sm[];
    const PcbKsArgs& A = G.ks;
    const uint32_t t = A.rows[blockIdx.y];
    const PcbPrimeConst& pc = A.pr[t];
    const uint64_t p = pc.p;
    const uint32_t tile0 = blockIdx.x * TILE, tslot = 2 * threadIdx.x, i = tile0 + tslot;
    const size_t roff = ((size_t)t << LOGN) + i;
    const int dt = (int)t < A.nq ? A.digit_of[t] : -1;
    KeyRow K;
    if constexpr (TAB) {
        K.bsrc = (const uint64_t*)G.key.kb[0] + (size_t)keyregen::key_slot(G.key, (int)t, A.nq) * G.key.row_words + i;
        K.bstride = (size_t)G.key.srows * G.key.row_words;
    } else {
        K.bsrc = (const uint64_t*)A.kb[0] + roff;
        K.bstride = A.key_digit_stride;
    }
    K.asrc = nullptr;
    K.astride = 0;
    K.seed = G.seed;
    K.nreg = A.ndig;
    keyregen::stage<LOGN>(&K.seed, 1, A.ndig, NSEG,
                          [tile0](int, int j) { return tile0 + (uint32_t)j * keyregen::SEG; }, pc, sm);
    const PcbEpiArgs& E = G.epi;
    uint64_t bi = 0, bis = 0, kk = 0, al = 0, als = 0;
    if constexpr (EPI) {
        bi = ((const uint64_t*)E.binv)[t];
        bis = ((const uint64_t*)E.binvs)[t];
        if (E.k) {
            const uint64_t kv = ((const uint64_t*)E.k)[t];
            kk = kv >= p ? kv - p : kv;
        }
        if (E.alpha) {
            al = ((const uint64_t*)E.alpha)[t];
            als = ((const uint64_t*)E.alphas)[t];
        }
    }
    for (int c = 0; c < A.K; ++c) {
        Acc s0[2], s1[2];
        digit_sums(A, K, sm, c, dt, roff, tslot, s0, s1);
        const uint64_t r[2][2] = {{reduce(s0[0], pc), reduce(s0[1], pc)}, {reduce(s1[0], pc), reduce(s1[1], pc)}};
        const size_t ob = (size_t)c * A.out_ct_stride + ((size_t)t << LOGN) + i;
        if constexpr (EPI) {
            // dst = f (alpha dst + (dot - conv) binv) [+ k on part 0] [+ add], f = 2 when dbl
            for (int part = 0; part < 2; ++part) {
                const size_t o = ob + (size_t)part * E.part_stride;
                uint64_t* dp = (uint64_t*)E.dst + o;
                const ulonglong2 cv = __ldg((const ulonglong2*)((const uint64_t*)E.conv + o));
                const ulonglong2 dv = *(const ulonglong2*)dp;
                ulonglong2 av = make_ulonglong2(0, 0);
                if (G.add) av = __ldg((const ulonglong2*)((const uint64_t*)G.add + o));
                const uint64_t cw[2] = {cv.x, cv.y}, dw[2] = {dv.x, dv.y}, aw[2] = {av.x, av.y};
                uint64_t v[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint64_t base = E.alpha ? shoup(dw[h], al, als, p) : dw[h];
                    v[h] = add_mod(base, shoup(sub_mod(r[part][h], cw[h], p), bi, bis, p), p);
                    if (E.dbl) v[h] = add_mod(v[h], v[h], p);
                    if (part == 0) v[h] = add_mod(v[h], kk, p);
                    if (G.add) v[h] = add_mod(v[h], aw[h], p);
                }
                *(ulonglong2*)dp = make_ulonglong2(v[0], v[1]);
            }
        } else {
            *(ulonglong2*)((uint64_t*)A.out0 + ob) = make_ulonglong2(r[0][0], r[0][1]);
            *(ulonglong2*)((uint64_t*)A.out1 + ob) = make_ulonglong2(r[1][0], r[1][1]);
        }
    }
}

__host__ inline bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <int LOGN, bool EPI, bool TAB>
void regen_go(const PcbKsRegenArgs& a, cudaStream_t s) {
    const dim3 g((1 << LOGN) / TILE, a.ks.nrows);
    ks_dot_regen<LOGN, EPI, TAB><<<g, BX, (size_t)a.ks.ndig * TILE * sizeof(uint64_t), s>>>(a);
}

template <int LOGN>
int ks_dot_regen_launch(const PcbKsRegenArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbKsRegenArgs& a = *ap;
    const PcbKsArgs& k = a.ks;
    const bool tab = a.key.kb != nullptr;
    if (k.K < 0 || k.K > 4 || k.ndig < 1 || k.ndig > MAX_DIG || k.nrows < 0 || !k.c1 || !k.rows || !k.digit_of ||
        !k.pr || !a.seed || (k.ndig > 1 && !k.modup))
        return PCB_BAD_ARGS;
    // key.kb / ks.kb are device arrays of device pointers: only the table pointers themselves are checked here
    if (tab ? (a.key.bits != 0 || a.key.srows < 1) : !k.kb) return PCB_BAD_ARGS;
    if (a.add && !a.use_epi) return PCB_BAD_ARGS;
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
// ks_dot over R keys read through the key table: key r's `a` regenerated from T.seed[r] for digits below T.nregen
// (staged per key; the CTA re-stages between keys), dense ks.ka[r] rows for the others; outputs scattered to
// automorph_slot(autok[r], i) with the c0 modes and accumulation of ks_dot.
template <int LOGN>
__global__ void __launch_bounds__(BX) ks_dot_key(PcbKsKeyArgs G) {
    extern __shared__ __align__(16) uint64_t sm[];
    const PcbKsArgs& A = G.ks;
    const PcbKeyTab& T = G.key;
    const uint32_t t = A.rows[blockIdx.y];
    const PcbPrimeConst& pc = A.pr[t];
    const uint64_t p = pc.p;
    const uint32_t tile0 = blockIdx.x * TILE, tslot = 2 * threadIdx.x, i = tile0 + tslot;
    const size_t roff = ((size_t)t << LOGN) + i;
    const int dt = (int)t < A.nq ? A.digit_of[t] : -1;
    const int nreg = T.nregen < A.ndig ? T.nregen : A.ndig;
    const uint64_t* c0 = (const uint64_t*)A.c0;
    const int mode = A.c0_mode & 3;
    uint64_t pm = 0, pms = 0;
    if (mode == 1 && (int)t < A.nq) {
        pm = ((const uint64_t*)A.pmod)[t];
        pms = ((const uint64_t*)A.pmods)[t];
    }
    const size_t brow = (size_t)keyregen::key_slot(T, (int)t, A.nq) * T.row_words + i;
    for (int r = 0; r < A.R; ++r) {
        KeyRow K;
        K.bsrc = (const uint64_t*)T.kb[r] + brow;
        K.bstride = (size_t)T.srows * T.row_words;
        K.asrc = nreg < A.ndig ? (const uint64_t*)A.ka[r] + roff : nullptr;
        K.astride = A.key_digit_stride;
        K.seed = T.seed[r];
        K.nreg = nreg;
        if (r > 0) __syncthreads();  // every thread is done with the previous key's staged words
        if (nreg > 0)
            keyregen::stage<LOGN>(&K.seed, 1, nreg, NSEG,
                                  [tile0](int, int j) { return tile0 + (uint32_t)j * keyregen::SEG; }, pc, sm);
        const uint32_t k = A.autok[r];
        const uint32_t o[2] = {k == 1 ? i : automorph_slot<LOGN>(k, i), k == 1 ? i + 1 : automorph_slot<LOGN>(k, i + 1)};
        for (int c = 0; c < A.K; ++c) {
            Acc s0[2], s1[2];
            digit_sums(A, K, sm, c, dt, roff, tslot, s0, s1);
            ulonglong2 cv = make_ulonglong2(0, 0);
            if (mode) cv = __ldg((const ulonglong2*)(c0 + (size_t)c * A.ct_stride + roff));
            const uint64_t cw[2] = {cv.x, cv.y};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint64_t r0 = reduce(s0[h], pc), r1 = reduce(s1[h], pc);
                if (mode == 1 && (int)t < A.nq) r0 = add_mod(r0, shoup(cw[h], pm, pms, p), p);
                else if (mode == 2) r0 = add_mod(r0, cw[h], p);
                const size_t ob = (size_t)c * A.out_ct_stride + (size_t)r * A.out_rot_stride + ((size_t)t << LOGN) + o[h];
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

template <int LOGN>
int ks_dot_key_launch(const PcbKsKeyArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbKsKeyArgs& a = *ap;
    const PcbKsArgs& k = a.ks;
    const PcbKeyTab& T = a.key;
    if (k.K < 0 || k.K > 4 || k.R < 0 || k.ndig < 1 || k.ndig > MAX_DIG || k.nrows < 0 || (k.c0_mode & 3) == 3 ||
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
    const int nreg = T.nregen < k.ndig ? T.nregen : k.ndig;
    const dim3 g((1 << LOGN) / TILE, k.nrows);
    ks_dot_key<LOGN><<<g, BX, (size_t)(nreg > 0 ? nreg : 1) * TILE * sizeof(uint64_t), s>>>(a);
    return PCB_LAUNCH_RESULT();
}

template int ks_dot_regen_launch<14>(const PcbKsRegenArgs*, cudaStream_t);
template int ks_dot_regen_launch<16>(const PcbKsRegenArgs*, cudaStream_t);
template int ks_dot_key_launch<14>(const PcbKsKeyArgs*, cudaStream_t);
template int ks_dot_key_launch<16>(const PcbKsKeyArgs*, cudaStream_t);

}  // namespace regen
}  // namespace pcb
