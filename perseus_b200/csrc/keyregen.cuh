// Switching keys whose `a` is regenerated inside the inner-product kernels (the reference's Regen key source:
// crates/pc-gpu/src/ks.rs:57 and :1315-1400). A key is stored as `b` and the 8-word seed of its `a`; `a` comes back
// from the frozen u64 expander lane (chacha.cuh: w13 = digit, the row's prime; crates/pc-core/src/keys.rs:508-559),
// half the key bytes of a dense key.
//
// Layout of the work: before its products, a CTA regenerates into shared memory the `a` words of every slot segment
// it will read. A segment is 32 aligned slots, i.e. 4 expander blocks of 8 slots; the CTA's threads take the
// (key, digit, segment, block) quadruples in turn, so every ChaCha12 block computed is used whole and none is
// computed twice. Contiguous kernels stage the CTA's own slot range; gather-form kernels stage, per key, the
// segments their output slots read (an automorphism maps aligned 32-slot segments onto aligned 32-slot segments).
#pragma once
#include "chacha.cuh"

namespace pcb {
namespace keyregen {

constexpr int SEG = 32;  // slots per staged segment (4 expander blocks)

// sm[((r ndig + d) nseg + j) SEG + k] = a_{r,d}[seg(r, j) + k] (canonical mod pc.p) for key r < nkeys, digit d < ndig,
// segment j < nseg, k < SEG, where seg(r, j) is segment j's first slot under key r (a multiple of SEG) and seeds[r]
// the 8-word seed of key r. Every thread of the CTA must call it; it ends with __syncthreads().
template <int LOGN, class SegFn>
__device__ __forceinline__ void stage(const uint32_t* const* seeds, int nkeys, int ndig, int nseg, SegFn seg,
                                      const PcbPrimeConst& pc, uint64_t* sm) {
    constexpr int BPS = SEG / 8;  // expander blocks per segment
    const int total = nkeys * ndig * nseg * BPS;
    for (int w = threadIdx.x; w < total; w += blockDim.x) {
        const int blk = w % BPS;
        const int js = w / BPS;          // (r ndig + d) nseg + j
        const int j = js % nseg, rd = js / nseg;
        const int r = rd / ndig, d = rd - r * ndig;
        uint64_t v[8];
        keys::expand8<LOGN>(seeds[r], (uint32_t)(seg(r, j) >> 3) + (uint32_t)blk, (uint32_t)d, keys::TAG_KSKA, pc, v);
        ulonglong2* o = (ulonglong2*)(sm + (size_t)js * SEG + blk * 8);
#pragma unroll
        for (int u = 0; u < 4; ++u) o[u] = make_ulonglong2(v[2 * u], v[2 * u + 1]);
    }
    __syncthreads();
}

// the key-table slot of prime id t: Q ids at their index up to q_top, special ids right after; q_top < 0: prime id
__device__ __forceinline__ int key_slot(const PcbKeyTab& T, int t, int nq) {
    return (t < nq || T.q_top < 0) ? t : T.q_top + 1 + (t - nq);
}

// The staged word of key r, digit d at slot `slot` of segment j (the slot's own segment, 0 <= slot % SEG < SEG)
__device__ __forceinline__ uint64_t at(const uint64_t* sm, int ndig, int nseg, int r, int d, int j, uint32_t slot) {
    return sm[((size_t)(r * ndig + d) * nseg + j) * SEG + (slot & (SEG - 1))];
}

}  // namespace keyregen
}  // namespace pcb
