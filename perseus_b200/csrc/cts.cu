// The fused CoeffToSlot stage of the launcher table: cts_fused and cts_fused_regen (semantics:
// crates/pc-kernels/kernels/args.cuh:325-352 and :754-758; caller crates/pc-gpu/src/bts/cts.rs). One BSGS stage:
// the baby rotations of x are hoisted (one ModUp, supplied by the caller) and never written; each is formed in the
// extended basis at the slot it is consumed and multiplied straight into the giant-step sums.
//
// Design. One thread per output slot o of one row, a CTA of BX consecutive slots and up to KG ciphertexts (grid z over
// the groups). For baby step i the thread reads its source slot s = sigma_i^-1(o); the automorphism maps aligned
// 32-slot segments onto aligned 32-slot segments of the bit-reversed order, so a warp's gathers are whole 256-byte
// segments of every row it reads. A key word is loaded once for the KG ciphertexts; the rotated pair is multiplied
// into the G <= 2 giant sums while still in registers (128-bit lazy sums reduced every 8 baby steps: 8 products below
// 2^124 and a residue stay below 2^128). Regenerated keys: before each baby step the CTA expands the `a` words of the
// BX / 32 source segments it is about to read into shared memory (keyregen::stage: whole ChaCha12 blocks, none twice),
// so only `b` is read from HBM.
#include "keyregen.cuh"
#include "kernels.h"

namespace pcb {
namespace cts {

constexpr int BX = 128;
constexpr int KG = 4;    // ciphertexts per CTA
constexpr int DMAX = 8;  // key digits (the reference's bound at 64-bit words)
constexpr int NSEG = BX / keyregen::SEG;

template <int LOGN, int G, bool REGEN, bool X0>
__global__ void __launch_bounds__(BX) cts_fused(PcbCtsRegenArgs R) {
    __shared__ __align__(16) uint64_t sm[REGEN ? DMAX * NSEG * keyregen::SEG : 2];
    const PcbCtsArgs& A = R.cts;
    const uint32_t t = A.rows[blockIdx.y];
    const PcbPrimeConst& pc = A.pr[t];
    const uint64_t p = pc.p;
    const bool isq = (int)t < A.nq;
    const int cbase = blockIdx.z * KG;
    const int kg = min(KG, A.K - cbase);
    const uint32_t tile0 = blockIdx.x * BX, o = tile0 + threadIdx.x;
    const size_t roff = (size_t)t << LOGN;
    const int dt = isq ? A.digit_of[t] : -1;
    const uint64_t pm = ((const uint64_t*)A.pmod)[t], pms = ((const uint64_t*)A.pmods)[t];
    const size_t pword = (size_t)(isq ? (int)t : A.pt_prow + ((int)t - A.nq)) * (size_t)A.ptw + pt_index(o, A.enc);
    const uint64_t* X = (const uint64_t*)A.x + (size_t)cbase * A.ct_stride + roff;
    const uint64_t* MU = (const uint64_t*)A.modup + (size_t)cbase * A.mu_ct_stride + roff;
    const int nreg = REGEN ? min(A.ndig, R.key.nregen) : 0;
    const size_t brow = REGEN ? (size_t)keyregen::key_slot(R.key, (int)t, A.nq) * R.key.row_words : 0;

    Acc acc0[KG][G], acc1[KG][G];
#pragma unroll
    for (int c = 0; c < KG; ++c)
#pragma unroll
        for (int j = 0; j < G; ++j) acc0[c][j] = acc1[c][j] = Acc{0, 0};

    for (int i = 0; i < A.B; ++i) {
        uint64_t v0[KG], v1[KG];
        if (i == 0) {
#pragma unroll
            for (int c = 0; c < KG; ++c) {
                v0[c] = v1[c] = 0;
                if (c >= kg) continue;
                if (X0) {  // a key-switched identity, stored extended
                    const uint64_t* y = (const uint64_t*)A.x0 + (size_t)(cbase + c) * A.ct_stride + roff;
                    v0[c] = y[o];
                    v1[c] = y[A.part_stride + o];
                } else if (isq) {
                    v0[c] = shoup(X[(size_t)c * A.ct_stride + o], pm, pms, p);
                    v1[c] = shoup(X[(size_t)c * A.ct_stride + A.part_stride + o], pm, pms, p);
                }
            }
        } else {
            const uint32_t k = A.kinv[i - 1];
            const uint32_t s = automorph_slot<LOGN>(k, o);
            if (REGEN && nreg > 0) {
                if (i > 1) __syncthreads();  // every thread is done with the previous baby step's staged words
                keyregen::stage<LOGN>(
                    R.key.seed + (i - 1), 1, nreg, NSEG,
                    [k, tile0](int, int j) {
                        return automorph_slot<LOGN>(k, tile0 + (uint32_t)j * keyregen::SEG) & ~(uint32_t)(keyregen::SEG - 1);
                    },
                    pc, sm);
            }
            Acc s0[KG], s1[KG];
#pragma unroll
            for (int c = 0; c < KG; ++c) s0[c] = s1[c] = Acc{0, 0};
            for (int d = 0; d < A.ndig; ++d) {
                uint64_t b, a;
                if (REGEN) {
                    b = __ldg((const uint64_t*)R.key.kb[i - 1] + (size_t)d * R.key.srows * R.key.row_words + brow + s);
                    a = d < nreg ? keyregen::at(sm, nreg, NSEG, 0, d, threadIdx.x / keyregen::SEG, s)
                                 : __ldg((const uint64_t*)A.ka[i - 1] + (size_t)d * A.key_digit_stride + roff + s);
                } else {
                    b = __ldg((const uint64_t*)A.kb[i - 1] + (size_t)d * A.key_digit_stride + roff + s);
                    a = __ldg((const uint64_t*)A.ka[i - 1] + (size_t)d * A.key_digit_stride + roff + s);
                }
#pragma unroll
                for (int c = 0; c < KG; ++c) {
                    if (c >= kg) continue;
                    const uint64_t x = d == dt ? X[(size_t)c * A.ct_stride + A.part_stride + s]
                                               : MU[(size_t)c * A.mu_ct_stride + (size_t)d * A.mu_digit_stride + s];
                    mac(s0[c], x, b);
                    mac(s1[c], x, a);
                }
            }
#pragma unroll
            for (int c = 0; c < KG; ++c) {
                v0[c] = v1[c] = 0;
                if (c >= kg) continue;
                uint64_t r0 = reduce(s0[c], pc);
                if (isq) r0 = add_mod(r0, shoup(X[(size_t)c * A.ct_stride + s], pm, pms, p), p);
                v0[c] = r0;
                v1[c] = reduce(s1[c], pc);
            }
        }
#pragma unroll
        for (int j = 0; j < G; ++j) {
            const int dg = A.B * j + i;
            if (dg >= A.npts) continue;
            const uint64_t w = __ldg((const uint64_t*)A.pts[dg] + pword);
#pragma unroll
            for (int c = 0; c < KG; ++c) {
                mac(acc0[c][j], v0[c], w);
                mac(acc1[c][j], v1[c], w);
            }
        }
        if ((i & 7) == 7) {
#pragma unroll
            for (int c = 0; c < KG; ++c)
#pragma unroll
                for (int j = 0; j < G; ++j) {
                    acc0[c][j] = Acc{reduce(acc0[c][j], pc), 0};
                    acc1[c][j] = Acc{reduce(acc1[c][j], pc), 0};
                }
        }
    }
#pragma unroll
    for (int c = 0; c < KG; ++c) {
        if (c >= kg) break;
#pragma unroll
        for (int j = 0; j < G; ++j) {
            uint64_t* r = (uint64_t*)A.res + (size_t)((cbase + c) * A.G + j) * A.ct_stride + roff;
            r[o] = reduce(acc0[c][j], pc);
            r[A.part_stride + o] = reduce(acc1[c][j], pc);
        }
    }
}

template <int LOGN, bool REGEN>
int launch_any(const PcbCtsRegenArgs& a, cudaStream_t s) {
    const PcbCtsArgs& c = a.cts;
    if (c.K < 0 || c.B < 1 || c.G < 1 || c.G > 2 || c.ndig < 1 || c.ndig > DMAX || c.nrows < 0 || c.npts < 0 ||
        c.ptw < 1 || c.pair_cts != 0)
        return PCB_BAD_ARGS;
    if (!c.x || !c.res || !c.pts || !c.rows || !c.digit_of || !c.pmod || !c.pmods || !c.pr) return PCB_BAD_ARGS;
    if (c.B > 1) {
        if (!c.kinv || !c.modup) return PCB_BAD_ARGS;
        if (REGEN ? (!a.key.kb || !a.key.seed || a.key.bits != 0 || a.key.srows < 1 || a.key.nregen < 0 ||
                     (a.key.nregen < c.ndig && !c.ka))
                  : (!c.kb || !c.ka))
            return PCB_BAD_ARGS;
    }
    if (c.K == 0 || c.nrows == 0) return 0;
    const dim3 g((1 << LOGN) / BX, c.nrows, (c.K + KG - 1) / KG);
    const bool x0 = c.x0 != nullptr;
    if (c.G == 1) {
        if (x0) cts_fused<LOGN, 1, REGEN, true><<<g, BX, 0, s>>>(a);
        else cts_fused<LOGN, 1, REGEN, false><<<g, BX, 0, s>>>(a);
    } else {
        if (x0) cts_fused<LOGN, 2, REGEN, true><<<g, BX, 0, s>>>(a);
        else cts_fused<LOGN, 2, REGEN, false><<<g, BX, 0, s>>>(a);
    }
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int cts_fused_launch(const PcbCtsArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    PcbCtsRegenArgs r;
    memset(&r, 0, sizeof r);
    r.cts = *ap;
    return launch_any<LOGN, false>(r, s);
}

template <int LOGN>
int cts_fused_regen_launch(const PcbCtsRegenArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    return launch_any<LOGN, true>(*ap, s);
}

template int cts_fused_launch<14>(const PcbCtsArgs*, cudaStream_t);
template int cts_fused_launch<16>(const PcbCtsArgs*, cudaStream_t);
template int cts_fused_regen_launch<14>(const PcbCtsRegenArgs*, cudaStream_t);
template int cts_fused_regen_launch<16>(const PcbCtsRegenArgs*, cudaStream_t);

}  // namespace cts
}  // namespace pcb
