// The frozen u64 expander lane (ChaCha12 counter mode; crates/pc-core/src/keys.rs:463-490, KSKB pinned by
// crates/pc-core/tests/kskb_frozen.rs): one ChaCha block gives 8 consecutive slots (two words per 64-bit value); a value
// at or above the largest multiple of p below 2^64 is redrawn from block counter + t N / 8 (t = 1 .. 15).
#pragma once
#include "arith.cuh"

namespace pcb {
namespace keys {

constexpr uint32_t TAG_KSKA = 0x4b534b41u;
constexpr uint32_t TAG_ENCA = 0x454e4341u;

__device__ __forceinline__ void qround(uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
    a += b;
    d = __funnelshift_l(d ^ a, d ^ a, 16);
    c += d;
    b = __funnelshift_l(b ^ c, b ^ c, 12);
    a += b;
    d = __funnelshift_l(d ^ a, d ^ a, 8);
    c += d;
    b = __funnelshift_l(b ^ c, b ^ c, 7);
}

// ChaCha with 12 rounds: constants, key words 4..11, state words 12..15 = (counter, w13, w14, tag), feed-forward
__device__ __forceinline__ void chacha12(const uint32_t* key, uint32_t ctr, uint32_t w13, uint32_t w14, uint32_t tag,
                                         uint32_t o[16]) {
    uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, key[0], key[1], key[2], key[3],
                      key[4],      key[5],      key[6],      key[7],      ctr,    w13,    w14,    tag};
    uint32_t x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = s[i];
#pragma unroll
    for (int r = 0; r < 6; ++r) {
        qround(x[0], x[4], x[8], x[12]);
        qround(x[1], x[5], x[9], x[13]);
        qround(x[2], x[6], x[10], x[14]);
        qround(x[3], x[7], x[11], x[15]);
        qround(x[0], x[5], x[10], x[15]);
        qround(x[1], x[6], x[11], x[12]);
        qround(x[2], x[7], x[8], x[13]);
        qround(x[3], x[4], x[9], x[14]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = x[i] + s[i];
}

// The 8 values of block b0 of the u64 lane for (seed, w13, tag, prime): out[j] = slot 8 b0 + j, reduced mod p.
template <int LOGN>
__device__ __forceinline__ void expand8(const uint32_t* seed, uint32_t b0, uint32_t w13, uint32_t tag,
                                        const PcbPrimeConst& pc, uint64_t out[8]) {
    const uint64_t p = pc.p;
    const uint32_t w13l = w13 ^ ((uint32_t)(p >> 32) << 4), tagl = tag + 1u;
    const uint64_t mp = (~0ull / p) * p;
    constexpr uint32_t NB = (1u << LOGN) / 8;
    uint32_t blk[16];
    chacha12(seed, b0, w13l, (uint32_t)p, tagl, blk);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint64_t v = (uint64_t)blk[2 * j] | (uint64_t)blk[2 * j + 1] << 32;
        for (uint32_t t = 1; v >= mp && t < 16; ++t) {
            uint32_t b2[16];
            chacha12(seed, b0 + t * NB, w13l, (uint32_t)p, tagl, b2);
            v = (uint64_t)b2[2 * j] | (uint64_t)b2[2 * j + 1] << 32;
        }
        out[j] = v < p ? v : reduce(Acc{v, 0}, pc);
    }
}

// The 4 slots 4 h .. 4 h + 3 of block b0 (h = 0, 1): half of expand8, for kernels that hold 4 slots per thread
template <int LOGN>
__device__ __forceinline__ void expand4(const uint32_t* seed, uint32_t b0, int h, uint32_t w13, uint32_t tag,
                                        const PcbPrimeConst& pc, uint64_t out[4]) {
    const uint64_t p = pc.p;
    const uint32_t w13l = w13 ^ ((uint32_t)(p >> 32) << 4), tagl = tag + 1u;
    const uint64_t mp = (~0ull / p) * p;
    constexpr uint32_t NB = (1u << LOGN) / 8;
    uint32_t blk[16];
    chacha12(seed, b0, w13l, (uint32_t)p, tagl, blk);
    // word pairs of slot 4 h + u, picked between two constant indices (no run-time index into the block)
    auto pick = [h](const uint32_t* b, int u) {
        const uint64_t lo = (uint64_t)b[2 * u] | (uint64_t)b[2 * u + 1] << 32;
        const uint64_t hi = (uint64_t)b[8 + 2 * u] | (uint64_t)b[9 + 2 * u] << 32;
        return h ? hi : lo;
    };
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        uint64_t v = pick(blk, u);
        for (uint32_t t = 1; v >= mp && t < 16; ++t) {
            uint32_t b2[16];
            chacha12(seed, b0 + t * NB, w13l, (uint32_t)p, tagl, b2);
            v = pick(b2, u);
        }
        out[u] = v < p ? v : reduce(Acc{v, 0}, pc);
    }
}

}  // namespace keys
}  // namespace pcb
