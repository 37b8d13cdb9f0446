// Key material on the device: the frozen u64 expander lane (ChaCha12), secret-key encryption, switching-key
// generation and key expansion. Semantics: crates/pc-kernels/kernels/args.cuh:306-323 (KskExpandArgs), :613-628
// (EncryptArgs), :630-654 (KskGenArgs); the lane rule of crates/pc-core/src/keys.rs:463-490 (KSKB: FROZEN, pinned by
// crates/pc-core/tests/kskb_frozen.rs) applied to the ENCA tag as crates/pc-kernels/kernels/chacha.cuh:60-98 does.
//
// One thread computes one ChaCha block = 8 consecutive slots (two words per 64-bit value); the rejection retry
// (probability < p / 2^64 per slot) recomputes only the rejected slot's block at counter + t N / 8.
#include "chacha.cuh"

namespace pcb {
namespace keys {

constexpr int BX = 128;
// ------------------------------------------------------------------------------------------------ ksk_expand
template <int LOGN>
__global__ void __launch_bounds__(BX) ksk_expand(PcbKskExpandArgs a) {
    const uint32_t b0 = blockIdx.x * BX + threadIdx.x;
    const int m = blockIdx.y, d = a.d0 + (int)blockIdx.z;
    const int id = a.prime_ids[m];
    uint64_t v[8];
    expand8<LOGN>(a.seed, b0, (uint32_t)d, TAG_KSKA, a.pr[id], v);
    uint64_t* o = (uint64_t*)a.out + (((size_t)(d - a.d0) * a.nmod + m) << LOGN) + 8 * (size_t)b0;
#pragma unroll
    for (int j = 0; j < 4; ++j) ((ulonglong2*)o)[j] = make_ulonglong2(v[2 * j], v[2 * j + 1]);
}

template <int LOGN>
int ksk_expand_launch(const PcbKskExpandArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbKskExpandArgs& a = *ap;
    if (a.nmod < 0 || a.dnum < 0 || a.dnum > 16 || a.d0 < 0 || a.d0 > a.dnum || !a.out || !a.seed || !a.prime_ids || !a.pr)
        return PCB_BAD_ARGS;
    if (a.nmod == 0 || a.dnum == a.d0) return 0;
    ksk_expand<LOGN><<<dim3((1 << LOGN) / 8 / BX, a.nmod, a.dnum - a.d0), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ encrypt
// c0 = (e + m) - a s, c1 = a, limb l (prime id l) at + l N; a from the ENCA lane keyed by the nonce
template <int LOGN>
__global__ void __launch_bounds__(BX) encrypt(PcbEncryptArgs a) {
    const uint32_t b0 = blockIdx.x * BX + threadIdx.x;
    const int l = blockIdx.y;
    const PcbPrimeConst& pc = a.pr[l];
    const uint64_t p = pc.p;
    uint64_t av[8];
    expand8<LOGN>(a.seed, b0, a.nonce, TAG_ENCA, pc, av);
    const size_t off = ((size_t)l << LOGN) + 8 * (size_t)b0;
    const uint64_t* s = (const uint64_t*)a.s + off;
    const uint64_t* e = (const uint64_t*)a.e + off;
    const uint64_t* m = a.m ? (const uint64_t*)a.m + off : nullptr;
    uint64_t r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint64_t x = e[j];
        if (m) x = add_mod(x, m[j], p);
        r[j] = sub_mod(x, mul_mod(av[j], s[j], pc), p);
    }
    uint64_t* c0 = (uint64_t*)a.c0 + off;
#pragma unroll
    for (int j = 0; j < 8; ++j) c0[j] = r[j];
    if (a.c1) {
        uint64_t* c1 = (uint64_t*)a.c1 + off;
#pragma unroll
        for (int j = 0; j < 8; ++j) c1[j] = av[j];
    }
}

template <int LOGN>
int encrypt_launch(const PcbEncryptArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbEncryptArgs& a = *ap;
    if (a.nl < 0 || !a.c0 || !a.s || !a.e || !a.seed || !a.pr) return PCB_BAD_ARGS;
    if (a.nl == 0) return 0;
    encrypt<LOGN><<<dim3((1 << LOGN) / 8 / BX, a.nl), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ ksk_gen
// b[d][m] = e[d][m] + (id < nq && digit_of[id] == d ? pmod[id] s_old'[id] : 0) - a s_new[id], a from the KSKB lane;
// s_old' = s_old^2 when sq (relinearization). Dense rows only (bits = 0).
template <int LOGN>
__global__ void __launch_bounds__(BX) ksk_gen(PcbKskGenArgs a) {
    const uint32_t b0 = blockIdx.x * BX + threadIdx.x;
    const int m = blockIdx.y, d = blockIdx.z;
    const int id = a.ids[m];
    const PcbPrimeConst& pc = a.pr[id];
    const uint64_t p = pc.p;
    uint64_t av[8];
    expand8<LOGN>(a.seed, b0, (uint32_t)d, TAG_KSKA, pc, av);
    const size_t off = (((size_t)d * a.nrows + m) << LOGN) + 8 * (size_t)b0;
    const size_t soff = ((size_t)id << LOGN) + 8 * (size_t)b0;
    const bool in_digit = id < a.nq && a.digit_of[id] == d;
    uint64_t pm = 0, pms = 0;
    if (in_digit) {
        pm = ((const uint64_t*)a.pmod)[id];
        pms = ((const uint64_t*)a.pmods)[id];
    }
    const uint64_t* e = (const uint64_t*)a.e + off;
    const uint64_t* sn = (const uint64_t*)a.s_new + soff;
    const uint64_t* so = (const uint64_t*)a.s_old + soff;
    uint64_t r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint64_t x = e[j];
        if (in_digit) {
            uint64_t t = so[j];
            if (a.sq) t = mul_mod(t, t, pc);
            x = add_mod(x, shoup(t, pm, pms, p), p);
        }
        r[j] = sub_mod(x, mul_mod(av[j], sn[j], pc), p);
    }
    uint64_t* bo = (uint64_t*)a.b + off;
#pragma unroll
    for (int j = 0; j < 8; ++j) bo[j] = r[j];
    if (a.a) {
        uint64_t* ao = (uint64_t*)a.a + off;
#pragma unroll
        for (int j = 0; j < 8; ++j) ao[j] = av[j];
    }
}

template <int LOGN>
int ksk_gen_launch(const PcbKskGenArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbKskGenArgs& a = *ap;
    if (a.bits != 0) return PCB_BAD_ARGS;  // bit-packed rows are a 32-bit-word storage form
    if (a.nrows < 0 || a.ndig < 0 || a.ndig > 16 || !a.b || !a.e || !a.s_new || !a.s_old || !a.seed || !a.ids ||
        !a.digit_of || !a.pmod || !a.pmods || !a.pr)
        return PCB_BAD_ARGS;
    if (a.nrows == 0 || a.ndig == 0) return 0;
    ksk_gen<LOGN><<<dim3((1 << LOGN) / 8 / BX, a.nrows, a.ndig), BX, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

template int ksk_expand_launch<14>(const PcbKskExpandArgs*, cudaStream_t);
template int ksk_expand_launch<16>(const PcbKskExpandArgs*, cudaStream_t);
template int encrypt_launch<14>(const PcbEncryptArgs*, cudaStream_t);
template int encrypt_launch<16>(const PcbEncryptArgs*, cudaStream_t);
template int ksk_gen_launch<14>(const PcbKskGenArgs*, cudaStream_t);
template int ksk_gen_launch<16>(const PcbKskGenArgs*, cudaStream_t);

}  // namespace keys
}  // namespace pcb
