// 64-bit modular arithmetic on the B200's integer pipes.
//
// Residues are uint64_t in [0, p) with p < 2^61 (the chains here use 50- and 60-bit primes). Constant operands
// (twiddles, per-row scalars) use Shoup products with a precomputed companion w' = floor(w 2^64 / p); products of two
// runtime residues and lazy sums of products go through a 128-bit accumulator reduced once by a double-word Barrett
// step with mu = floor((2^128 - 1) / p) (the PrimeConst's mu_lo / mu_hi, crates/pc-kernels/kernels/args.cuh:26-37).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pcb200.h"

namespace pcb {

__device__ __forceinline__ uint64_t add_mod(uint64_t a, uint64_t b, uint64_t p) {
    const uint64_t s = a + b;
    return s >= p ? s - p : s;
}
__device__ __forceinline__ uint64_t sub_mod(uint64_t a, uint64_t b, uint64_t p) {
    return a >= b ? a - b : a + p - b;
}
// a w mod p in [0, 2p) for any a < 2^64 (Shoup): the quotient estimate is low by at most one
__device__ __forceinline__ uint64_t shoup_lazy(uint64_t a, uint64_t w, uint64_t ws, uint64_t p) {
    const uint64_t q = __umul64hi(a, ws);
    return a * w - q * p;
}
__device__ __forceinline__ uint64_t shoup(uint64_t a, uint64_t w, uint64_t ws, uint64_t p) {
    const uint64_t r = shoup_lazy(a, w, ws, p);
    return r >= p ? r - p : r;
}

// ------------------------------------------------------------------------------------------------ FP64 arithmetic
// For primes below 2^50 residues can live in the FP64 pipe as integer-valued doubles (B200: 64 FP64 FMAs per clock
// per SM, as many as 32-bit integer multiplies, and a 50-bit product takes one FMA pair instead of four IMADs).
constexpr double MAGIC = 6755399441055744.0;  // 1.5 * 2^52: fl(t + MAGIC) - MAGIC = rint(t) while |t| < 2^51
constexpr double TWO52 = 4503599627370496.0;

// y w mod p as an integer-valued double in [-0.75p, 0.75p], exact, for |y| < 2^52 and |w| <= p/2 (|y wp| < 2^51).
// h + l = y w exactly (FMA error-free product); q = rint(y wp) is within 0.75 of y w / p (wp carries a relative
// error of 2^-53), so h - q p is an integer below 2^53 and the FMA computes it exactly; |l| <= ulp(h) / 2 <= 2^47.
__device__ __forceinline__ double mul_f(double y, double w, double wp, double p) {
    const double h = __dmul_rn(y, w);
    const double l = __fma_rn(y, w, -h);
    const double q = __dsub_rn(__fma_rn(y, wp, MAGIC), MAGIC);
    return __dadd_rn(__fma_rn(-q, p, h), l);
}
// x - rint(x / p) p, in [-p/2 - 1, p/2 + 1] for integer-valued |x| < 2^52
__device__ __forceinline__ double red_f(double x, double p, double pinv) {
    const double q = __dsub_rn(__fma_rn(x, pinv, MAGIC), MAGIC);
    return __fma_rn(-q, p, x);
}
// the canonical word of an integer-valued |x| < 2^52: floor(x / p) is off by at most one, fixed by two selects; the
// result r < 2^52 is the mantissa of r + 2^52
__device__ __forceinline__ uint64_t canon_f(double x, double p, double pinv) {
    const double q = __dsub_rn(__fma_rd(x, pinv, MAGIC), MAGIC);
    double r = __fma_rn(-q, p, x);
    r = r < 0.0 ? __dadd_rn(r, p) : r;
    r = r >= p ? __dsub_rn(r, p) : r;
    return (uint64_t)__double_as_longlong(__dadd_rn(r, TWO52)) & ((1ull << 52) - 1);
}
// a word below 2^52 as a double (exact)
__device__ __forceinline__ double to_f(uint64_t x) {
    return __dsub_rn(__longlong_as_double((long long)(x | 0x4330000000000000ull)), TWO52);
}
// a canonical word as a centred double and its quotient by p (per-row constants of the FP64 path)
__device__ __forceinline__ void centred_f(uint64_t w, uint64_t p, double pf, double& wc, double& wp) {
    wc = w > p / 2 ? -to_f(p - w) : to_f(w);
    wp = wc / pf;
}

// 128-bit accumulator: acc += a b with the carry chain in PTX (mad.lo.cc / madc.hi)
struct Acc {
    uint64_t lo, hi;
};
__device__ __forceinline__ void mac(Acc& acc, uint64_t a, uint64_t b) {
    asm("mad.lo.cc.u64 %0, %2, %3, %0;\n\tmadc.hi.u64 %1, %2, %3, %1;"
        : "+l"(acc.lo), "+l"(acc.hi)
        : "l"(a), "l"(b));
}
__device__ __forceinline__ Acc mul_wide(uint64_t a, uint64_t b) { return Acc{a * b, __umul64hi(a, b)}; }

// Exact x mod p for any 128-bit x, p < 2^62. q = floor(x mu / 2^128) estimated from the three upper partial
// products (the dropped low product and carries make it low by at most 2); only q mod 2^64 matters because the true
// remainder x - q p is below 4p < 2^64.
__device__ __forceinline__ uint64_t reduce(Acc x, uint64_t p, uint64_t m0, uint64_t m1) {
    const uint64_t t = __umul64hi(x.lo, m0);
    uint64_t s_hi;
    // s = x.hi m0 + x.lo m1 + t, we need its high word (mod 2^64)
    asm("{\n\t"
        ".reg .u64 l1, h1, l2, h2, sl;\n\t"
        "mul.lo.u64 l1, %1, %2;\n\t"
        "mul.hi.u64 h1, %1, %2;\n\t"
        "mul.lo.u64 l2, %3, %4;\n\t"
        "mul.hi.u64 h2, %3, %4;\n\t"
        "add.cc.u64 sl, l1, l2;\n\t"
        "addc.u64 %0, h1, h2;\n\t"
        "add.cc.u64 sl, sl, %5;\n\t"
        "addc.u64 %0, %0, 0;\n\t"
        "}"
        : "=l"(s_hi)
        : "l"(x.hi), "l"(m0), "l"(x.lo), "l"(m1), "l"(t));
    const uint64_t q = x.hi * m1 + s_hi;
    uint64_t r = x.lo - q * p;
    if (r >= p) r -= p;
    if (r >= p) r -= p;
    if (r >= p) r -= p;
    return r;
}
__device__ __forceinline__ uint64_t reduce(Acc x, const PcbPrimeConst& c) { return reduce(x, c.p, c.mu_lo, c.mu_hi); }
__device__ __forceinline__ uint64_t mul_mod(uint64_t a, uint64_t b, const PcbPrimeConst& c) {
    return reduce(mul_wide(a, b), c);
}

// Source slot of sigma_k in the bit-reversed evaluation order (crates/pc-host/src/arith.rs:181-187):
// brev(((2 brev(o) + 1) k mod 2N) >> 1)
template <int LOGN>
__device__ __forceinline__ uint32_t automorph_slot(uint32_t k, uint32_t o) {
    const uint32_t j = __brev(o) >> (32 - LOGN);
    const uint32_t r = (((j << 1) + 1) * k & ((2u << LOGN) - 1)) >> 1;
    return __brev(r) >> (32 - LOGN);
}
// compact plaintext index (args.cuh:184-188): enc = 0xFFFFFFFF full rows; (enc >> 24) == 0x7F: i >> (enc & 0xFF)
// (each plaintext word serves 2^s consecutive slots); otherwise i & enc (a period)
__device__ __forceinline__ uint32_t pt_index(uint32_t i, uint32_t enc) {
    return (enc >> 24) == 0x7Fu ? i >> (enc & 0xFFu) : i & enc;
}
__device__ __forceinline__ uint32_t automorph_slot_n(uint32_t k, uint32_t o, int logn) {
    const uint32_t j = __brev(o) >> (32 - logn);
    const uint32_t r = (((j << 1) + 1) * k & ((2u << logn) - 1)) >> 1;
    return __brev(r) >> (32 - logn);
}

__device__ __forceinline__ const uint64_t* at_row(const PcbPolyRef& r, int c, int part, int row, int logn) {
    return (const uint64_t*)r.base + (size_t)c * r.ct_stride + (size_t)part * r.part_stride + ((size_t)row << logn);
}
__device__ __forceinline__ uint64_t* at_row_w(const PcbPolyRef& r, int c, int part, int row, int logn) {
    return (uint64_t*)r.base + (size_t)c * r.ct_stride + (size_t)part * r.part_stride + ((size_t)row << logn);
}
__device__ __forceinline__ int rs_row(const PcbRowSet& rs, int y) { return y < rs.nq ? y : rs.qmax + (y - rs.nq); }

// Programmatic dependent launch: a kernel may start while the previous kernel of its stream is finishing; it stages
// constant tables (twiddles, conversion matrices, keys: written when the context was built), then waits for the
// previous kernel's writes before it reads anything that kernel may have produced. Every CTA allows the next kernel to
// launch as soon as it has passed its wait; that takes effect once the whole grid has (its last wave), so the next
// kernel's CTAs fill SMs as this one's finish.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Start moving the 128-byte line holding p into L2 (no register result, no wait)
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// Launch with programmatic stream serialization: the kernel must call pdl_wait before its dependent reads
template <typename... KArgs, typename... Args>
__host__ inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, args...);
}

// launch_pdl with dynamic shared memory
template <typename... KArgs, typename... Args>
__host__ inline void launch_pdl_smem(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                     Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, args...);
}

// ------------------------------------------------------------------------------------------------ bulk copies
// Asynchronous global -> shared bulk copies (cp.async.bulk, the TMA engine's untiled form; no multicast) completing
// on a shared-memory mbarrier by transaction bytes. Addresses 16-byte aligned, sizes multiples of 16 bytes.
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
// order the barrier initialisation before its use by the async proxy
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// order this thread's earlier generic-proxy accesses to shared memory before a later bulk copy into it
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// one arrival that also expects `bytes` of transactions on the barrier's current phase
__device__ __forceinline__ void mbar_expect(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for phase `parity` of the barrier with an iteration limit (each try_wait blocks for a hardware-bounded time):
// false when the limit ran out, which the caller reports (the wait never spins forever)
constexpr uint32_t MBAR_WAIT_LIMIT = 1u << 20;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t it = 0; it < MBAR_WAIT_LIMIT; ++it)
        if (mbar_test(bar, parity)) return true;
    return false;
}

// process-wide count of kernels this library launched (pcb_launch_count)
void note_launches(unsigned n);

}  // namespace pcb

// launcher return codes (crates/pc-kernels/kernels/args.cuh:1036); PCB_LAUNCH_RESULT counts one launch
#define PCB_BAD_ARGS (-1)
#define PCB_LAUNCHED(n) (pcb::note_launches(n), (int)cudaGetLastError())
#define PCB_LAUNCH_RESULT() PCB_LAUNCHED(1)
