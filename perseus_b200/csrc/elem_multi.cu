// The table entries the reference's device evaluator calls on its main path besides the core ones (crates/pc-gpu/src:
// ops.rs wsum / wsum_k / tensor_sum / tensor_multi, relin.rs wsum, ks.rs ew_many / submul_many, rescale.rs
// rescale_fwd / rescale_combine_to, bts/evalmod.rs wsum_multi / md_epilogue_to), with the semantics of
// crates/pc-kernels/kernels/args.cuh (EwManyArgs :159-170, SubMulManyArgs :172-182, TensorSumArgs :380-389,
// TensorMultiArgs :391-404, MdEpiToArgs :449-457, WsumArgs :459-468, WsumKArgs :470-474, WsumMultiArgs :476-489,
// RescaleNttArgs :553-562, RescaleCombineToArgs :573-578). Every output is the canonical residue of an exact sum, so
// the words equal the reference's whatever the order of the reduction.
//
// The subring switch's pack_split / pack_dot (crates/pc-gpu/src/ks/pack.rs; PackSplitArgs :230-242, PackDotArgs
// :244-261) sit here too. All are HBM-bound streams laid out as elem.cu's: 4 consecutive words per thread with 16-byte accesses, grids
// (N / 1024, rows, ciphertexts [x parts]).
#include "arith.cuh"
#include "kernels.h"

namespace pcb {
namespace elem {

namespace {
constexpr int BXM = 256;
struct W4 {
    uint64_t v[4];
};
__device__ __forceinline__ W4 ld(const uint64_t* p) {
    const ulonglong2 a = ((const ulonglong2*)p)[0], b = ((const ulonglong2*)p)[1];
    return W4{{a.x, a.y, b.x, b.y}};
}
__device__ __forceinline__ void st(uint64_t* p, const uint64_t (&r)[4]) {
    ((ulonglong2*)p)[0] = make_ulonglong2(r[0], r[1]);
    ((ulonglong2*)p)[1] = make_ulonglong2(r[2], r[3]);
}
__host__ __forceinline__ bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }
__host__ __forceinline__ bool ref16(const PcbPolyRef& r) {
    return al16(r.base) && (r.ct_stride & 1) == 0 && (r.part_stride & 1) == 0;
}
__device__ __forceinline__ size_t word0() { return ((size_t)blockIdx.x * BXM + threadIdx.x) * 4; }
}  // namespace

// ------------------------------------------------------------------------------------------------ ew_many, submul_many
// out[j] = a[j] (+ b[j]) (+ c[j]), and out[j] = (a[j] - b[j]) t, over Q rows [0, nrows) of polynomials by pointer
template <int LOGN>
__global__ void __launch_bounds__(BXM) ew_many(PcbEwManyArgs a) {
    const int j = blockIdx.z, row = blockIdx.y;
    const uint64_t p = a.pr[row].p;
    const size_t i = ((size_t)row << LOGN) + word0();
    const W4 x = ld((const uint64_t*)a.a[j] + i);
    uint64_t r[4] = {x.v[0], x.v[1], x.v[2], x.v[3]};
    if (a.b[j]) {
        const W4 y = ld((const uint64_t*)a.b[j] + i);
#pragma unroll
        for (int w = 0; w < 4; ++w) r[w] = add_mod(r[w], y.v[w], p);
    }
    if (a.c[j]) {
        const W4 y = ld((const uint64_t*)a.c[j] + i);
#pragma unroll
        for (int w = 0; w < 4; ++w) r[w] = add_mod(r[w], y.v[w], p);
    }
    st((uint64_t*)a.out[j] + i, r);
}

template <int LOGN>
__global__ void __launch_bounds__(BXM) submul_many(PcbSubMulManyArgs a) {
    const int j = blockIdx.z, row = blockIdx.y;
    const PcbPrimeConst& pc = a.pr[row];
    const size_t i = ((size_t)row << LOGN) + word0();
    const W4 x = ld((const uint64_t*)a.a[j] + i), y = ld((const uint64_t*)a.b[j] + i), t = ld((const uint64_t*)a.t + i);
    uint64_t r[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) r[w] = mul_mod(sub_mod(x.v[w], y.v[w], pc.p), t.v[w], pc);
    st((uint64_t*)a.out[j] + i, r);
}

template <int LOGN>
int ew_many_launch(const PcbEwManyArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbEwManyArgs& a = *ap;
    if (a.n < 1 || a.n > PCB_EWM_MAX || a.nrows < 0 || !a.pr) return PCB_BAD_ARGS;
    for (int j = 0; j < a.n; ++j)
        if (!a.out[j] || !a.a[j] || !al16(a.out[j]) || !al16(a.a[j]) || !al16(a.b[j]) || !al16(a.c[j]))
            return PCB_BAD_ARGS;
    if (a.nrows == 0) return 0;
    ew_many<LOGN><<<dim3((1 << LOGN) / (BXM * 4), a.nrows, a.n), BXM, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int submul_many_launch(const PcbSubMulManyArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbSubMulManyArgs& a = *ap;
    if (a.n < 1 || a.n > PCB_EWM_MAX || a.nrows < 0 || !a.pr || !a.t || !al16(a.t)) return PCB_BAD_ARGS;
    for (int j = 0; j < a.n; ++j)
        if (!a.out[j] || !a.a[j] || !a.b[j] || !al16(a.out[j]) || !al16(a.a[j]) || !al16(a.b[j])) return PCB_BAD_ARGS;
    if (a.nrows == 0) return 0;
    submul_many<LOGN><<<dim3((1 << LOGN) / (BXM * 4), a.nrows, a.n), BXM, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ weighted sums
// out = sum_{j < nsrc} w[j][row] src_j (both parts; w at w + j rowstride + row, Shoup companions ws) [+ k[row] on part
// 0, raw, reduced once when >= p]; wsum_multi: up to 3 such sums of one source list, out[m] on rows [0, n[m])
template <int LOGN, int NOUT>
__device__ __forceinline__ void wsums(const PcbPolyRef* out, const PcbPolyRef* src, int nsrc, const void* const* w,
                                      const void* const* ws, const void* const* k, const int* n, int rowstride, int c,
                                      int row, const PcbPrimeConst* pr) {
    const uint64_t p = pr[row].p;
    const size_t i = word0();
    uint64_t r[NOUT][2][4] = {};
    bool on[NOUT];
#pragma unroll
    for (int m = 0; m < NOUT; ++m) on[m] = row < n[m];
    for (int j = 0; j < nsrc; ++j) {
        const W4 x0 = ld(at_row(src[j], c, 0, row, LOGN) + i), x1 = ld(at_row(src[j], c, 1, row, LOGN) + i);
#pragma unroll
        for (int m = 0; m < NOUT; ++m) {
            if (!on[m]) continue;
            const uint64_t wv = ((const uint64_t*)w[m])[(size_t)j * rowstride + row];
            const uint64_t wsv = ((const uint64_t*)ws[m])[(size_t)j * rowstride + row];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                r[m][0][u] = add_mod(r[m][0][u], shoup(x0.v[u], wv, wsv, p), p);
                r[m][1][u] = add_mod(r[m][1][u], shoup(x1.v[u], wv, wsv, p), p);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < NOUT; ++m) {
        if (!on[m]) continue;
        if (k[m]) {
            const uint64_t kv = ((const uint64_t*)k[m])[row];
            const uint64_t kr = kv >= p ? kv - p : kv;
#pragma unroll
            for (int u = 0; u < 4; ++u) r[m][0][u] = add_mod(r[m][0][u], kr, p);
        }
        st(at_row_w(out[m], c, 0, row, LOGN) + i, r[m][0]);
        st(at_row_w(out[m], c, 1, row, LOGN) + i, r[m][1]);
    }
}

template <int LOGN>
__global__ void __launch_bounds__(BXM) wsum(PcbWsumArgs a, const void* k) {
    const void* w[1] = {a.w};
    const void* ws[1] = {a.ws};
    const void* kk[1] = {k};
    const int n[1] = {a.n};
    wsums<LOGN, 1>(&a.out, a.src, a.nsrc, w, ws, kk, n, a.rowstride, blockIdx.z, blockIdx.y, a.pr);
}

template <int LOGN>
__global__ void __launch_bounds__(BXM) wsum_multi(PcbWsumMultiArgs a) {
    int n[3];
    const void* k[3];
#pragma unroll
    for (int m = 0; m < 3; ++m) {
        n[m] = m < a.nout ? a.n[m] : 0;
        k[m] = m < a.nout ? a.k[m] : nullptr;
    }
    wsums<LOGN, 3>(a.out, a.src, a.nsrc, a.w, a.ws, k, n, a.rowstride, blockIdx.z, blockIdx.y, a.pr);
}

namespace {
int wsum_check(const PcbWsumArgs& a) {
    if (a.nsrc < 1 || a.nsrc > 8 || a.n < 0 || a.K < 0 || a.rowstride < 0 || !a.pr || !a.w || !a.ws || !a.out.base ||
        !ref16(a.out))
        return PCB_BAD_ARGS;
    for (int j = 0; j < a.nsrc; ++j)
        if (!a.src[j].base || !ref16(a.src[j])) return PCB_BAD_ARGS;
    return 0;
}
}  // namespace

template <int LOGN>
int wsum_launch(const PcbWsumArgs* ap, cudaStream_t s) {
    if (!ap || wsum_check(*ap)) return PCB_BAD_ARGS;
    if (ap->n == 0 || ap->K == 0) return 0;
    wsum<LOGN><<<dim3((1 << LOGN) / (BXM * 4), ap->n, ap->K), BXM, 0, s>>>(*ap, nullptr);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int wsum_k_launch(const PcbWsumKArgs* ap, cudaStream_t s) {
    if (!ap || wsum_check(ap->w) || !ap->k) return PCB_BAD_ARGS;
    if (ap->w.n == 0 || ap->w.K == 0) return 0;
    wsum<LOGN><<<dim3((1 << LOGN) / (BXM * 4), ap->w.n, ap->w.K), BXM, 0, s>>>(ap->w, ap->k);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int wsum_multi_launch(const PcbWsumMultiArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbWsumMultiArgs& a = *ap;
    if (a.nsrc < 1 || a.nsrc > 8 || a.nout < 1 || a.nout > 3 || a.K < 0 || a.nmax < 0 || a.rowstride < 0 || !a.pr)
        return PCB_BAD_ARGS;
    for (int m = 0; m < a.nout; ++m)
        if (!a.out[m].base || !ref16(a.out[m]) || !a.w[m] || !a.ws[m] || a.n[m] < 0 || a.n[m] > a.nmax)
            return PCB_BAD_ARGS;
    for (int j = 0; j < a.nsrc; ++j)
        if (!a.src[j].base || !ref16(a.src[j])) return PCB_BAD_ARGS;
    if (a.nmax == 0 || a.K == 0) return 0;
    wsum_multi<LOGN><<<dim3((1 << LOGN) / (BXM * 4), a.nmax, a.K), BXM, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ tensor sums
// output o: c0 = sum_j a0 b0, c1 = sum_j (a0 b1 + a1 b0) into out[o], d2 = sum_j a1 b1 into part 1 of d2[o]; every
// product summed exactly in 128 bits and reduced once; acc: add the outputs' previous words (acc & 2: d2's too)
template <int LOGN, int MAXP>
__device__ __forceinline__ void tensor_out(const PcbPolyRef& out, const PcbPolyRef& d2, const PcbPolyRef* A,
                                           const PcbPolyRef* B, int npairs, int acc, int c, int row,
                                           const PcbPrimeConst& pc) {
    const size_t i = word0();
    Acc s0[4] = {}, s1[4] = {}, s2[4] = {};
    for (int j = 0; j < npairs; ++j) {
        const W4 x0 = ld(at_row(A[j], c, 0, row, LOGN) + i), x1 = ld(at_row(A[j], c, 1, row, LOGN) + i);
        const W4 y0 = ld(at_row(B[j], c, 0, row, LOGN) + i), y1 = ld(at_row(B[j], c, 1, row, LOGN) + i);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            mac(s0[w], x0.v[w], y0.v[w]);
            mac(s1[w], x0.v[w], y1.v[w]);
            mac(s1[w], x1.v[w], y0.v[w]);
            mac(s2[w], x1.v[w], y1.v[w]);
        }
    }
    uint64_t r0[4], r1[4], r2[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        r0[w] = reduce(s0[w], pc);
        r1[w] = reduce(s1[w], pc);
        r2[w] = reduce(s2[w], pc);
    }
    uint64_t* o0 = at_row_w(out, c, 0, row, LOGN) + i;
    uint64_t* o1 = at_row_w(out, c, 1, row, LOGN) + i;
    uint64_t* o2 = at_row_w(d2, c, 1, row, LOGN) + i;
    if (acc) {
        const W4 d0 = ld(o0), d1 = ld(o1);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            r0[w] = add_mod(r0[w], d0.v[w], pc.p);
            r1[w] = add_mod(r1[w], d1.v[w], pc.p);
        }
    }
    if (acc & 2) {
        const W4 d = ld(o2);
#pragma unroll
        for (int w = 0; w < 4; ++w) r2[w] = add_mod(r2[w], d.v[w], pc.p);
    }
    st(o0, r0);
    st(o1, r1);
    st(o2, r2);
}

template <int LOGN>
__global__ void __launch_bounds__(BXM) tensor_sum(PcbTensorSumArgs a) {
    tensor_out<LOGN, PCB_TSUM_MAX>(a.out, a.d2, a.a, a.b, a.npairs, a.acc, blockIdx.z, blockIdx.y, a.pr[blockIdx.y]);
}

// one block row per (ciphertext, output): the outputs of one launch are independent sums; the 6.4 KiB argument struct
// is passed by value as a grid constant (kernel parameters up to 32 KiB)
template <int LOGN>
__global__ void __launch_bounds__(BXM) tensor_multi(const __grid_constant__ PcbTensorMultiArgs a) {
    const int o = blockIdx.z % a.nout, c = blockIdx.z / a.nout;
    tensor_out<LOGN, PCB_TMULTI_PAIRS>(a.out[o], a.d2[o], a.a[o], a.b[o], a.npairs, a.acc, c, blockIdx.y,
                                       a.pr[blockIdx.y]);
}

namespace {
bool tensor_refs_ok(const PcbPolyRef& out, const PcbPolyRef& d2, const PcbPolyRef* A, const PcbPolyRef* B, int np) {
    if (!out.base || !d2.base || !ref16(out) || !ref16(d2)) return false;
    for (int j = 0; j < np; ++j)
        if (!A[j].base || !B[j].base || !ref16(A[j]) || !ref16(B[j])) return false;
    return true;
}
}  // namespace

template <int LOGN>
int tensor_sum_launch(const PcbTensorSumArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbTensorSumArgs& a = *ap;
    if (a.npairs < 1 || a.npairs > PCB_TSUM_MAX || a.n < 0 || a.K < 0 || !a.pr ||
        !tensor_refs_ok(a.out, a.d2, a.a, a.b, a.npairs))
        return PCB_BAD_ARGS;
    if (a.n == 0 || a.K == 0) return 0;
    tensor_sum<LOGN><<<dim3((1 << LOGN) / (BXM * 4), a.n, a.K), BXM, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int tensor_multi_launch(const PcbTensorMultiArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbTensorMultiArgs& a = *ap;
    if (a.nout < 1 || a.nout > PCB_TMULTI_OUT || a.npairs < 1 || a.npairs > PCB_TMULTI_PAIRS || a.n < 0 || a.K < 0 ||
        !a.pr)
        return PCB_BAD_ARGS;
    for (int o = 0; o < a.nout; ++o)
        if (!tensor_refs_ok(a.out[o], a.d2[o], a.a[o], a.b[o], a.npairs)) return PCB_BAD_ARGS;
    if (a.n == 0 || a.K == 0) return 0;
    tensor_multi<LOGN><<<dim3((1 << LOGN) / (BXM * 4), a.n, a.K * a.nout), BXM, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

// ------------------------------------------------------------------------------------------------ epilogues
// md_epilogue_to: dst = a +- (x - t) binv over Q rows [0, n), both parts; rescale_combine_to: out = alpha x + tmp
template <int LOGN>
__global__ void __launch_bounds__(BXM) md_epilogue_to(PcbMdEpiToArgs b) {
    const PcbMdEpiArgs& m = b.m;
    const int row = blockIdx.y, c = blockIdx.z >> 1, part = blockIdx.z & 1;
    const uint64_t p = m.pr[row].p;
    const size_t i = word0();
    const uint64_t bi = ((const uint64_t*)m.binv)[row], bis = ((const uint64_t*)m.binvs)[row];
    const W4 x = ld(at_row(m.x, c, part, row, LOGN) + i), t = ld(at_row(m.t, c, part, row, LOGN) + i);
    const W4 av = ld(at_row(b.a, c, part, row, LOGN) + i);
    uint64_t r[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint64_t v = shoup(sub_mod(x.v[w], t.v[w], p), bi, bis, p);
        r[w] = b.sub ? sub_mod(av.v[w], v, p) : add_mod(av.v[w], v, p);
    }
    st(at_row_w(m.dst, c, part, row, LOGN) + i, r);
}

template <int LOGN>
__global__ void __launch_bounds__(BXM) rescale_combine_to(PcbRescaleCombineToArgs b) {
    const PcbRescaleCombineArgs& a = b.a;
    const int row = blockIdx.y, c = blockIdx.z >> 1, part = blockIdx.z & 1;
    const uint64_t p = a.pr[row].p;
    const size_t i = word0();
    const uint64_t al = ((const uint64_t*)a.alpha)[row], als = ((const uint64_t*)a.alphas)[row];
    const W4 x = ld(at_row(a.x, c, part, row, LOGN) + i), t = ld(at_row(a.tmp, c, part, row, LOGN) + i);
    uint64_t r[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) r[w] = add_mod(shoup(x.v[w], al, als, p), t.v[w], p);
    st(at_row_w(b.out, c, part, row, LOGN) + i, r);
}

template <int LOGN>
int md_epilogue_to_launch(const PcbMdEpiToArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbMdEpiArgs& m = ap->m;
    if (m.n < 0 || m.K < 0 || !m.pr || !m.dst.base || !m.x.base || !m.t.base || !ap->a.base || !m.binv || !m.binvs ||
        !ref16(m.dst) || !ref16(m.x) || !ref16(m.t) || !ref16(ap->a))
        return PCB_BAD_ARGS;
    if (m.n == 0 || m.K == 0) return 0;
    md_epilogue_to<LOGN><<<dim3((1 << LOGN) / (BXM * 4), m.n, 2 * m.K), BXM, 0, s>>>(*ap);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int rescale_combine_to_launch(const PcbRescaleCombineToArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbRescaleCombineArgs& a = ap->a;
    if (a.n < 0 || a.K < 0 || !a.pr || !a.x.base || !a.tmp.base || !ap->out.base || !a.alpha || !a.alphas ||
        !ref16(a.x) || !ref16(a.tmp) || !ref16(ap->out))
        return PCB_BAD_ARGS;
    if (a.n == 0 || a.K == 0) return 0;
    rescale_combine_to<LOGN><<<dim3((1 << LOGN) / (BXM * 4), a.n, 2 * a.K), BXM, 0, s>>>(*ap);
    return PCB_LAUNCH_RESULT();
}

// rescale_fwd (two dropped primes): the corrections tmp_i (rescale_coef) and their forward NTT with its epilogue
// (`ntt`, normally 3 = MUL_ADD: x_i = alpha_i x_i + NTT(tmp_i)). The reference generates tmp_i inside the transform's
// column pass from two prepared rows; here rescale_coef writes them and the transform runs in place, the same words
// out in x (tmp is scratch either way). The reference's argument rules: ndrop 2, no out-of-place source.
template <int LOGN>
int rescale_fwd_launch(const PcbRescaleNttArgs* ap, cudaStream_t s) {
    if (!ap || ap->rs.ndrop != 2 || ap->ntt.soff || ap->ntt.epi < 0 || ap->ntt.epi > 3) return PCB_BAD_ARGS;
    const int rc = rescale_coef_launch<LOGN>(&ap->rs, s);
    if (rc) return rc;
    return ntt::fwd<LOGN>(&ap->ntt, s);
}

// ------------------------------------------------------------------------------------------------ subring switch
// pack_split (coefficient form): digit j of row y keeps the coefficients whose exponent is j mod sub, zeros elsewhere;
// rows y < nq come from q, the others from p (row y - nq). Four words per thread: their classes are consecutive.
template <int LOGN>
__global__ void __launch_bounds__(BXM) pack_split(PcbPackSplitArgs a) {
    const int y = blockIdx.y, c = blockIdx.z;
    const size_t i = word0();
    const uint64_t* src = y < a.nq ? (const uint64_t*)a.q + (size_t)c * a.q_stride + ((size_t)y << LOGN)
                                   : (const uint64_t*)a.p + (size_t)c * a.p_stride + ((size_t)(y - a.nq) << LOGN);
    const W4 v = ld(src + i);
    uint64_t* o = (uint64_t*)a.out + (size_t)c * a.out_stride + ((size_t)y << LOGN) + i;
    const size_t dstride = (size_t)a.nrows << LOGN;
    const uint32_t m = (uint32_t)a.sub - 1;
    for (int j = 0; j < a.sub; ++j) {
        uint64_t r[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) r[w] = ((uint32_t)(i + w) & m) == (uint32_t)j ? v.v[w] : 0;
        st(o + (size_t)j * dstride, r);
    }
}

// pack_dot (evaluation form): s1 = sum_j D_j a_j, s0 = sum_j D_j b_j (+ P c0 on rows y < nq) at prime id rows[y]; the
// digits and the key rows by row index y, c0 and the outputs by prime id. sub <= 16 products of words below 2^62
// stay below 2^128: one reduction.
template <int LOGN>
__global__ void __launch_bounds__(BXM) pack_dot(PcbPackDotArgs a) {
    const int y = blockIdx.y, c = blockIdx.z;
    const uint32_t t = a.rows[y];
    const PcbPrimeConst& pc = a.pr[t];
    const uint64_t p = pc.p;
    const size_t i = word0();
    const size_t koff = ((size_t)y << LOGN) + i, dstride = (size_t)a.nrows << LOGN;
    const uint64_t* dg = (const uint64_t*)a.dig + (size_t)c * a.dig_stride + koff;
    Acc s0[4], s1[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) s0[w] = s1[w] = Acc{0, 0};
    for (int j = 0; j < a.sub; ++j) {
        const W4 x = ld(dg + (size_t)j * dstride);
        const W4 b = ld((const uint64_t*)a.kb + koff + (size_t)j * dstride);
        const W4 k = ld((const uint64_t*)a.ka + koff + (size_t)j * dstride);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            mac(s0[w], x.v[w], b.v[w]);
            mac(s1[w], x.v[w], k.v[w]);
        }
    }
    const size_t roff = ((size_t)t << LOGN) + i;
    uint64_t r0[4], r1[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        r0[w] = reduce(s0[w], pc);
        r1[w] = reduce(s1[w], pc);
    }
    if (y < a.nq) {
        const uint64_t pm = ((const uint64_t*)a.pmod)[t], pms = ((const uint64_t*)a.pmods)[t];
        const W4 x = ld((const uint64_t*)a.c0 + (size_t)c * a.ct_stride + roff);
#pragma unroll
        for (int w = 0; w < 4; ++w) r0[w] = add_mod(r0[w], shoup(x.v[w], pm, pms, p), p);
    }
    st((uint64_t*)a.out0 + (size_t)c * a.out_ct_stride + roff, r0);
    st((uint64_t*)a.out1 + (size_t)c * a.out_ct_stride + roff, r1);
}

__host__ inline bool pack_ok(int sub, int nq, int nrows, int K) {
    return sub >= 2 && sub <= 16 && (sub & (sub - 1)) == 0 && nq >= 0 && nq <= nrows && K >= 1;
}

template <int LOGN>
int pack_split_launch(const PcbPackSplitArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbPackSplitArgs& a = *ap;
    if (!pack_ok(a.sub, a.nq, a.nrows, a.K) || !a.out || (a.nq > 0 && !a.q) || (a.nrows > a.nq && !a.p))
        return PCB_BAD_ARGS;
    if (!al16(a.out) || (a.q && !al16(a.q)) || (a.p && !al16(a.p)) || ((a.q_stride | a.p_stride | a.out_stride) & 1))
        return PCB_BAD_ARGS;
    if (a.nrows == 0) return 0;
    pack_split<LOGN><<<dim3((1 << LOGN) / (BXM * 4), a.nrows, a.K), BXM, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

template <int LOGN>
int pack_dot_launch(const PcbPackDotArgs* ap, cudaStream_t s) {
    if (!ap) return PCB_BAD_ARGS;
    const PcbPackDotArgs& a = *ap;
    if (!pack_ok(a.sub, a.nq, a.nrows, a.K) || !a.dig || !a.kb || !a.ka || !a.out0 || !a.out1 || !a.rows || !a.pr ||
        (a.nq > 0 && (!a.c0 || !a.pmod || !a.pmods)))
        return PCB_BAD_ARGS;
    if (!al16(a.dig) || !al16(a.kb) || !al16(a.ka) || !al16(a.out0) || !al16(a.out1) || (a.c0 && !al16(a.c0)) ||
        ((a.dig_stride | a.ct_stride | a.out_ct_stride) & 1))
        return PCB_BAD_ARGS;
    if (a.nrows == 0) return 0;
    pack_dot<LOGN><<<dim3((1 << LOGN) / (BXM * 4), a.nrows, a.K), BXM, 0, s>>>(a);
    return PCB_LAUNCH_RESULT();
}

#define PCB_MULTI_INST(L)                                                                    \
    template int pack_split_launch<L>(const PcbPackSplitArgs*, cudaStream_t);                \
    template int pack_dot_launch<L>(const PcbPackDotArgs*, cudaStream_t);                    \
    template int ew_many_launch<L>(const PcbEwManyArgs*, cudaStream_t);                      \
    template int submul_many_launch<L>(const PcbSubMulManyArgs*, cudaStream_t);              \
    template int wsum_launch<L>(const PcbWsumArgs*, cudaStream_t);                           \
    template int wsum_k_launch<L>(const PcbWsumKArgs*, cudaStream_t);                        \
    template int wsum_multi_launch<L>(const PcbWsumMultiArgs*, cudaStream_t);                \
    template int tensor_sum_launch<L>(const PcbTensorSumArgs*, cudaStream_t);                \
    template int tensor_multi_launch<L>(const PcbTensorMultiArgs*, cudaStream_t);            \
    template int md_epilogue_to_launch<L>(const PcbMdEpiToArgs*, cudaStream_t);              \
    template int rescale_combine_to_launch<L>(const PcbRescaleCombineToArgs*, cudaStream_t); \
    template int rescale_fwd_launch<L>(const PcbRescaleNttArgs*, cudaStream_t);
PCB_MULTI_INST(14)
PCB_MULTI_INST(16)

}  // namespace elem
}  // namespace pcb
