/*
 * perseus-b200 — the C ABI of the B200-native CKKS hot path.
 *
 * Two layers, both plain C (pointers and sizes; no torch types):
 *
 *  1. The launcher table that the reference's device runtime binds (crates/pc-kernels/kernels/args.cuh:1034-1097,
 *     Rust mirror crates/pc-kernels/src/args.rs, loader crates/pc-kernels/src/table.rs:325-336):
 *        const PcbKernelTable* pc_table_u64_barrett64(void);   ring N = 2^16
 *        const PcbRingTable*   pc_ring_u64_14(void);           ring N = 2^14 (args.cuh:1099-1119)
 *     Every argument struct below keeps the reference's field order, types and size (checked by static asserts and
 *     by tests/test_abi.py) so a reference caller's #[repr(C)] values can be handed over unchanged. Launchers copy
 *     their arguments, are stream-ordered and return 0 (ok), -1 / -2 (argument out of range) or a positive
 *     cudaError_t (args.cuh:1036). Entries this library does not provide are non-null and return -1.
 *     Rows are moved 16 bytes at a time: row bases must be 16-byte aligned and row strides even (in words); the
 *     NTT and element-wise launchers refuse other pointers with -1 (device allocations are 256-byte aligned).
 *
 *  2. The evaluator (the reference's pc-gpu Evaluator / KeySwitcher / Rescaler, crates/pc-gpu/src/{relin,rotate,
 *     ks,rescale,encrypt,keygen}.rs): a context over one chain with device-resident keys, and ciphertext ops on
 *     caller-owned device buffers (pcb_*). The same return-code convention; pcb_last_error() gives the message.
 *
 * Words are uint64_t residues in [0, p). A row holds N words. A ciphertext of the evaluator is [2][nq + kp][N]
 * words (part 0 = c0, part 1 = c1; row r = prime id r; Q ids 0..nq-1 then the special ids), evaluation form
 * (bit-reversed negacyclic NTT order), matching the reference's layout (crates/pc-gpu/src/poly.rs).
 */
#ifndef PCB200_H
#define PCB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__CUDACC__) || defined(PCB_WITH_CUDA_RUNTIME)
#include <cuda_runtime_api.h>
#else
typedef struct CUstream_st* cudaStream_t;
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ================================================================ 1. launcher table (args.cuh layouts) */

/* args.cuh:38-49: per prime id, 64 bytes. u64 words: mu = floor((2^128 - 1) / p) split into mu_lo / mu_hi. */
typedef struct PcbPrimeConst {
    uint64_t p, mu_lo, mu_hi, neal_mu;
    uint32_t bits, word_bits;
    uint64_t mont_pinv, mont_r2, split;
} PcbPrimeConst;

/* args.cuh:51-58: grid row y -> prime id y < nq ? y : qmax + (y - nq) */
typedef struct PcbRowSet {
    int32_t nq, np, qmax, pad;
} PcbRowSet;

/* args.cuh:60-65: part `part` of ciphertext c, row r at base + c*ct_stride + part*part_stride + r*N words */
typedef struct PcbPolyRef {
    void* base;
    uint64_t ct_stride, part_stride;
} PcbPolyRef;

/* args.cuh:67-107: in-place negacyclic NTT of nrows rows (row i at base + roff[i]*N, prime id rprime[i]);
 * twiddles [prime id][N] bit-reversed (fw[m+i] = psi^brev(m+i)) with Shoup companions; soff: out-of-place sources
 * (sum of snum rows sstride words apart); forward epilogues epi 1: eout = (x - v) es, 2: eout = d + (x - v) es,
 * 3: eout = x es + v; inverse: es non-null scales row i by es[i] in place of N^-1. */
typedef struct PcbNttArgs {
    void* base;
    const uint32_t* roff;
    const int32_t* rprime;
    const void* fw;
    const void* fws;
    const void* iw;
    const void* iws;
    const void* ninv;
    const void* ninvs;
    const PcbPrimeConst* pr;
    int32_t nrows, chunk;
    const void* src;
    const uint32_t* soff;
    void* eout;
    const void* ex;
    const void* es;
    const void* ess;
    int32_t epi, snum;
    uint64_t sstride;
    int32_t xnum, lazy;
    uint64_t xstride;
    const void* ed;
} PcbNttArgs;

/* args.cuh:109-141: batched fast base conversion, pool layout src_row[ns] src_prime[ns] pre[ns] tgt_row[nt]
 * tgt_prime[nt] M[ns][nt] (words). out_t = sum_i y_i M[i][t] mod t, y_i = x_i pre_i (or x_i when prescaled). */
typedef struct PcbBconvJob {
    uint32_t src_off, dst_off, nsrc, ntgt, pool_off, exact, prescaled, split;
} PcbBconvJob;
typedef struct PcbBconvArgs {
    const void* src;
    void* dst;
    const PcbBconvJob* jobs;
    const void* pool;
    const PcbPrimeConst* pr;
    int32_t njobs, max_tgt;
    int32_t kind, pad;
} PcbBconvArgs;

/* args.cuh:143-157: ew_add (sub: a - b), ew_scale (a * sc[row]), ew_sub_mul ((a - b) * sc[row]), ew_copy */
typedef struct PcbEwArgs {
    PcbPolyRef out, a, b;
    PcbRowSet rs;
    const void* sc;
    const void* scs;
    const PcbPrimeConst* pr;
    int32_t K, nparts, sub, zero_p;
} PcbEwArgs;

/* args.cuh:202-228: key inner product of K ciphertexts x R keys; outputs at automorph_slot(autok[r], i) */
#define PCB_KS_ACC 4
typedef struct PcbKsArgs {
    const void* c1;
    const void* modup;
    const void* c0;
    void* out0;
    void* out1;
    const void* const* kb;
    const void* const* ka;
    const uint32_t* autok;
    const uint32_t* rows;
    const int32_t* digit_of;
    const void* pmod;
    const void* pmods;
    const PcbPrimeConst* pr;
    uint64_t ct_stride, mu_ct_stride, mu_digit_stride, out_ct_stride, out_rot_stride, key_digit_stride;
    int32_t K, R, ndig, c0_mode, nq, nrows;
} PcbKsArgs;

/* args.cuh:258-271 (relin epilogue), :273-283 (KeyTab), :285-304 (KsRegenArgs), :764-768 (KsKeyArgs).
 * ks_dot_regen: the relinearization inner product (K <= 4, no automorphism, no c0 term) with the key's `a`
 * regenerated from `seed` by the frozen u64 expander lane (w13 = digit, the row's prime), `b` from ks.kb[0] (dense
 * prime-id rows, key_digit_stride) or, with key.kb set, key 0 of the table (dense rows in the key's slot order);
 * use_epi writes dst = f (alpha dst + (dot - conv) binv) [+ k on part 0] [+ add] on both parts instead of out0/out1.
 * ks_dot_key: ks_dot (K <= 4 x R keys, automorphism, c0 modes, PCB_KS_ACC) with the keys read through the table:
 * `a` regenerated for digits below key.nregen (key.seed[r]), else ks.ka[r]; `b` dense in the key's slot order
 * (Q id t <= q_top at slot t, special id nq + j at q_top + 1 + j; q_top < 0: slot = prime id). Packed `b` rows
 * (key.bits != 0, the reference's 32-bit words) are refused. */
typedef struct PcbEpiArgs {
    void* dst;
    const void* conv;
    const void* binv;
    const void* binvs;
    const void* k;
    uint64_t part_stride;
    int32_t dbl, pad;
    const void* alpha;
    const void* alphas;
} PcbEpiArgs;
typedef struct PcbKeyTab {
    const void* const* kb;
    const uint32_t* const* seed;
    uint64_t row_words;
    int32_t bits, q_top, srows, nregen;
} PcbKeyTab;
typedef struct PcbKsRegenArgs {
    PcbKsArgs ks;
    const uint32_t* seed;
    PcbEpiArgs epi;
    int32_t use_epi, pad;
    PcbKeyTab key;
    const void* add;
} PcbKsRegenArgs;
typedef struct PcbKsKeyArgs {
    PcbKsArgs ks;
    PcbKeyTab key;
} PcbKsKeyArgs;

/* args.cuh:909-927 (coeff_sum): out (+)= sum_{r < n} ct[r] pt_r over Q limbs 0..L-1 (prime id = limb), pt_r[k] =
 * round(rows[r][k] scale) (half to even; past the int64 range clamped to +-2^62 and counted per limb in *overflow when
 * non-null) mod p_l, in the NTT domain (fw / fws: the forward twiddle tables of ntt_fwd). ct[r] and out: part 0 row 0,
 * part 1 at + part_stride words, row l at + l N. rows[r]: N float32 coefficients in device memory. scratch: n L N
 * words. accumulate != 0 adds onto out. n in [1, 32], L in [1, 64]. */
#define PCB_COEFF_MAXT 32
#define PCB_COEFF_MAXL 64
typedef struct PcbCoeffArgs {
    void* scratch;
    void* out;
    const void* fw;
    const void* fws;
    const PcbPrimeConst* pr;
    unsigned long long* overflow;
    uint64_t part_stride;
    double scale;
    int32_t n, L, accumulate, pad;
    const float* rows[PCB_COEFF_MAXT];
    const void* ct[PCB_COEFF_MAXT];
} PcbCoeffArgs;

/* args.cuh:230-242 (pack_split, the subring switch): rows y < nq of polynomial c at q + c q_stride + y N, the others
 * at p + c p_stride + (y - nq) N (coefficient form); digit j (the exponents = j mod sub, zeros elsewhere) written
 * at out + c out_stride + (j nrows + y) N. sub in {2, 4, 8, 16}, 0 <= nq <= nrows, K >= 1. */
typedef struct PcbPackSplitArgs {
    const void* q;
    const void* p;
    void* out;
    uint64_t q_stride, p_stride, out_stride;
    int32_t K, sub, nq, nrows;
} PcbPackSplitArgs;

/* args.cuh:244-261 (pack_dot, evaluation form): s1 = sum_j D_j a_j, s0 = sum_j D_j b_j (+ P c0 on rows y < nq) at prime
 * id rows[y]; D as pack_split's out (dig, dig_stride), kb / ka [digit][row y][N]; c0 and the outputs by prime id
 * rows, polynomial c at + c ct_stride / + c out_ct_stride. */
typedef struct PcbPackDotArgs {
    const void* dig;
    const void* kb;
    const void* ka;
    const void* c0;
    void* out0;
    void* out1;
    const uint32_t* rows;
    const void* pmod;
    const void* pmods;
    const PcbPrimeConst* pr;
    uint64_t dig_stride, ct_stride, out_ct_stride;
    int32_t K, sub, nq, nrows;
} PcbPackDotArgs;

/* args.cuh:325-352 (cts_fused): one BSGS stage of CoeffToSlot with its baby rotations hoisted and never written, in
 * the extended basis (Q rows and the special rows), K ciphertexts. For output slot o of row rows[y] (prime id t):
 *   rot_0[o] = (P c0[o], P c1[o]) on Q rows, 0 on special rows (x0 non-null: the stored extended x0 row instead);
 *   rot_i[o] = (P c0[s] + sum_d D_d[s] kb[i-1]_d[s], sum_d D_d[s] ka[i-1]_d[s]), s = automorph_slot(kinv[i-1], o),
 *              D_d = c1 on digit d's own Q rows, else the ModUp output of digit d;
 *   res_j[o] = sum_{i < B, B j + i < npts} rot_i[o] pts[B j + i][o]  for j < G <= 2.
 * x: ct c at x + c ct_stride (c1 at + part_stride); modup: + c mu_ct_stride + d mu_digit_stride; keys [digit][prime id][N]
 * (key_digit_stride); pts rows: Q prime id t at row t, special ids at pt_prow + (t - nq), ptw words, compact index enc;
 * res (c, j) at res + (c G + j) ct_stride. ngrp is the launcher's; kmax a grouping hint; pair_cts must be 0 here. */
typedef struct PcbCtsArgs {
    const void* x;
    const void* modup;
    void* res;
    const void* const* kb;
    const void* const* ka;
    const uint32_t* kinv;
    const void* const* pts;
    const uint32_t* rows;
    const int32_t* digit_of;
    const void* pmod;
    const void* pmods;
    const PcbPrimeConst* pr;
    uint64_t ct_stride, part_stride, mu_ct_stride, mu_digit_stride, key_digit_stride;
    int32_t K, B, G, npts, ndig, nq, nlive, ptw, pt_prow;
    uint32_t enc;
    int32_t ngrp;
    int32_t nrows, kmax;
    int32_t pair_cts;
    const void* x0;
} PcbCtsArgs;

/* args.cuh:754-758 (cts_fused_regen): cts_fused with the baby keys read through the key table: `b` dense rows of
 * key.kb[i-1] in the key's slot order, `a` regenerated from key.seed[i-1] below key.nregen (cts.ka[i-1] above). */
typedef struct PcbCtsRegenArgs {
    PcbCtsArgs cts;
    PcbKeyTab key;
} PcbCtsRegenArgs;

/* args.cuh:306-323: out[d][m][N] = expander(seed, digit d, prime prime_ids[m]) (u64: the frozen KSKB lane) */
typedef struct PcbKskExpandArgs {
    void* out;
    const uint32_t* seed;
    const int32_t* prime_ids;
    const PcbPrimeConst* pr;
    int32_t nmod, dnum;
    int32_t d0, pad;
} PcbKskExpandArgs;

/* args.cuh:355-367: (c0, c1, d2) (= | +=) sum_j (a0 b0, a0 b1 + a1 b0, a1 b1) over Q rows [0, n) of K cts */
typedef struct PcbTensorArgs {
    PcbPolyRef out, d2, a0, b0, a1, b1;
    void* coef;
    uint64_t coef_ct_stride;
    const PcbPrimeConst* pr;
    int32_t npairs, acc, n, K;
    int32_t dbl, acc_d2;
} PcbTensorArgs;

/* args.cuh:369-378 (tensor_y): the tensor above, then (c0, c1) += c[row] y (sub: -=) with Shoup companion cs[row],
 * both parts of y, after the doubling; d2 unchanged. EvalMod's x y +- c t before its relinearization in one pass. */
typedef struct PcbTensorYArgs {
    PcbTensorArgs t;
    PcbPolyRef y;
    const void* c;
    const void* cs;
    int32_t sub, pad;
} PcbTensorYArgs;

/* args.cuh:184-200: BSGS plaintext dot of K ciphertexts' baby rotations (rows of rs, both parts):
 *   res[c][j] = sum_{b < bstep, d = bstep j + b < npts} rot[c][b] * pts[d]   for j < gstep
 * rot (c, b) at rot.base + c rot.ct_stride + b rot_stride, res (c, j) at res.base + c res.ct_stride + j res_stride.
 * pts[d] (a device array of device pointers): rows of ptw words, Q rows at their grid index y, special rows at
 * pt_prow + (y - nq); word i read at the compact index (enc = 0xFFFFFFFF: i; (enc >> 24) == 0x7F: i >> (enc & 0xFF);
 * else i & enc). K <= 8; bstep (max p)^2 below 2^128 (128-bit sums, one reduction). */
typedef struct PcbPtDotArgs {
    PcbPolyRef rot, res;
    uint64_t rot_stride, res_stride;
    const void* const* pts;
    const PcbPrimeConst* pr;
    PcbRowSet rs;
    int32_t npts, bstep, gstep, K;
    int32_t ptw, pt_prow;
    uint32_t enc;
    int32_t pad;
} PcbPtDotArgs;

/* args.cuh:491-498: part 0 of K ciphertexts += k[row] over rows [0, n) (k raw words, k == p allowed) */
typedef struct PcbAddConstArgs {
    PcbPolyRef x;
    const void* k;
    const PcbPrimeConst* pr;
    int32_t n, K;
} PcbAddConstArgs;

/* args.cuh:500-506: out = in * t[row] over rows [0, n) of K ciphertexts, both parts (t: [row][N] words) */
typedef struct PcbMulTableArgs {
    PcbPolyRef out, in;
    const void* t;
    const PcbPrimeConst* pr;
    int32_t n, K;
} PcbMulTableArgs;

/* args.cuh:508-515: out = y + m (sub 0), y - m (1), m - y (2), m = in * t as mul_table; out may alias y or in */
typedef struct PcbMulAddArgs {
    PcbMulTableArgs m;
    PcbPolyRef y;
    int32_t sub, pad;
} PcbMulAddArgs;

/* args.cuh:517-528: out = y + sum_{j < nterm} x[j] * t[j] (y.base null: no y), rows [0, n) of K ciphertexts, both
 * parts, nterm <= 8; lazy selects one reduction of the 128-bit sum or one per product (the same canonical words) */
typedef struct PcbMulAddNArgs {
    PcbPolyRef out, y;
    PcbPolyRef x[8];
    const void* t[8];
    const PcbPrimeConst* pr;
    int32_t n, K, nterm, lazy;
} PcbMulAddNArgs;

/* args.cuh:438-447: for parts 0, 1: dst = f (dst + (x - t) binv) [+ k on part 0], f = 2 when dbl */
typedef struct PcbMdEpiArgs {
    PcbPolyRef dst, x, t;
    const void* binv;
    const void* binvs;
    const void* k;
    const PcbPrimeConst* pr;
    int32_t dbl, n, K, pad;
} PcbMdEpiArgs;

/* args.cuh:525-572: composite rescale; ndrop 1: tmp_i = A_i lift(y_top); combine x_i = alpha_i x_i + tmp_i */
typedef struct PcbRescaleArgs {
    PcbPolyRef x, tmp;
    const void* A;
    const void* B;
    const void* As;
    const void* Bs;
    const void* qam;
    const void* qbm;
    const PcbPrimeConst* pr;
    uint64_t qinv_ab, C_ab, ca, cb;
    int32_t top, nrows, K, ndrop;
} PcbRescaleArgs;
typedef struct PcbRescaleCombineArgs {
    PcbPolyRef x, tmp;
    const void* alpha;
    const void* alphas;
    const PcbPrimeConst* pr;
    int32_t n, K;
} PcbRescaleCombineArgs;

/* args.cuh:553-562: rescale_fwd, rescale_coef's corrections and their forward NTT `ntt` (rows of tmp, epilogue 3 = MUL_ADD:
 * x = alpha x + NTT(tmp)) in one entry (the corrections are written to tmp here; the reference forms them inside the
 * transform: the same words in x) */
typedef struct PcbRescaleNttArgs {
    PcbRescaleArgs rs;
    PcbNttArgs ntt;
} PcbRescaleNttArgs;

/* args.cuh:573-578: rescale_combine_to, out = alpha x + tmp (x read only) */
typedef struct PcbRescaleCombineToArgs {
    PcbRescaleCombineArgs a;
    PcbPolyRef out;
} PcbRescaleCombineToArgs;

/* args.cuh:580-592: out[o] = in[automorph_slot(k, o)] (+ add[o]) over row set rs, K cts x nparts parts */
typedef struct PcbAutomorphArgs {
    PcbPolyRef out, in, add;
    PcbRowSet rs;
    const PcbPrimeConst* pr;
    uint32_t k;
    int32_t K, nparts, has_add;
} PcbAutomorphArgs;

/* args.cuh:613-628: c0 = -a s + e + m, c1 = a, a from the ENCA lane (u64: ENCB) keyed by the nonce */
typedef struct PcbEncryptArgs {
    void* c0;
    void* c1;
    const void* s;
    const void* e;
    const void* m;
    const uint32_t* seed;
    const PcbPrimeConst* pr;
    uint32_t nonce;
    int32_t nl;
} PcbEncryptArgs;

/* args.cuh:630-654: b = e - a s_new + [digit] P s_old' (dense rows only at u64: bits must be 0) */
typedef struct PcbKskGenArgs {
    void* b;
    void* a;
    const void* e;
    const void* s_new;
    const void* s_old;
    const uint32_t* seed;
    const int32_t* ids;
    const int32_t* digit_of;
    const void* pmod;
    const void* pmods;
    const PcbPrimeConst* pr;
    uint64_t row_words;
    int32_t nrows, ndig, nq, bits, sq, pad;
} PcbKskGenArgs;

/* args.cuh:159-170: ew_many, out[j] = a[j] (+ b[j]) (+ c[j]) for n <= 48 polynomials by pointer, Q rows [0, nrows) (row r
 * at + r N words; a null b / c skipped; out may alias its sources) */
#define PCB_EWM_MAX 48
typedef struct PcbEwManyArgs {
    void* out[PCB_EWM_MAX];
    const void* a[PCB_EWM_MAX];
    const void* b[PCB_EWM_MAX];
    const void* c[PCB_EWM_MAX];
    const PcbPrimeConst* pr;
    int32_t n, nrows;
} PcbEwManyArgs;

/* args.cuh:172-182: submul_many, out[j] = (a[j] - b[j]) t[row] for n <= 48 polynomials (t one table of nrows rows) */
typedef struct PcbSubMulManyArgs {
    void* out[PCB_EWM_MAX];
    const void* a[PCB_EWM_MAX];
    const void* b[PCB_EWM_MAX];
    const void* t;
    const PcbPrimeConst* pr;
    int32_t n, nrows;
} PcbSubMulManyArgs;

/* args.cuh:380-389: tensor_sum, c0 = sum_j a0 b0, c1 = sum_j a0 b1 + a1 b0 into out, d2 = sum_j a1 b1 into part 1 of d2, over
 * npairs <= 16 pairs (acc as tensor's) */
#define PCB_TSUM_MAX 16
typedef struct PcbTensorSumArgs {
    PcbPolyRef out, d2;
    PcbPolyRef a[PCB_TSUM_MAX], b[PCB_TSUM_MAX];
    const PcbPrimeConst* pr;
    int32_t npairs, acc, n, K;
} PcbTensorSumArgs;

/* args.cuh:391-404: tensor_multi, nout <= 4 tensor sums of npairs <= 32 pairs in one launch */
#define PCB_TMULTI_OUT 4
#define PCB_TMULTI_PAIRS 32
typedef struct PcbTensorMultiArgs {
    PcbPolyRef out[PCB_TMULTI_OUT], d2[PCB_TMULTI_OUT];
    PcbPolyRef a[PCB_TMULTI_OUT][PCB_TMULTI_PAIRS], b[PCB_TMULTI_OUT][PCB_TMULTI_PAIRS];
    const PcbPrimeConst* pr;
    int32_t nout, npairs, acc, n, K, pad;
} PcbTensorMultiArgs;

/* args.cuh:449-457: md_epilogue_to, dst = a +- (x - t) binv over Q rows [0, n), both parts (sub: minus) */
typedef struct PcbMdEpiToArgs {
    PcbMdEpiArgs m;
    PcbPolyRef a;
    int32_t sub, pad;
} PcbMdEpiToArgs;

/* args.cuh:459-468: wsum, out = sum_{j < nsrc <= 8} w[j rowstride + row] src_j (both parts, Shoup companions ws), rows
 * [0, n) */
typedef struct PcbWsumArgs {
    PcbPolyRef out;
    PcbPolyRef src[8];
    const void* w;
    const void* ws;
    const PcbPrimeConst* pr;
    int32_t nsrc, rowstride, n, K;
} PcbWsumArgs;

/* args.cuh:470-474: wsum_k, wsum then part 0 += k[row] (raw, reduced once when >= p) */
typedef struct PcbWsumKArgs {
    PcbWsumArgs w;
    const void* k;
} PcbWsumKArgs;

/* args.cuh:476-489: wsum_multi, nout <= 3 weighted sums of one source list, out[m] on rows [0, n[m]) (k[m]: wsum_k's) */
typedef struct PcbWsumMultiArgs {
    PcbPolyRef out[3];
    PcbPolyRef src[8];
    const void* w[3];
    const void* ws[3];
    const void* k[3];
    const PcbPrimeConst* pr;
    int32_t nout, nsrc, rowstride, K;
    int32_t n[3], nmax;
} PcbWsumMultiArgs;

/* args.cuh:656-663: packed key rows -> dense rows, out[r][i] = value i of packed row r (in + r row_words), r < nrows.
 * Values are `bits` bits LSB first (the wire format's pack_row order); the reference's u64 table takes bits 1..32, this
 * one 1..64 (a 50-bit residue of these chains packs at 50). */
typedef struct PcbKskUnpackArgs {
    void* out;
    const uint32_t* in;
    uint64_t row_words;
    int32_t nrows, bits;
} PcbKskUnpackArgs;

/* args.cuh:665-677: composite ModRaise, coefficient form: for rows t in [r0, r1) of K ciphertexts (nparts polynomials
 * from part 0), x[t] = sum_{k < d} centred([x_k qhatinv_k]_{q_k}) qhat[k][t] mod q_t, the sources x_k = rows 0..d-1
 * of the same polynomial (d <= 4, t < 64; the sources are not written). d = 1, qhatinv = qhat = 1: the level-0 raise
 * of CKKS bootstrapping (every row t gets the centred lift of row 0). */
typedef struct PcbModRaiseArgs {
    void* x;
    const PcbPrimeConst* pr;
    uint64_t ct_stride, part_stride;
    uint64_t qhatinv[4];
    uint64_t qhat[4][64];
    int32_t K, d, r0, r1, nparts, pad;
} PcbModRaiseArgs;

/* args.cuh:892-907 (small_int1): the exact post-raise scaling from one source prime, in place over rows [0, nrows)
 * of K cts (nparts polynomials from part 0, coefficient form): x = row 0 centred against q0, q = round(|x| mc / 2^sh)
 * (half up; 1 <= sh <= 127, q < 2^64 by the caller), row t := sign(x) q mod q_t. Row 0 is read before any write. */
typedef struct PcbSmallInt1Args {
    void* x;
    const PcbPrimeConst* pr;
    uint64_t ct_stride, part_stride;
    uint64_t mc;
    int32_t sh, nrows, K, nparts;
} PcbSmallInt1Args;

typedef int (*PcbLaunch)(const void* args, cudaStream_t stream);

/* args.cuh:1034-1097: 16-byte header then 52 launchers, in the reference's order */
typedef struct PcbKernelTable {
    uint32_t abi, word_bytes, mm, log_n;
    int (*ntt_fwd)(const PcbNttArgs*, cudaStream_t);
    int (*ntt_inv)(const PcbNttArgs*, cudaStream_t);
    int (*bconv)(const PcbBconvArgs*, cudaStream_t);
    int (*ew_add)(const PcbEwArgs*, cudaStream_t);
    int (*ew_scale)(const PcbEwArgs*, cudaStream_t);
    int (*ew_sub_mul)(const PcbEwArgs*, cudaStream_t);
    int (*ew_copy)(const PcbEwArgs*, cudaStream_t);
    int (*pt_dot)(const PcbPtDotArgs*, cudaStream_t);
    int (*ks_dot)(const PcbKsArgs*, cudaStream_t);
    int (*ks_dot_regen)(const PcbKsRegenArgs*, cudaStream_t);
    int (*ksk_expand)(const PcbKskExpandArgs*, cudaStream_t);
    int (*cts_fused)(const PcbCtsArgs*, cudaStream_t);
    int (*tensor)(const PcbTensorArgs*, cudaStream_t);
    int (*md_epilogue)(const PcbMdEpiArgs*, cudaStream_t);
    int (*wsum)(const PcbWsumArgs*, cudaStream_t);
    int (*add_const)(const PcbAddConstArgs*, cudaStream_t);
    int (*mul_table)(const PcbMulTableArgs*, cudaStream_t);
    int (*rescale_coef)(const PcbRescaleArgs*, cudaStream_t);
    int (*rescale_combine)(const PcbRescaleCombineArgs*, cudaStream_t);
    int (*automorph)(const PcbAutomorphArgs*, cudaStream_t);
    PcbLaunch encode;
    int (*encrypt)(const PcbEncryptArgs*, cudaStream_t);
    int (*ksk_gen)(const PcbKskGenArgs*, cudaStream_t);
    int (*ksk_unpack)(const PcbKskUnpackArgs*, cudaStream_t);
    int (*mod_raise)(const PcbModRaiseArgs*, cudaStream_t);
    PcbLaunch small_int, spru_extract, spru_fft_pass, spru_scatter;
    int (*cts_fused_regen)(const PcbCtsRegenArgs*, cudaStream_t);
    int (*ks_dot_key)(const PcbKsKeyArgs*, cudaStream_t);
    PcbLaunch pcmm, ccmm;
    int (*wsum_k)(const PcbWsumKArgs*, cudaStream_t);
    int (*rescale_combine_to)(const PcbRescaleCombineToArgs*, cudaStream_t);
    int (*md_epilogue_to)(const PcbMdEpiToArgs*, cudaStream_t);
    int (*small_int1)(const PcbSmallInt1Args*, cudaStream_t);
    int (*coeff_sum)(const PcbCoeffArgs*, cudaStream_t);
    int (*mul_add)(const PcbMulAddArgs*, cudaStream_t);
    int (*rescale_fwd)(const PcbRescaleNttArgs*, cudaStream_t);
    int (*mul_add_n)(const PcbMulAddNArgs*, cudaStream_t);
    int (*tensor_y)(const PcbTensorYArgs*, cudaStream_t);
    int (*wsum_multi)(const PcbWsumMultiArgs*, cudaStream_t);
    int (*bconv_wide)(const PcbBconvArgs*, cudaStream_t);
    PcbLaunch tfhe;
    int (*tensor_sum)(const PcbTensorSumArgs*, cudaStream_t);
    int (*tensor_multi)(const PcbTensorMultiArgs*, cudaStream_t);
    PcbLaunch tensor_seeded;
    int (*ew_many)(const PcbEwManyArgs*, cudaStream_t);
    int (*submul_many)(const PcbSubMulManyArgs*, cudaStream_t);
    int (*pack_split)(const PcbPackSplitArgs*, cudaStream_t);
    int (*pack_dot)(const PcbPackDotArgs*, cudaStream_t);
} PcbKernelTable;

/* args.cuh:1099-1119: ring-size tables (rows of 2^log_n words) */
typedef struct PcbRingTable {
    uint32_t abi, word_bytes, mm, log_n;
    int (*ntt_fwd)(const PcbNttArgs*, cudaStream_t);
    int (*ntt_inv)(const PcbNttArgs*, cudaStream_t);
    int (*ntt_fwd_g)(const PcbNttArgs*, cudaStream_t);
    int (*ntt_inv_g)(const PcbNttArgs*, cudaStream_t);
    int (*bconv)(const PcbBconvArgs*, cudaStream_t);
    int (*ew_add)(const PcbEwArgs*, cudaStream_t);
    int (*ew_scale)(const PcbEwArgs*, cudaStream_t);
    int (*ew_sub_mul)(const PcbEwArgs*, cudaStream_t);
    int (*ew_copy)(const PcbEwArgs*, cudaStream_t);
} PcbRingTable;

#define PCB_KERNELS_ABI 30u
#define PCB_RING_ABI 7u

/* replaces `pc_table_u64_barrett64` of crates/pc-kernels/kernels/inst/instantiate.inc:368-428 (u64, Barrett64) */
const PcbKernelTable* pc_table_u64_barrett64(void);
/* replaces `pc_ring_u64_<log_n>` of crates/pc-kernels/kernels/args.cuh:1099-1104 at log_n 14 and 16 */
const PcbRingTable* pc_ring_u64_14(void);
const PcbRingTable* pc_ring_u64_16(void);
/* The full 52-launcher table at log_n 14 or 16 (NULL otherwise): the reference builds one table per ring size
 * (PC_LOGN at compile time); this library carries both. pcb_kernel_table(16) == pc_table_u64_barrett64(). */
const PcbKernelTable* pcb_kernel_table(int32_t log_n);

/* Kernels this library has launched since it was loaded (all threads, all devices). */
uint64_t pcb_launch_count(void);
/* Bounded waits in this library's pipelined kernels (the NTT's bulk-copy stages) that ran out on the current device
 * since the library was loaded: 0 in normal operation; a nonzero count means a copy never completed and the affected
 * rows were left untransformed (synchronizes the device). No counterpart in the reference. */
uint32_t pcb_device_timeouts(void);
/* Measurement: iters x 8 dependent-chain FP64 FMAs on every thread of 4 x 256-thread blocks per SM, on stream s; returns
 * the FMA count (negative: a cudaError_t). Timed by the caller with CUDA events, it gives the FP64 pipe's throughput
 * (the denominator of the benchmark's FP64 fractions). `sink`: one double per block. No counterpart in the reference. */
int64_t pcb_fp64_fma_loop(double* sink, int32_t iters, cudaStream_t s);

/* ================================================================ 2. evaluator */

typedef struct PcbCtx PcbCtx;

/* Chain parameters (the reference's Chain, crates/pc-core/src/params.rs:225-258, given as explicit prime lists). */
typedef struct PcbParams {
    uint32_t log_n;      /* 14 or 16 */
    int32_t nq, kp;      /* Q primes (bottom first), special primes */
    int32_t dnum;        /* hybrid digits: ceil(nq / dnum) limbs each (params.rs:486-495) */
    const uint64_t* q;   /* nq primes, p = 1 mod 2N, < 2^61 */
    const uint64_t* p;   /* kp primes */
    int32_t k_max;       /* ciphertexts per batched key switch */
    int32_t key_source;  /* PCB_KEYS_DENSE or PCB_KEYS_REGEN */
} PcbParams;

/* How the context stores its switching keys (the reference's KeySource, crates/pc-gpu/src/ks.rs:57):
 *  PCB_KEYS_DENSE  b and a resident, 2 dnum (nq + kp) N words per key (the reference's Cached source);
 *  PCB_KEYS_REGEN  b and the 8-word seed of a: a is regenerated from the seed inside every inner product (the frozen
 *                  u64 expander lane), half the bytes per key (the reference's Regen source). The same keys and the
 *                  same results word for word; pcb_key_ptrs gives a = NULL, pcb_key_copy expands a. */
#define PCB_KEYS_DENSE 0
#define PCB_KEYS_REGEN 1

/* Message of the last failed call on this thread (empty when none). */
const char* pcb_last_error(void);

/* Device bytes a context of `prm` needs in its arena (tables, plans, key-switch workspaces for k_max cts) plus
 * `nkeys` switching keys with stored `a`. */
int64_t pcb_ctx_bytes(const PcbParams* prm, int32_t nkeys);
/* Build a context on the current device. `arena` is caller-owned device memory of `arena_bytes` >= pcb_ctx_bytes
 * (the frozen arena of crates/pc-cuda/src/lib.rs:9-10); the context allocates nothing else on the device. */
int pcb_ctx_create(const PcbParams* prm, int32_t nkeys, void* arena, size_t arena_bytes, cudaStream_t stream,
                   PcbCtx** out);
void pcb_ctx_destroy(PcbCtx* ctx);
int pcb_ctx_rows(const PcbCtx* ctx);
/* Device tables: PrimeConst by prime id, and the four NTT twiddle tables [prime id][N] + N^-1 (value, Shoup). */
int pcb_ctx_tables(const PcbCtx* ctx, const PcbPrimeConst** pr, const uint64_t** fw, const uint64_t** fws,
                   const uint64_t** iw, const uint64_t** iws, const uint64_t** ninv, const uint64_t** ninvs);

/* Session keys (crates/pc-gpu/src/keygen.rs:184-284, crates/pc-py/src/session.rs:1438-1450): the DRBG
 * Prng([0x5e551013, lo32(seed), hi32(seed), 4..8], 0) draws the secret (sparse ternary of Hamming weight h; 0 =
 * uniform ternary), then per key (galois[i]; 1 = relinearization) its KSKB seed and error-stream seed, then the
 * encryptor seed. Keys are generated on the device (ksk_gen) into the arena. */
int pcb_keygen(PcbCtx* ctx, uint64_t seed, uint32_t h, double sigma, int32_t ngal, const uint64_t* galois,
               cudaStream_t stream);
/* key `idx` in keygen order: device pointers of b and a ([dnum][nq + kp][N]; a = NULL for PCB_KEYS_REGEN) and its
 * galois element */
int pcb_key_ptrs(const PcbCtx* ctx, int32_t idx, const uint64_t** b, const uint64_t** a, uint64_t* galois);

/* Copy key `idx` (b then a, [dnum][nq + kp][N] words each) into caller device buffers on `stream` (a regenerated
 * key's a is expanded from its seed). */
int pcb_key_copy(const PcbCtx* ctx, int32_t idx, uint64_t* b_out, uint64_t* a_out, cudaStream_t stream);
/* The 8-word KSKB seed key `idx`'s `a` is drawn from (host copy; synchronizes). */
int pcb_key_seed(const PcbCtx* ctx, int32_t idx, uint32_t* seed8);
/* Load key `idx` from a client's material (a key bundle's Ksk entry, crates/pc-client/src/wire.rs:78-85): its galois
 * element (1: relinearization), b ([dnum][nq + kp][N] words, device or host) and the seed of its a (KSKA: the frozen
 * ChaCha12 lane; a dense context expands a once here, a regenerating one keeps the seed). Keys load in order: idx is
 * at most the number already loaded or generated; no secret is needed (a server context). Synchronizes `stream`. */
int pcb_key_load(PcbCtx* ctx, int32_t idx, uint64_t galois, const uint64_t* b, const uint32_t* seed8,
                 cudaStream_t stream);

/* Secret-key encryption of nvals (re, im) values into nslots slots at `scale`, rows 0..=top of ct (device). */
int pcb_encrypt(PcbCtx* ctx, const double* vals, int32_t nvals, int32_t nslots, double scale, int32_t top,
                uint64_t* ct, cudaStream_t stream);
/* Decrypt rows 0..=top of ct (device) to nslots (re, im) values on the host (synchronizes `stream`). */
int pcb_decrypt(PcbCtx* ctx, const uint64_t* ct, int32_t top, int32_t nslots, double scale, double* vals,
                cudaStream_t stream);
/* Encode values into coefficient-form rows 0..=top on the host (plaintext operands of pcb_mult_pt / pcb_add_pt). */
int pcb_encode(PcbCtx* ctx, const double* vals, int32_t nvals, int32_t nslots, double scale, int32_t top,
               uint64_t* rows);
/* Upload host coefficient rows 0..=top and take them to evaluation form into pt (device, [nq][N]). */
int pcb_pt_load(PcbCtx* ctx, const uint64_t* rows_host, int32_t top, uint64_t* pt, cudaStream_t stream);
/* The same over the extended rows: rows 0..=top of the Q primes, then one row per special prime (top + 1 + kp rows),
 * for pcb_linear_transform_ext's plaintexts. No counterpart in the reference's Fhe API (its fused CoeffToSlot stage
 * encodes its diagonals over the special primes too, crates/pc-gpu/src/bts/cts.rs). */
int pcb_encode_ext(PcbCtx* ctx, const double* vals, int32_t nvals, int32_t nslots, double scale, int32_t top,
                   uint64_t* rows);
int pcb_pt_load_ext(PcbCtx* ctx, const uint64_t* rows_host, int32_t top, uint64_t* pt, cudaStream_t stream);

/* Ciphertext ops over K ciphertexts `ct_stride` words apart (0 = one ciphertext layout apart), rows 0..=top. */
int pcb_add(PcbCtx* ctx, const uint64_t* a, const uint64_t* b, uint64_t* out, int32_t top, int32_t K,
            cudaStream_t stream);
int pcb_sub(PcbCtx* ctx, const uint64_t* a, const uint64_t* b, uint64_t* out, int32_t top, int32_t K,
            cudaStream_t stream);
/* out = a * b relinearized, rescale pending (crates/pc-gpu/src/relin.rs:213-232); out may alias a or b */
/* out = a_0 + a_1 + ... + a_(n-1) for n (1 .. 32) batches of K ciphertexts at level top, every input read once; out
 * may be one of the inputs. No counterpart in the reference (its Fhe.add is pairwise): one pass instead of n - 1. */
int pcb_sum(PcbCtx* ctx, const uint64_t* const* ins, int32_t n, uint64_t* out, int32_t top, int32_t K,
            cudaStream_t stream);
int pcb_mult(PcbCtx* ctx, const uint64_t* a, const uint64_t* b, uint64_t* out, int32_t top, int32_t K,
             cudaStream_t stream);
/* in place: rows 0..top-1 = q_top^-1 (x - lift(x_top)) (crates/pc-gpu/src/rescale.rs:230) */
int pcb_rescale(PcbCtx* ctx, uint64_t* ct, int32_t top, int32_t K, cudaStream_t stream);
/* The rescale of ONE ciphertext (as pcb_rescale with K = 1, the same words out) without any workspace from the
 * arena: its working rows live in a fixed 16 MiB device array the library owns (every GPU that loads the library
 * holds it until exit). For callers that must not allocate device memory where they call it. No counterpart in the
 * reference. Limit: 2 (nq + kp) N <= 2^21 words, else -1 with a message. The first call on each device looks the
 * array's address up (make it before any stream capture) and keeps it for the life of the process (a cudaDeviceReset
 * invalidates it: reload the library after one); the device current at the call must be the context's, else -1
 * with a message. Calls share the array, so calls that overlap on the GPU (other streams, other threads) race —
 * issue them in one stream order. */
int pcb_rescale_static(PcbCtx* ctx, uint64_t* ct, int32_t top, cudaStream_t stream);
/* out = rot(x, step), left by step slots (crates/pc-gpu/src/rotate.rs:147-204); out must not alias x */
int pcb_rotate(PcbCtx* ctx, const uint64_t* x, int64_t step, uint64_t* out, int32_t top, int32_t K,
               cudaStream_t stream);
/* outs[i] = rot(x, steps[i]) for nsteps steps sharing one ModUp of x (crates/pc-gpu/src/rotate.rs:456,
 * crates/pc-py/src/fhe.rs:1156 rotate_hoisted): word for word the plain rotations. outs: host array of device
 * pointers, none aliasing x. */
int pcb_rotate_hoisted(PcbCtx* ctx, const uint64_t* x, const int64_t* steps, int32_t nsteps, uint64_t* const* outs,
                       int32_t top, int32_t K, cudaStream_t stream);
/* out = x + rot(x, g) ladder over gaps start, 2 start, .. < stop (crates/pc-gpu/src/rotate.rs:924-992) */
int pcb_rotate_and_sum(PcbCtx* ctx, const uint64_t* x, int64_t start, int64_t stop, uint64_t* out, int32_t top,
                       int32_t K, cudaStream_t stream);
/* out = x + sum_k rot(x, steps[k]), the rotations summed in the extended basis with one ModDown (crates/pc-gpu/src/
 * rotate.rs:690-775 rotate_sum); out may be x; steps of Galois element 1 are refused. */
int pcb_rotate_sum(PcbCtx* ctx, const uint64_t* x, const int64_t* steps, int32_t nsteps, uint64_t* out, int32_t top,
                   int32_t K, cudaStream_t stream);
/* rotate_and_sum with radix groups (crates/pc-gpu/src/rotate.rs:924-992, radix_bits >= 2): groups of gaps whose
 * steps all have keys run as one pcb_rotate_sum, the rest rung by rung; radix_bits < 2 is pcb_rotate_and_sum. */
int pcb_rotate_and_sum_radix(PcbCtx* ctx, const uint64_t* x, int64_t start, int64_t stop, int32_t radix_bits,
                             uint64_t* out, int32_t top, int32_t K, cudaStream_t stream);
/* out = x * pt (pt: device evaluation rows [nq][N] from pcb_pt_load); out = x + pt on part 0 */
int pcb_mult_pt(PcbCtx* ctx, const uint64_t* x, const uint64_t* pt, uint64_t* out, int32_t top, int32_t K,
                cudaStream_t stream);
int pcb_add_pt(PcbCtx* ctx, const uint64_t* x, const uint64_t* pt, uint64_t* out, int32_t top, int32_t K,
               cudaStream_t stream);
/* out = y + x * pt (sub 0), y - x * pt (1), x * pt - y (2) in one pass: the reference's mult_pt_add
 * (crates/pc-gpu/src/ops.rs:968-1005, one mul_add launch). out may alias x or y. */
int pcb_mult_pt_add(PcbCtx* ctx, const uint64_t* x, const uint64_t* pt, const uint64_t* y, uint64_t* out, int32_t sub,
                    int32_t top, int32_t K, cudaStream_t stream);
/* out = sum_{j < n} xs[j] * pts[j] (n in [1, 8]; xs: host array of device ciphertext batches, pts: host array of
 * device plaintexts as pcb_mult_pt's) in one pass, the table's mul_add_n: e.g. every term of a polynomial multiplied
 * by its coefficient and summed, one read of each operand and one write. out may alias one of xs. No counterpart in
 * the reference's Fhe API (its evaluator chains mult_pt_add). */
int pcb_mult_pt_sum(PcbCtx* ctx, const uint64_t* const* xs, const uint64_t* const* pts, int32_t n, uint64_t* out,
                    int32_t top, int32_t K, cudaStream_t stream);
/* The BSGS plaintext-matrix product of K ciphertexts (the LT stage of crates/pc-gpu/src/bts/cts.rs; apply_linear of
 * python/perseus/impl/linear.py):
 *   out = sum_{j < gstep} rot(sum_{b < bstep} rot(x, b stride) * pts[bstep j + b], bstep j stride),
 * gstep = ceil(npts / bstep). pts: a DEVICE array of npts device plaintexts ([nq][N] evaluation rows, pcb_pt_load),
 * diagonal d pre-rotated by -bstep j stride. Needs rotation keys for b stride (b < bstep) and bstep j stride (j >= 1,
 * none the identity). work: (bstep + gstep) K ciphertexts of device scratch ([2][nq + kp][N] each) that neither x nor
 * out may overlap. The result's scale is x's times the plaintexts'; out may be x. */
int pcb_linear_transform(PcbCtx* ctx, const uint64_t* x, const uint64_t* const* pts, int32_t npts, int32_t bstep,
                         int64_t stride, uint64_t* work, uint64_t* out, int32_t top, int32_t K, cudaStream_t stream);
/* nw weights over the same input (linear_multi of python/perseus/impl/linear.py: Q, K, V of one activation): the
 * babies computed once; weight w's plaintexts at pts[w npts .. w npts + npts - 1]; out holds nw K ciphertexts,
 * weight w's results at out + w K (ciphertexts), and the giant rotations run over that one batch (nw K <= k_max).
 * work: (bstep K + gstep nw K) ciphertexts. x is not read after the babies, so out may hold x. */
int pcb_linear_transform_multi(PcbCtx* ctx, const uint64_t* x, const uint64_t* const* pts, int32_t nw, int32_t npts,
                               int32_t bstep, int64_t stride, uint64_t* work, uint64_t* out, int32_t top, int32_t K,
                               cudaStream_t stream);
/* pcb_linear_transform_multi with the babies kept in the extended basis (double hoisting: the sums of the reference's
 * fused CoeffToSlot stage, crates/pc-gpu/src/bts/cts.rs and the cts_fused launcher): babies as key inner products
 * with P c0 added and no ModDown, baby 0 = P x; the baby sums over the Q rows and the special rows (plaintexts of
 * top + 1 + kp rows, pcb_pt_load_ext); each giant step's sum brought down, rotated, and the extended outputs summed
 * with giant step 0's for one ModDown. Fewer ModDowns than pcb_linear_transform_multi (gstep against bstep - 1), so
 * it pays with many baby steps. Same arguments and workspace; the words differ from pcb_linear_transform_multi's
 * (the ModDowns round at other points), the decrypted values agree within the key-switch noise. baby_offset: baby b
 * is x rotated by (b + baby_offset) stride, i.e. the product of rot(x, baby_offset stride) with that rotation folded
 * into the hoisted babies (keys for those steps); 0 is the plain product. */
int pcb_linear_transform_ext(PcbCtx* ctx, const uint64_t* x, const uint64_t* const* pts, int32_t nw, int32_t npts,
                             int32_t bstep, int64_t stride, int64_t baby_offset, uint64_t* work, uint64_t* out,
                             int32_t top, int32_t K, cudaStream_t stream);

/* ModRaise of K ciphertexts for bootstrapping (crates/pc-gpu/src/bts/raise.rs): rows 0 of both parts (evaluation
 * form, level 0) become rows 0..top_out: every residue the centred lift of the level-0 residue (the mod_raise entry
 * with d = 1), back in evaluation form. In place; the ciphertext then decrypts to m + q_0 I with small integer I. */
int pcb_mod_raise(PcbCtx* ctx, uint64_t* ct, int32_t top_out, int32_t K, cudaStream_t stream);

/* ================================================================ 3. wire format (crates/pc-client/src/wire.rs) */

/* The compressed ciphertext frame's payload (wire.rs CtHeader::bits, pack_coeffs + pack_bits per part, as
 * crates/pc-py/src/client.rs:596-612 export_ct(bits=) writes it): rows 0..=top (1 or 2 limbs) of both parts of ct
 * (device, evaluation form) to coefficient form, each coefficient's CRT x in [0, Q) as round(x 2^bits / Q) mod
 * 2^bits, packed LSB first: out (device) = part 0's N bits / 32 words, then part 1's. bits 1..64 with the primes'
 * bits + bits <= 127. The rounding is exact (the reference's exact path; its f64 shortcut serves only two primes with
 * Q < 2^63, which these chains never have). */
int pcb_ct_compress(PcbCtx* ctx, const uint64_t* ct, int32_t top, int32_t bits, uint32_t* out, cudaStream_t stream);

/* wire.rs:12-25 sum64: FNV-1a over little-endian u64 words (a trailing odd u32 word widened). */
uint64_t pcb_wire_sum64(const uint32_t* words, size_t n);
/* wire.rs packed_words: ceil(n bits / 32). */
size_t pcb_wire_packed_words(size_t n, int32_t bits);
/* wire.rs:124-128 packed_row_words: n bits / 32 + 1 (a zero guard word), padded to a multiple of 4. */
size_t pcb_wire_packed_row_words(size_t n, int32_t bits);
/* wire.rs pack_bits / unpack_bits: n values of `bits` (1..64) bits LSB first (values masked to `bits`); unpack reads
 * at most in_words words. 0, or -1 on a bad argument. */
int pcb_wire_pack_bits(const uint64_t* v, size_t n, int32_t bits, uint32_t* out);
int pcb_wire_unpack_bits(const uint32_t* in, size_t in_words, size_t n, int32_t bits, uint64_t* out);
/* wire.rs:137-150 pack_row, widened to values of up to 64 bits: the values packed, the rest of out (out_words >=
 * pcb_wire_packed_row_words) zero. pcb_wire_unpack_bits reads a row back (wire.rs unpack_row). */
int pcb_wire_pack_row(const uint64_t* v, size_t n, int32_t bits, uint32_t* out, size_t out_words);
/* wire.rs:42-74 frame header: magic (4 bytes), version 1 (u32 LE), JSON length (u64 LE), the JSON. write returns the
 * bytes written (16 + len) or -1; read returns the JSON's offset (16) and its length, or -1 (short), -2 (magic),
 * -3 (version), -4 (length above 1 GiB or past the buffer). */
int64_t pcb_wire_write_header(const char* magic, const uint8_t* json, uint64_t len, uint8_t* out, uint64_t cap);
int64_t pcb_wire_read_header(const uint8_t* buf, uint64_t n, const char* magic, uint64_t* json_len);
/* wire.rs:405-410 unpack_coeffs (the client's side of a compressed frame): rows[r][i] = round(y_i Q / 2^bits) mod
 * q[r] for nq = 1..2 primes below 2^63. 0, or -1 on a bad argument. */
int pcb_wire_unpack_coeffs(const uint64_t* q, int32_t nq, const uint64_t* y, size_t n, int32_t bits, uint64_t* rows);

/* The hybrid key switch of one polynomial per ciphertext (the north star's fused KeySwitcher): ext = dot(ModUp(d))
 * against key `kidx` with c0 mode (0 none, 1 P c0 on Q rows) and output permutation autok, then ModDown into out.
 * d, c0: rows 0..=top of K polynomials `in_stride` words apart; out: K ciphertexts. */
int pcb_keyswitch(PcbCtx* ctx, const uint64_t* d, const uint64_t* c0, int32_t c0_mode, int32_t kidx, uint32_t autok,
                  uint64_t* out, int32_t top, int32_t K, uint64_t in_stride, cudaStream_t stream);

/* Batched NTT over nrows rows of `x` ([nrows][N]) cycling over the Q primes (row i: prime i mod nq). */
int pcb_ntt_batch(PcbCtx* ctx, uint64_t* x, int32_t nrows, int32_t inverse, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#ifdef __cplusplus
static_assert(sizeof(PcbPrimeConst) == 64, "PrimeConst layout");
static_assert(sizeof(PcbRowSet) == 16, "RowSet layout");
static_assert(sizeof(PcbPolyRef) == 24, "PolyRef layout");
static_assert(sizeof(PcbNttArgs) == 176, "NttArgs layout");
static_assert(sizeof(PcbBconvJob) == 32, "BconvJob layout");
static_assert(sizeof(PcbBconvArgs) == 56, "BconvArgs layout");
static_assert(sizeof(PcbEwArgs) == 128, "EwArgs layout");
static_assert(sizeof(PcbKsArgs) == 176, "KsArgs layout");
static_assert(sizeof(PcbEpiArgs) == 72, "EpiArgs layout");
static_assert(sizeof(PcbKeyTab) == 40, "KeyTab layout");
static_assert(sizeof(PcbKsRegenArgs) == 312, "KsRegenArgs layout");
static_assert(sizeof(PcbKsKeyArgs) == 216, "KsKeyArgs layout");
static_assert(sizeof(PcbKskExpandArgs) == 48, "KskExpandArgs layout");
static_assert(sizeof(PcbTensorArgs) == 192, "TensorArgs layout");
static_assert(sizeof(PcbTensorYArgs) == 240, "TensorYArgs layout");
static_assert(sizeof(PcbCtsArgs) == 200, "CtsArgs layout");
static_assert(sizeof(PcbPackSplitArgs) == 64, "PackSplitArgs layout");
static_assert(sizeof(PcbCoeffArgs) == 80 + 16 * PCB_COEFF_MAXT, "CoeffArgs layout");
static_assert(sizeof(PcbPackDotArgs) == 120, "PackDotArgs layout");
static_assert(sizeof(PcbCtsRegenArgs) == 240, "CtsRegenArgs layout");
static_assert(sizeof(PcbSmallInt1Args) == 56, "SmallInt1Args layout");
static_assert(sizeof(PcbMdEpiArgs) == 120, "MdEpiArgs layout");
static_assert(sizeof(PcbRescaleArgs) == 152, "RescaleArgs layout");
static_assert(sizeof(PcbRescaleCombineArgs) == 80, "RescaleCombineArgs layout");
static_assert(sizeof(PcbAutomorphArgs) == 112, "AutomorphArgs layout");
static_assert(sizeof(PcbEncryptArgs) == 64, "EncryptArgs layout");
static_assert(sizeof(PcbKskGenArgs) == 120, "KskGenArgs layout");
static_assert(sizeof(PcbKskUnpackArgs) == 32, "KskUnpackArgs layout");
static_assert(sizeof(PcbEwManyArgs) == 4 * PCB_EWM_MAX * 8 + 16, "EwManyArgs layout");
static_assert(sizeof(PcbSubMulManyArgs) == 3 * PCB_EWM_MAX * 8 + 24, "SubMulManyArgs layout");
static_assert(sizeof(PcbTensorSumArgs) == 2 * 24 + 2 * PCB_TSUM_MAX * 24 + 8 + 16, "TensorSumArgs layout");
static_assert(sizeof(PcbTensorMultiArgs) == (2 * PCB_TMULTI_OUT + 2 * PCB_TMULTI_OUT * PCB_TMULTI_PAIRS) * 24 + 8 + 24,
              "TensorMultiArgs layout");
static_assert(sizeof(PcbMdEpiToArgs) == 152, "MdEpiToArgs layout");
static_assert(sizeof(PcbWsumArgs) == 256, "WsumArgs layout");
static_assert(sizeof(PcbWsumKArgs) == 264, "WsumKArgs layout");
static_assert(sizeof(PcbWsumMultiArgs) == 376, "WsumMultiArgs layout");
static_assert(sizeof(PcbRescaleNttArgs) == 328, "RescaleNttArgs layout");
static_assert(sizeof(PcbRescaleCombineToArgs) == 104, "RescaleCombineToArgs layout");
static_assert(sizeof(PcbModRaiseArgs) == 2136, "ModRaiseArgs layout");
static_assert(sizeof(PcbPtDotArgs) == 128, "PtDotArgs layout");
static_assert(sizeof(PcbAddConstArgs) == 48, "AddConstArgs layout");
static_assert(sizeof(PcbMulTableArgs) == 72, "MulTableArgs layout");
static_assert(sizeof(PcbMulAddArgs) == 104, "MulAddArgs layout");
static_assert(sizeof(PcbMulAddNArgs) == 328, "MulAddNArgs layout");
static_assert(sizeof(PcbKernelTable) == 16 + 52 * 8, "KernelTable layout");
static_assert(sizeof(PcbRingTable) == 16 + 9 * 8, "RingTable layout");
#endif

#endif /* PCB200_H */
