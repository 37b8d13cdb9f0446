/*
 * TEST INFRASTRUCTURE ONLY — the parity oracle of perseus-b200.
 *
 * A plain C++ CPU restatement of the u64 CKKS hot path of gladia-research-group/perseus (the CPU kernel twin
 * `crates/pc-host`, the math crate `crates/pc-core` and the key-switching orchestration of `crates/pc-gpu`). Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this library; the product never does.
 *
 * Parity pins: the frozen KSKB expander vectors (crates/pc-core/tests/kskb_frozen.rs:47-51), the number-theory
 * known answers (crates/pc-core/src/params/nbtheory.rs:170-180), the u64 Barrett cases
 * (crates/pc-host/src/arith.rs:197-214), the DRBG block identity (crates/pc-core/src/keys.rs:770-776) and the
 * selftest host formulas (crates/pc-kernels/src/bin/selftest/host.rs). See tests/test_oracle_pins.py.
 *
 * Words are uint64_t residues, canonical in [0, p). Rows hold N = 2^logn words. Ciphertexts are [2][rows][N]
 * (part 0 = c0, part 1 = c1), evaluation (bit-reversed NTT) form, row r = prime id r.
 */
#pragma once
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- arithmetic and number theory */
void orc_prime_const(uint64_t p, uint64_t out[8]);          /* the 64-byte PrimeConst of the u64 word */
uint64_t orc_reduce128(uint64_t lo, uint64_t hi, uint64_t p); /* device double-word Barrett, exact */
uint64_t orc_mulmod(uint64_t a, uint64_t b, uint64_t p);
uint64_t orc_powmod(uint64_t a, uint64_t e, uint64_t p);
uint64_t orc_invmod(uint64_t a, uint64_t m);
int orc_is_prime(uint64_t n);
uint64_t orc_first_prime(uint32_t bits, uint64_t m);
uint64_t orc_previous_prime(uint64_t q, uint64_t m);
uint64_t orc_root_of_unity(uint64_t m, uint64_t p);
/* `count` primes p = 1 mod 2^(logn+1) just below 2^bits, largest first, skipping `skip` of them */
void orc_ntt_primes(uint32_t bits, uint32_t logn, uint32_t skip, uint32_t count, uint64_t* out);
uint32_t orc_automorph_slot(uint32_t k, uint32_t slot, uint32_t logn);
uint64_t orc_rotation_galois(int64_t r, uint32_t logn);
uint64_t orc_galois_inverse(uint64_t g, uint32_t logn);

/* ---------------------------------------------------------------- ChaCha, DRBG, samplers, expanders */
void orc_chacha_block(const uint32_t key[8], uint32_t w12, uint32_t w13, uint32_t w14, uint32_t w15,
                      uint32_t rounds, uint32_t out[16]);
/* The frozen u64 expander lane (KSKB; ENCB for tag ENCA): one row of n = 2^logn slots. */
void orc_expand_row_u64(const uint32_t seed[8], uint32_t w13, uint64_t p, uint32_t tag, uint32_t logn,
                        uint64_t* out);
void* orc_prng_new(const uint32_t key[8], uint32_t stream);
void orc_prng_free(void* g);
uint32_t orc_prng_u32(void* g);
uint64_t orc_prng_u64(void* g);
uint64_t orc_prng_below(void* g, uint64_t q);
double orc_prng_f64(void* g);
int orc_sample_sparse_ternary(void* g, uint32_t n, uint32_t h, int8_t* out);
void orc_sample_ternary(void* g, uint32_t n, int8_t* out);
void orc_sample_gaussian(void* g, double sigma, uint32_t n, int64_t* out);

/* ---------------------------------------------------------------- NTT */
void orc_twiddles(uint64_t p, uint64_t psi, uint32_t logn, uint64_t* fw, uint64_t* fws, uint64_t* iw,
                  uint64_t* iws);
/* in place over nrows rows (row i modulo primes[i]), exact CT forward / GS inverse (N^-1 folded) */
void orc_ntt_fwd(uint64_t* x, int nrows, const uint64_t* primes, uint32_t logn);
void orc_ntt_inv(uint64_t* x, int nrows, const uint64_t* primes, uint32_t logn);

/* ---------------------------------------------------------------- CKKS context */
/* q: nq Q primes (bottom first), p: kp special primes, dnum digits; psi = minimal primitive 2N-th roots */
void* orc_ctx_new(uint32_t logn, int nq, const uint64_t* q, int kp, const uint64_t* p, int dnum);
void orc_ctx_free(void* c);
int orc_ctx_rows(void* c); /* nq + kp */
void orc_set_threads(int n);
int orc_get_threads(void);

/* Session randomness: Prng::from_seed([0x5e551013, lo32(seed), hi32(seed), 4, 5, 6, 7, 8], 0); the secret
 * (sparse ternary of Hamming weight h, or uniform ternary when h = 0), then one switching key per galois element
 * (1 = relinearization), then the encryptor seed. */
int orc_keygen(void* c, uint64_t seed, uint32_t h, double sigma, int ngal, const uint64_t* galois);
void orc_secret(void* c, int8_t* out);
/* key `idx` (keygen order): b and a, [dnum][nq + kp][N] each */
int orc_key(void* c, int idx, uint64_t* b, uint64_t* a, uint32_t seed[8]);

/* Encoding: values (re, im) interleaved, nslots <= N/2 a power of two; rows 0..=top coefficient form. */
int orc_encode(void* c, const double* vals, int nvals, int nslots, double scale, int top, uint64_t* rows);
int orc_decode(void* c, const uint64_t* row0_coef, int nslots, double scale, double* vals);
/* Secret-key encryption of encoded values at `top` into ct [2][rows][N] (rows 0..=top written). */
int orc_encrypt(void* c, const double* vals, int nvals, int nslots, double scale, int top, uint64_t* ct);
/* Decrypt rows 0..=top of ct: slots (re, im) interleaved. */
int orc_decrypt(void* c, const uint64_t* ct, int top, int nslots, double scale, double* vals);

/* ---------------------------------------------------------------- homomorphic ops (ct layout [2][rows][N]) */
int orc_add(void* c, const uint64_t* a, const uint64_t* b, uint64_t* out, int top);
int orc_sub(void* c, const uint64_t* a, const uint64_t* b, uint64_t* out, int top);
/* out = a * b relinearized (no rescale) */
int orc_mult(void* c, const uint64_t* a, const uint64_t* b, uint64_t* out, int top);
/* tensor: (c0, c1, d2) each [rows][N] */
int orc_tensor(void* c, const uint64_t* a, const uint64_t* b, uint64_t* c01, uint64_t* d2, int top);
/* rescale by q_top in place: rows 0..top-1 hold the result */
int orc_rescale(void* c, uint64_t* ct, int top);
/* ModRaise in place: row 0 (level 0) of both parts lifted (centred) to rows 0..top_out, evaluation form */
int orc_mod_raise(void* c, uint64_t* ct, int top_out);
/* rotation by `step` slots (left), key of galois element 5^step must exist */
int orc_rotate(void* c, const uint64_t* x, int64_t step, uint64_t* out, int top);
/* x + rot(x, s) ladder: gaps start, 2 start, ... < stop (rotate_and_sum, radix 1) */
int orc_rotate_and_sum(void* c, const uint64_t* x, int64_t start, int64_t stop, uint64_t* out, int top);
int orc_rotate_sum(void* c, const uint64_t* x, const int64_t* steps, int nsteps, uint64_t* out, int top);
int orc_rotate_and_sum_radix(void* c, const uint64_t* x, int64_t start, int64_t stop, int radix_bits, uint64_t* out,
                             int top);
/* out = x * pt (pt: encoded rows in coefficient form, NTT'd inside), rows 0..=top */
int orc_mult_pt_rows(void* c, const uint64_t* x, const uint64_t* pt_coef, uint64_t* out, int top);
/* out = x + pt (part 0 only) */
int orc_add_pt_rows(void* c, const uint64_t* x, const uint64_t* pt_coef, uint64_t* out, int top);

/* The three key-switching steps on one polynomial d (rows 0..=top, eval form) against key `kidx`:
 * (ks0, ks1) [2][rows][N] over Q rows 0..=top and the special rows (prime-id rows), then ModDown. */
int orc_keyswitch_ext(void* c, const uint64_t* d, const uint64_t* c0, int c0_mode, int kidx, uint32_t autok,
                      uint64_t* ext, int top);
int orc_moddown(void* c, const uint64_t* ext, uint64_t* out, int top);

/* Batched config-2 microbenchmark pieces (CPU baseline): NTT of `nrows` rows of the context's primes cycling over
 * Q ids; one rotation key switch of k ciphertexts. */
int orc_ntt_batch(void* c, uint64_t* x, int nrows, int inverse);
int orc_rotate_batch(void* c, const uint64_t* x, int k, int64_t step, uint64_t* out, int top);
/* Hoisted rotations of one ciphertext: one ModUp shared by the nsteps steps, each with its own inner product and
 * ModDown (a step of galois 1 is a copy); outs[i] [2][rows][N]. */
int orc_rotate_hoisted(void* c, const uint64_t* x, const int64_t* steps, int nsteps, uint64_t* const* outs, int top);

/* ---------------------------------------------------------------- plaintext-operand kernels (linear layers)
 * out[m][y] = x[m][y] t[y] for nx polynomials of nrows rows ([nx][nrows][N]; t [nrows][N]; row y mod primes[y]) */
int orc_mul_rows(const uint64_t* x, const uint64_t* t, uint64_t* out, const uint64_t* primes, int nrows, int logn,
                 int nx);
/* BSGS plaintext dot: rot [K][bstep][2][nrows][N] -> res [K][gstep][2][nrows][N]; pts [npts][nprow][ptw], grid row y
 * reads plaintext row prow[y] at the compact index of enc (0xFFFFFFFF: i; 0x7F0000ss: i >> ss; else i & enc) */
int orc_pt_dot(const uint64_t* rot, uint64_t* res, const uint64_t* pts, const uint64_t* primes, const int32_t* prow,
               int nrows, int logn, int K, int bstep, int gstep, int npts, int ptw, int nprow, uint32_t enc);
/* out = sum_{j < gstep} rot(sum_{b < bstep} rot(x, b stride) pts[bstep j + b], bstep j stride), gstep =
 * ceil(npts / bstep); pts [npts][nq][N] evaluation form; the giant rotations summed in the extended basis */
int orc_linear_transform(void* c, const uint64_t* x, const uint64_t* pts, int npts, int bstep, int64_t stride,
                         uint64_t* out, int top);
/* the encoding's rows over the Q primes 0..=top and then every special prime; the same product with the babies in
 * the extended basis (pts [npts][top + 1 + kp][N]): res_j over the extended rows, each brought down and rotated;
 * baby b is x rotated by (b + baby_offset) stride */
int orc_encode_ext(void* c, const double* vals, int nvals, int nslots, double scale, int top, uint64_t* rows);
int orc_linear_transform_ext(void* c, const uint64_t* x, const uint64_t* pts, int npts, int bstep, int64_t stride,
                             int64_t baby_offset, uint64_t* out, int top);

#ifdef __cplusplus
}
#endif
