// The evaluator: context, device-resident keys and the ciphertext ops of the hot path, behind the pcb_* C ABI.
//
// Restates the orchestration of the reference's device runtime (crates/pc-gpu): the per-level key-switching plans
// of ks.rs:602-677 (level_specs_with), ModUp = INTT with the digit pre factor folded in (ks.rs:954-980) -> one
// conversion launch over every live digit -> NTT of the targets (ks.rs:1037-1043), the inner product (ks.rs:1109),
// ModDown = INTT of the special rows -> conversion P -> Q -> NTT whose epilogue writes (x - conv) P^-1 (ks.rs:
// 1604-1656); relinearized products (relin.rs:84-134), rotations (rotate.rs:147-204, 924-992), the rescale
// (rescale.rs:230), encryption (encrypt.rs:93-134) and key generation (keygen.rs:184-284).
//
// All device memory comes from one caller-owned arena carved at creation (the frozen arena of
// crates/pc-cuda/src/lib.rs:9-10); the context never allocates device memory itself. Every op is stream-ordered on
// the caller's stream and batches K ciphertexts per launch.
#include <stdarg.h>
#include <stdio.h>

#include <string>
#include <vector>

#include "arith.cuh"
#include "host_math.h"
#include "kernels.h"

namespace pcb {
const PcbKernelTable* table_for(int logn);
}

using namespace pcb;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}
#define CK(call)                                                                                  \
    do {                                                                                          \
        int _rc = (int)(call);                                                                    \
        if (_rc != 0) return fail(_rc, "%s failed with %d (%s:%d)", #call, _rc, __FILE__, __LINE__); \
    } while (0)

// Bump allocator over the caller's arena; in measuring mode it only counts bytes.
struct Arena {
    char* base = nullptr;
    size_t cap = 0, used = 0;
    bool measure = true;
    template <class T>
    T* take(size_t count) {
        used = (used + 255) & ~(size_t)255;
        T* p = measure ? nullptr : (T*)(base + used);
        used += count * sizeof(T);
        return p;
    }
};

struct LevelPlan {
    int top = 0, ndig = 0, mu_rows = 0, mu_max_tgt = 0, mu_ns = 0;  // mu_ns: limbs of every live digit (< 0: mixed, -max)
    // FP64 chains with a partial top digit: the jobs are stored full digits first (mu_ns limbs each), the partial
    // digit's (mu_part_ns limbs) after all of them, and ModUp converts them in two launches of exact source counts
    int mu_part_ns = 0;
    // ModUp: INTT rows (out of place, last pass x N^-1 pre_t), conversion jobs, NTT of the targets
    uint32_t *mu_intt_roff = nullptr, *mu_intt_soff = nullptr;
    int32_t* mu_intt_rprime = nullptr;
    uint64_t *mu_intt_es = nullptr, *mu_intt_ess = nullptr;
    PcbBconvJob* mu_jobs = nullptr;
    uint64_t* mu_pool = nullptr;
    uint32_t* mu_ntt_roff = nullptr;
    int32_t* mu_ntt_rprime = nullptr;
    uint32_t* ks_rows = nullptr;
    // ModDown: INTT of the special rows (N^-1 pre_j), conversion P -> Q rows 0..top, NTT + epilogue
    uint32_t* md_intt_roff = nullptr;
    int32_t* md_intt_rprime = nullptr;
    uint64_t *md_es = nullptr, *md_ess = nullptr;
    PcbBconvJob* md_jobs = nullptr;
    uint64_t* md_pool = nullptr;
    uint32_t* md_ntt_roff = nullptr;
    int32_t* md_ntt_rprime = nullptr;
    // rescale by q_top: INTT of the top rows, correction rows, NTT + combine epilogue
    uint32_t* rs_intt_roff = nullptr;
    int32_t* rs_intt_rprime = nullptr;
    uint32_t* rs_ntt_roff = nullptr;
    int32_t* rs_ntt_rprime = nullptr;
    uint64_t *rs_A = nullptr, *rs_As = nullptr, *rs_qam = nullptr, *rs_alpha = nullptr, *rs_alphas = nullptr;
};

struct KeySlot {
    uint64_t galois = 0, autok = 1;
    uint64_t *b = nullptr, *a = nullptr;  // a null: regenerated from seed in the inner products (PCB_KEYS_REGEN)
    uint32_t* seed = nullptr;
    const void** kb = nullptr;  // device arrays of one pointer (KsArgs kb / ka)
    const void** ka = nullptr;
    uint32_t* autok_dev = nullptr;
};

}  // namespace

struct PcbCtx {
    int logn = 0;
    size_t n = 0;
    int nq = 0, kp = 0, rows = 0, dnum = 0, alpha = 0, k_max = 0, nkeys = 0;
    int device = -1;  // the device current at pcb_ctx_create: the arena, the tables and the keys live there
    std::vector<uint64_t> primes;
    const PcbKernelTable* tab = nullptr;
    bool narrow = false;  // every prime below 2^52: the 26-bit-split conversion and inner-product kernels
    bool f64 = false;     // every prime below 2^50: FP64 NTT butterflies
    bool regen = false;   // PCB_KEYS_REGEN: keys stored as b + seed, `a` regenerated in the inner products
    Arena arena;
    // device tables
    PcbPrimeConst* pr = nullptr;
    uint64_t *fw = nullptr, *fws = nullptr, *iw = nullptr, *iws = nullptr, *ninv = nullptr, *ninvs = nullptr;
    double *fpk = nullptr, *ipk = nullptr;  // f64: forward / inverse twiddle packs, pack_words() doubles per prime
    // (n / 256 + 256) {w, fl(w / p)} pairs, then n single twist factors (ntt.cu Pack)
    size_t pack_words() const { return 2 * ((n >> 8) + 256) + n; }
    int32_t* digit_of = nullptr;
    uint64_t *pmod = nullptr, *pmods = nullptr, *pinv = nullptr, *pinvs = nullptr;
    uint32_t* id_roff = nullptr;   // i
    int32_t* id_rprime = nullptr;  // i mod rows (keys, secret) — see id_rprime_q for batches
    int32_t* id_rprime_q = nullptr;
    uint32_t* key_roff = nullptr;
    int32_t* key_rprime = nullptr;
    uint32_t* mr_roff = nullptr;  // pcb_mod_raise: the rows it transforms (filled per call), [2 k_max nq]
    int32_t* mr_rprime = nullptr;
    std::vector<LevelPlan> lv;
    // workspaces
    uint64_t *coef = nullptr, *digits = nullptr, *ext = nullptr, *conv = nullptr, *dbuf = nullptr, *row = nullptr;
    int ext_groups = 1;  // extended-output batches in c.ext (keys of one grouped inner product)
    // keys and session
    std::vector<KeySlot> keys;
    int nkeys_made = 0;
    uint64_t* s_eval = nullptr;
    uint32_t* enc_seed = nullptr;
    std::vector<int8_t> secret;
    hm::Drbg* drbg = nullptr;
    hm::Gauss* gauss = nullptr;
    uint32_t nonce = 0;
    hm::Encoder* enc = nullptr;
    ~PcbCtx() {
        delete drbg;
        delete gauss;
        delete enc;
    }
    size_t ct_words() const { return 2 * (size_t)rows * n; }
    int live_digits(int top) const { return top / alpha + 1; }
    void digit_range(int d, int top, int& lo, int& hi) const {
        lo = d * alpha;
        hi = std::min(std::min((d + 1) * alpha, nq), top + 1);
    }
};

namespace {

template <class T>
int upload(T* dst, const std::vector<T>& v, cudaStream_t s) {
    if (!dst || v.empty()) return 0;
    return (int)cudaMemcpyAsync(dst, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, s);
}

uint64_t prod_mod(const std::vector<uint64_t>& ps, int skip, uint64_t t) {
    uint64_t v = 1 % t;
    for (size_t k = 0; k < ps.size(); ++k)
        if ((int)k != skip) v = hm::mulmod(v, ps[k] % t, t);
    return v;
}

// One conversion job's pool words (crates/pc-kernels/kernels/args.cuh:114-118): src rows, src primes, pre, target
// rows, target primes, M[i][t] = (B / b_i) mod t
void job_pool(const std::vector<uint64_t>& primes, const std::vector<int>& src, const std::vector<int>& tgt,
              std::vector<uint64_t>& pool) {
    std::vector<uint64_t> bp;
    for (int s : src) bp.push_back(primes[s]);
    for (int s : src) pool.push_back((uint64_t)s);
    for (int s : src) pool.push_back((uint64_t)s);
    for (size_t i = 0; i < src.size(); ++i)
        pool.push_back(hm::invmod(prod_mod(bp, (int)i, bp[i]), bp[i]));
    for (int t : tgt) pool.push_back((uint64_t)t);
    for (int t : tgt) pool.push_back((uint64_t)t);
    for (size_t i = 0; i < src.size(); ++i)
        for (int t : tgt) pool.push_back(prod_mod(bp, (int)i, primes[t]));
}

// Carve (or measure) every device buffer and fill the tables. Host tables are built only when not measuring.
int layout(PcbCtx& c, int nkeys, cudaStream_t s) {
    Arena& A = c.arena;
    const bool fill = !A.measure;
    const size_t n = c.n;
    const int rows = c.rows, nq = c.nq, kp = c.kp, km = c.k_max, L = c.logn;
    const uint32_t m = 2u << L;
    // primes and NTT tables
    c.pr = A.take<PcbPrimeConst>(rows);
    c.fw = A.take<uint64_t>((size_t)rows * n);
    c.fws = A.take<uint64_t>((size_t)rows * n);
    c.iw = A.take<uint64_t>((size_t)rows * n);
    c.iws = A.take<uint64_t>((size_t)rows * n);
    c.ninv = A.take<uint64_t>(rows);
    c.ninvs = A.take<uint64_t>(rows);
    if (c.f64) {
        c.fpk = A.take<double>((size_t)rows * c.pack_words());
        c.ipk = A.take<double>((size_t)rows * c.pack_words());
    }
    if (fill) {
        std::vector<PcbPrimeConst> pr(rows);
        std::vector<uint64_t> ni(rows), nis(rows);
        for (int r = 0; r < rows; ++r) {
            pr[r] = hm::prime_const(c.primes[r]);
            ni[r] = hm::invmod(n % c.primes[r], c.primes[r]);
            nis[r] = hm::shoup_of(ni[r], c.primes[r]);
        }
        CK(upload(c.pr, pr, s));
        CK(upload(c.ninv, ni, s));
        CK(upload(c.ninvs, nis, s));
        std::vector<uint64_t> w(n), ws(n), iw(n), iws(n), pw(n), ipw(n);
        std::vector<double> fpk(c.f64 ? c.pack_words() : 0), ipk(c.f64 ? c.pack_words() : 0);
        // a pack entry: the centred twiddle and its quotient by p, exact and correctly rounded (|w| < 2^49)
        auto centred = [](std::vector<double>& pk, size_t at, uint64_t v, uint64_t p) {
            const int64_t cv = v > p / 2 ? -(int64_t)(p - v) : (int64_t)v;
            pk[2 * at] = (double)cv;
            pk[2 * at + 1] = (double)cv / (double)p;
        };
        for (int r = 0; r < rows; ++r) {
            const uint64_t p = c.primes[r], psi = hm::min_root(m, p), ipsi = hm::invmod(psi, p);
            if (!psi) return fail(PCB_BAD_ARGS, "prime %llu has no primitive %u-th root of unity", (unsigned long long)p, m);
            pw[0] = ipw[0] = 1;
            for (size_t i = 1; i < n; ++i) {
                pw[i] = hm::mulmod(pw[i - 1], psi, p);
                ipw[i] = hm::mulmod(ipw[i - 1], ipsi, p);
            }
            for (size_t i = 0; i < n; ++i) {
                const uint32_t b = hm::bitrev((uint32_t)i, L);
                w[i] = pw[b];
                iw[i] = ipw[b];
                ws[i] = hm::shoup_of(w[i], p);
                iws[i] = hm::shoup_of(iw[i], p);
            }
            CK(cudaMemcpyAsync(c.fw + (size_t)r * n, w.data(), n * 8, cudaMemcpyHostToDevice, s));
            CK(cudaMemcpyAsync(c.fws + (size_t)r * n, ws.data(), n * 8, cudaMemcpyHostToDevice, s));
            CK(cudaMemcpyAsync(c.iw + (size_t)r * n, iw.data(), n * 8, cudaMemcpyHostToDevice, s));
            CK(cudaMemcpyAsync(c.iws + (size_t)r * n, iws.data(), n * 8, cudaMemcpyHostToDevice, s));
            if (c.f64) {
                // pack: column twiddles w[0 .. R), the 256-point twiddles of psi^(N/256) in OpenFHE order (pairs), the
                // twist gamma_b^k = psi^(k c_b) at b 256 + k with c_b = 1 - 2^(L-8) + 2 brev(b) (inverse: psi^-(k c_b)),
                // single centred doubles after the pairs.
                // Entry 0 is psi^0 = 1: {1, fl(1 / p)}, which the kernels read as 1 / p
                const size_t R = n >> 8, m2 = 2 * n;
                auto psi_pow = [&](size_t e) { e %= m2; return e < n ? pw[e] : (pw[e - n] ? p - pw[e - n] : 0); };
                for (size_t t = 0; t < R; ++t) {
                    centred(fpk, t, w[t], p);
                    centred(ipk, t, iw[t], p);
                }
                for (uint32_t t = 0; t < 256; ++t) {
                    const size_t e = (size_t)hm::bitrev(t, 8) * (n >> 8);
                    centred(fpk, R + t, psi_pow(e), p);
                    centred(ipk, R + t, psi_pow(m2 - e), p);
                }
                for (size_t b = 0; b < R; ++b) {
                    const size_t cb = (1 + m2 - (n >> 8) + 2 * (size_t)hm::bitrev((uint32_t)b, L - 8)) % m2;
                    for (size_t k = 0; k < 256; ++k) {
                        const size_t e = k * cb % m2;
                        const uint64_t fv = psi_pow(e), iv = psi_pow(m2 - e);
                        fpk[2 * (R + 256) + b * 256 + k] = (double)(fv > p / 2 ? -(int64_t)(p - fv) : (int64_t)fv);
                        ipk[2 * (R + 256) + b * 256 + k] = (double)(iv > p / 2 ? -(int64_t)(p - iv) : (int64_t)iv);
                    }
                }
                const size_t pwd = c.pack_words();
                CK(cudaMemcpyAsync(c.fpk + r * pwd, fpk.data(), pwd * 8, cudaMemcpyHostToDevice, s));
                CK(cudaMemcpyAsync(c.ipk + r * pwd, ipk.data(), pwd * 8, cudaMemcpyHostToDevice, s));
            }
            CK(cudaStreamSynchronize(s));  // the host staging vectors are reused per prime
        }
    }
    // digit map, P mod q, P^-1 mod q
    c.digit_of = A.take<int32_t>(rows);
    c.pmod = A.take<uint64_t>(rows);
    c.pmods = A.take<uint64_t>(rows);
    c.pinv = A.take<uint64_t>(rows);
    c.pinvs = A.take<uint64_t>(rows);
    std::vector<uint64_t> P(c.primes.begin() + nq, c.primes.end());
    if (fill) {
        std::vector<int32_t> dof(rows, -1);
        std::vector<uint64_t> pm(rows, 0), pms(rows, 0), pi(rows, 0), pis(rows, 0);
        for (int t = 0; t < nq; ++t) {
            const uint64_t q = c.primes[t];
            dof[t] = t / c.alpha;
            pm[t] = prod_mod(P, -1, q);
            pms[t] = hm::shoup_of(pm[t], q);
            pi[t] = hm::invmod(pm[t], q);
            pis[t] = hm::shoup_of(pi[t], q);
        }
        CK(upload(c.digit_of, dof, s));
        CK(upload(c.pmod, pm, s));
        CK(upload(c.pmods, pms, s));
        CK(upload(c.pinv, pi, s));
        CK(upload(c.pinvs, pis, s));
    }
    // identity row tables: batches up to k_max cts x 2 parts x rows
    const size_t nid = (size_t)km * 2 * rows;
    c.id_roff = A.take<uint32_t>(nid);
    c.id_rprime = A.take<int32_t>(nid);
    c.id_rprime_q = A.take<int32_t>(nid);
    c.key_roff = A.take<uint32_t>((size_t)c.dnum * rows);
    c.key_rprime = A.take<int32_t>((size_t)c.dnum * rows);
    if (fill) {
        std::vector<uint32_t> ro(nid);
        std::vector<int32_t> rp(nid), rq(nid);
        for (size_t i = 0; i < nid; ++i) {
            ro[i] = (uint32_t)i;
            rp[i] = (int32_t)(i % rows);
            rq[i] = (int32_t)(i % nq);
        }
        CK(upload(c.id_roff, ro, s));
        CK(upload(c.id_rprime, rp, s));
        CK(upload(c.id_rprime_q, rq, s));
        std::vector<uint32_t> kro((size_t)c.dnum * rows);
        std::vector<int32_t> krp((size_t)c.dnum * rows);
        for (int d = 0; d < c.dnum; ++d)
            for (int r = 0; r < rows; ++r) {
                kro[(size_t)d * rows + r] = (uint32_t)(d * rows + r);
                krp[(size_t)d * rows + r] = r;
            }
        CK(upload(c.key_roff, kro, s));
        CK(upload(c.key_rprime, krp, s));
    }
    // per-level plans (crates/pc-gpu/src/ks.rs:602-677)
    c.lv.assign(nq, LevelPlan());
    std::vector<uint64_t> preP(kp);
    for (int j = 0; j < kp; ++j) preP[j] = hm::invmod(prod_mod(P, j, P[j]), P[j]);
    for (int top = 0; top < nq; ++top) {
        LevelPlan& l = c.lv[top];
        l.top = top;
        l.ndig = c.live_digits(top);
        const int T = top + 1;
        // ModUp INTT
        l.mu_intt_roff = A.take<uint32_t>((size_t)km * T);
        l.mu_intt_soff = A.take<uint32_t>((size_t)km * T);
        l.mu_intt_rprime = A.take<int32_t>((size_t)km * T);
        l.mu_intt_es = A.take<uint64_t>((size_t)km * T);
        l.mu_intt_ess = A.take<uint64_t>((size_t)km * T);
        // targets of every live digit
        std::vector<std::vector<int>> src(l.ndig), tgt(l.ndig);
        for (int d = 0; d < l.ndig; ++d) {
            int lo, hi;
            c.digit_range(d, top, lo, hi);
            for (int t = lo; t < hi; ++t) src[d].push_back(t);
            for (int t = 0; t <= top; ++t)
                if (t < lo || t >= hi) tgt[d].push_back(t);
            for (int j = 0; j < kp; ++j) tgt[d].push_back(nq + j);
            l.mu_max_tgt = std::max(l.mu_max_tgt, (int)tgt[d].size());
        }
        // the digits' common limb count, or minus the largest when they differ (a partial top digit)
        int ns_max = 0;
        bool same = true;
        for (int d = 0; d < l.ndig; ++d) {
            ns_max = std::max(ns_max, (int)src[d].size());
            same = same && src[d].size() == src[0].size();
        }
        l.mu_ns = same ? ns_max : -ns_max;
        l.mu_part_ns = 0;
        if (!same && c.f64 && l.ndig >= 2) {
            bool full_same = true;
            for (int d = 0; d + 1 < l.ndig; ++d) full_same = full_same && src[d].size() == src[0].size();
            if (full_same && src[l.ndig - 1].size() < src[0].size()) {
                l.mu_ns = (int)src[0].size();
                l.mu_part_ns = (int)src[l.ndig - 1].size();
            }
        }
        l.mu_rows = 0;
        for (int d = 0; d < l.ndig; ++d) l.mu_rows += (int)tgt[d].size();
        std::vector<uint64_t> pool;
        std::vector<uint32_t> pool_off(l.ndig);
        for (int d = 0; d < l.ndig; ++d) {
            pool_off[d] = (uint32_t)pool.size();
            job_pool(c.primes, src[d], tgt[d], pool);
        }
        l.mu_jobs = A.take<PcbBconvJob>((size_t)km * l.ndig);
        l.mu_pool = A.take<uint64_t>(pool.size());
        l.mu_ntt_roff = A.take<uint32_t>((size_t)km * l.mu_rows);
        l.mu_ntt_rprime = A.take<int32_t>((size_t)km * l.mu_rows);
        l.ks_rows = A.take<uint32_t>(T + kp);
        // ModDown
        l.md_intt_roff = A.take<uint32_t>((size_t)km * 2 * kp);
        l.md_intt_rprime = A.take<int32_t>((size_t)km * 2 * kp);
        l.md_es = A.take<uint64_t>((size_t)km * 2 * kp);
        l.md_ess = A.take<uint64_t>((size_t)km * 2 * kp);
        std::vector<int> psrc, qtgt;
        for (int j = 0; j < kp; ++j) psrc.push_back(nq + j);
        for (int t = 0; t <= top; ++t) qtgt.push_back(t);
        std::vector<uint64_t> mdpool;
        job_pool(c.primes, psrc, qtgt, mdpool);
        l.md_jobs = A.take<PcbBconvJob>((size_t)km * 2);
        l.md_pool = A.take<uint64_t>(mdpool.size());
        l.md_ntt_roff = A.take<uint32_t>((size_t)km * 2 * T);
        l.md_ntt_rprime = A.take<int32_t>((size_t)km * 2 * T);
        // rescale
        l.rs_intt_roff = A.take<uint32_t>((size_t)km * 2);
        l.rs_intt_rprime = A.take<int32_t>((size_t)km * 2);
        l.rs_ntt_roff = A.take<uint32_t>((size_t)km * 2 * (top ? top : 1));
        l.rs_ntt_rprime = A.take<int32_t>((size_t)km * 2 * (top ? top : 1));
        l.rs_A = A.take<uint64_t>(rows);
        l.rs_As = A.take<uint64_t>(rows);
        l.rs_qam = A.take<uint64_t>(rows);
        l.rs_alpha = A.take<uint64_t>(rows);
        l.rs_alphas = A.take<uint64_t>(rows);
        if (!fill) continue;
        // ModUp tables: row (c, t) of the coefficient workspace [c][rows] reads part 1 of ct c ([c][2][rows])
        std::vector<uint32_t> ro, so;
        std::vector<int32_t> rp;
        std::vector<uint64_t> es, ess;
        std::vector<uint64_t> pre(T);
        for (int d = 0; d < l.ndig; ++d) {
            std::vector<uint64_t> bp;
            for (int t : src[d]) bp.push_back(c.primes[t]);
            for (size_t i = 0; i < src[d].size(); ++i) pre[src[d][i]] = hm::invmod(prod_mod(bp, (int)i, bp[i]), bp[i]);
        }
        for (int cc = 0; cc < km; ++cc)
            for (int t = 0; t <= top; ++t) {
                const uint64_t q = c.primes[t];
                ro.push_back((uint32_t)(cc * rows + t));
                so.push_back((uint32_t)(cc * 2 * rows + t));
                rp.push_back(t);
                const uint64_t v = hm::mulmod(hm::invmod(n % q, q), pre[t], q);
                es.push_back(v);
                ess.push_back(hm::shoup_of(v, q));
            }
        CK(upload(l.mu_intt_roff, ro, s));
        CK(upload(l.mu_intt_soff, so, s));
        CK(upload(l.mu_intt_rprime, rp, s));
        CK(upload(l.mu_intt_es, es, s));
        CK(upload(l.mu_intt_ess, ess, s));
        std::vector<PcbBconvJob> jobs, part;
        std::vector<uint32_t> nro;
        std::vector<int32_t> nrp;
        for (int cc = 0; cc < km; ++cc)
            for (int d = 0; d < l.ndig; ++d) {
                PcbBconvJob j;
                j.src_off = (uint32_t)(cc * rows);
                j.dst_off = (uint32_t)((cc * c.dnum + d) * rows);
                j.nsrc = (uint32_t)src[d].size();
                j.ntgt = (uint32_t)tgt[d].size();
                j.pool_off = pool_off[d];
                j.exact = 0;
                j.prescaled = 1;
                j.split = 0;
                (l.mu_part_ns && d == l.ndig - 1 ? part : jobs).push_back(j);
                for (int t : tgt[d]) {
                    nro.push_back(j.dst_off + (uint32_t)t);
                    nrp.push_back(t);
                }
            }
        jobs.insert(jobs.end(), part.begin(), part.end());
        CK(upload(l.mu_jobs, jobs, s));
        CK(upload(l.mu_pool, pool, s));
        CK(upload(l.mu_ntt_roff, nro, s));
        CK(upload(l.mu_ntt_rprime, nrp, s));
        std::vector<uint32_t> ksr;
        for (int t = 0; t <= top; ++t) ksr.push_back((uint32_t)t);
        for (int j = 0; j < kp; ++j) ksr.push_back((uint32_t)(nq + j));
        CK(upload(l.ks_rows, ksr, s));
        // ModDown tables over the extended ciphertext layout [c][2][rows]
        std::vector<uint32_t> mro;
        std::vector<int32_t> mrp;
        std::vector<uint64_t> mes, mess;
        for (int cc = 0; cc < km; ++cc)
            for (int part = 0; part < 2; ++part)
                for (int j = 0; j < kp; ++j) {
                    mro.push_back((uint32_t)((2 * cc + part) * rows + nq + j));
                    mrp.push_back(nq + j);
                    const uint64_t p = P[j], v = hm::mulmod(hm::invmod(n % p, p), preP[j], p);
                    mes.push_back(v);
                    mess.push_back(hm::shoup_of(v, p));
                }
        CK(upload(l.md_intt_roff, mro, s));
        CK(upload(l.md_intt_rprime, mrp, s));
        CK(upload(l.md_es, mes, s));
        CK(upload(l.md_ess, mess, s));
        std::vector<PcbBconvJob> mj;
        std::vector<uint32_t> qro;
        std::vector<int32_t> qrp;
        for (int cc = 0; cc < km; ++cc)
            for (int part = 0; part < 2; ++part) {
                PcbBconvJob j;
                j.src_off = j.dst_off = (uint32_t)((2 * cc + part) * rows);
                j.nsrc = (uint32_t)kp;
                j.ntgt = (uint32_t)T;
                j.pool_off = 0;
                j.exact = 0;
                j.prescaled = 1;
                j.split = 0;
                mj.push_back(j);
                for (int t = 0; t <= top; ++t) {
                    qro.push_back(j.dst_off + (uint32_t)t);
                    qrp.push_back(t);
                }
            }
        CK(upload(l.md_jobs, mj, s));
        CK(upload(l.md_pool, mdpool, s));
        CK(upload(l.md_ntt_roff, qro, s));
        CK(upload(l.md_ntt_rprime, qrp, s));
        // rescale tables (ndrop 1; crates/pc-kernels/kernels/args.cuh:530-552)
        std::vector<uint32_t> rro, nro2;
        std::vector<int32_t> rrp, nrp2;
        for (int cc = 0; cc < km; ++cc)
            for (int part = 0; part < 2; ++part) {
                rro.push_back((uint32_t)((2 * cc + part) * rows + top));
                rrp.push_back(top);
                for (int i = 0; i < top; ++i) {
                    nro2.push_back((uint32_t)((2 * cc + part) * rows + i));
                    nrp2.push_back(i);
                }
            }
        if (top == 0) {
            nro2.assign((size_t)km * 2, 0);
            nrp2.assign((size_t)km * 2, 0);
        }
        CK(upload(l.rs_intt_roff, rro, s));
        CK(upload(l.rs_intt_rprime, rrp, s));
        CK(upload(l.rs_ntt_roff, nro2, s));
        CK(upload(l.rs_ntt_rprime, nrp2, s));
        std::vector<uint64_t> Av(rows, 0), Asv(rows, 0), qam(rows, 0), al(rows, 0), als(rows, 0);
        const uint64_t qa = c.primes[top];
        for (int i = 0; i < top; ++i) {
            const uint64_t q = c.primes[i];
            al[i] = hm::invmod(qa % q, q);
            als[i] = hm::shoup_of(al[i], q);
            Av[i] = (q - al[i]) % q;
            Asv[i] = hm::shoup_of(Av[i], q);
            qam[i] = qa % q;
        }
        CK(upload(l.rs_A, Av, s));
        CK(upload(l.rs_As, Asv, s));
        CK(upload(l.rs_qam, qam, s));
        CK(upload(l.rs_alpha, al, s));
        CK(upload(l.rs_alphas, als, s));
        CK(cudaStreamSynchronize(s));
    }
    // workspaces: coefficients [k][rows], ModUp digits [k][dnum][rows], extended / conversion / d2 in ct layout
    c.coef = A.take<uint64_t>((size_t)km * rows * n);
    c.digits = A.take<uint64_t>((size_t)km * c.dnum * rows * n);
    // extended outputs: one batch per key of a hoisted group (FP64 chains group up to KEYS_MAX keys), else one
    c.ext_groups = c.f64 ? ks::KEYS_MAX : 1;
    c.ext = A.take<uint64_t>((size_t)c.ext_groups * km * c.ct_words());
    c.conv = A.take<uint64_t>((size_t)km * c.ct_words());
    c.dbuf = A.take<uint64_t>((size_t)km * c.ct_words());
    c.row = A.take<uint64_t>(n);
    // keys and the session secret
    c.keys.assign(nkeys, KeySlot());
    for (int k = 0; k < nkeys; ++k) {
        KeySlot& ks = c.keys[k];
        ks.b = A.take<uint64_t>((size_t)c.dnum * rows * n);
        ks.a = c.regen ? nullptr : A.take<uint64_t>((size_t)c.dnum * rows * n);
        ks.seed = A.take<uint32_t>(8);
        ks.kb = A.take<const void*>(1);
        ks.ka = A.take<const void*>(1);
        ks.autok_dev = A.take<uint32_t>(1);
        if (fill) {
            std::vector<const void*> pb{ks.b}, pa{ks.a};
            CK(upload(ks.kb, pb, s));
            CK(upload(ks.ka, pa, s));
        }
    }
    c.s_eval = A.take<uint64_t>((size_t)rows * n);
    c.enc_seed = A.take<uint32_t>(8);
    c.mr_roff = A.take<uint32_t>((size_t)2 * km * c.nq);
    c.mr_rprime = A.take<int32_t>((size_t)2 * km * c.nq);
    if (fill) CK(cudaStreamSynchronize(s));
    return 0;
}

// ------------------------------------------------------------------------------------------------ launch helpers
PcbNttArgs ntt_args(const PcbCtx& c, void* base, const uint32_t* roff, const int32_t* rprime, int nrows) {
    PcbNttArgs a;
    memset(&a, 0, sizeof a);
    a.base = base;
    a.roff = roff;
    a.rprime = rprime;
    if (c.f64) {
        a.fw = a.fws = c.fpk;
        a.iw = a.iws = c.ipk;
    } else {
        a.fw = c.fw;
        a.fws = c.fws;
        a.iw = c.iw;
        a.iws = c.iws;
    }
    a.ninv = c.ninv;
    a.ninvs = c.ninvs;
    a.pr = c.pr;
    a.nrows = nrows;
    a.snum = 1;
    a.xnum = 1;
    return a;
}

// NTT launches of the context (the tables of ntt_args: FP64 ones when every prime is below 2^50)
int ntt_fwd(const PcbCtx& c, const PcbNttArgs* a, cudaStream_t s) {
    return c.logn == 14 ? ntt::fwd_run<14>(a, c.f64, s) : ntt::fwd_run<16>(a, c.f64, s);
}
int ntt_inv(const PcbCtx& c, const PcbNttArgs* a, cudaStream_t s) {
    return c.logn == 14 ? ntt::inv_run<14>(a, c.f64, s) : ntt::inv_run<16>(a, c.f64, s);
}

PcbPolyRef ct_ref(const PcbCtx& c, const void* base) {
    PcbPolyRef r;
    r.base = (void*)base;
    r.ct_stride = c.ct_words();
    r.part_stride = (uint64_t)c.rows * c.n;
    return r;
}

int check_top(const PcbCtx& c, int top, int K) {
    if (top < 0 || top >= c.nq) return fail(PCB_BAD_ARGS, "top limb %d outside [0, %d)", top, c.nq);
    if (K < 1 || K > c.k_max) return fail(PCB_BAD_ARGS, "batch of %d ciphertexts outside [1, k_max = %d]", K, c.k_max);
    return 0;
}

// ModUp of the c1 parts of K cts (ct layout at `x`, part 1 read) into the digits workspace
int modup(PcbCtx& c, const uint64_t* c1, int top, int K, cudaStream_t s) {
    const LevelPlan& l = c.lv[top];
    const int T = top + 1;
    PcbNttArgs a = ntt_args(c, c.coef, l.mu_intt_roff, l.mu_intt_rprime, K * T);
    a.src = c1;
    a.soff = l.mu_intt_soff;
    a.es = l.mu_intt_es;
    a.ess = l.mu_intt_ess;
    CK(ntt_inv(c, &a, s));
    PcbBconvArgs b;
    memset(&b, 0, sizeof b);
    b.src = c.coef;
    b.dst = c.digits;
    b.jobs = l.mu_jobs;
    b.pool = l.mu_pool;
    b.pr = c.pr;
    b.njobs = K * l.ndig;
    b.max_tgt = l.mu_max_tgt;
    if (l.mu_part_ns) {  // the full digits, then the partial top digit, each at its exact source count
        b.njobs = K * (l.ndig - 1);
        CK(c.logn == 14 ? ks::bconv_run<14>(&b, c.narrow, c.f64, l.mu_ns, s) : ks::bconv_run<16>(&b, c.narrow, c.f64, l.mu_ns, s));
        b.jobs = l.mu_jobs + (size_t)c.k_max * (l.ndig - 1);
        b.njobs = K;
        CK(c.logn == 14 ? ks::bconv_run<14>(&b, c.narrow, c.f64, l.mu_part_ns, s)
                        : ks::bconv_run<16>(&b, c.narrow, c.f64, l.mu_part_ns, s));
    } else {
        CK(c.logn == 14 ? ks::bconv_run<14>(&b, c.narrow, c.f64, l.mu_ns, s) : ks::bconv_run<16>(&b, c.narrow, c.f64, l.mu_ns, s));
    }
    PcbNttArgs f = ntt_args(c, c.digits, l.mu_ntt_roff, l.mu_ntt_rprime, K * l.mu_rows);
    CK(ntt_fwd(c, &f, s));
    return 0;
}

// key inner product of K cts against key `ks` into c.ext: c1 / c0 in ct layout (c0 mode 1 adds P c0 on Q rows)
int dot(PcbCtx& c, const KeySlot& ks, const uint64_t* c1, const uint64_t* c0, int c0_mode, int top, int K,
        cudaStream_t s, uint64_t* dst = nullptr) {
    const LevelPlan& l = c.lv[top];
    const size_t cw = c.ct_words(), rn = (size_t)c.rows * c.n;
    if (!dst) dst = c.ext;
    // one launch for the batch: every key word is read once (the inputs never alias c.ext)
    {
        const int c0i = 0, kk = K;
        PcbKsArgs a;
        memset(&a, 0, sizeof a);
        a.c1 = c1 + c0i * cw;
        a.modup = c.digits + (size_t)c0i * c.dnum * rn;
        a.c0 = c0 ? c0 + c0i * cw : nullptr;
        a.out0 = dst + c0i * cw;
        a.out1 = dst + c0i * cw + rn;
        a.kb = ks.kb;
        a.ka = ks.a ? ks.ka : nullptr;
        a.autok = ks.autok_dev;
        a.rows = l.ks_rows;
        a.digit_of = c.digit_of;
        a.pmod = c.pmod;
        a.pmods = c.pmods;
        a.pr = c.pr;
        a.ct_stride = cw;
        a.mu_ct_stride = (uint64_t)c.dnum * rn;
        a.mu_digit_stride = rn;
        a.out_ct_stride = cw;
        a.out_rot_stride = 0;
        a.key_digit_stride = rn;
        a.K = kk;
        a.R = 1;
        a.ndig = l.ndig;
        a.c0_mode = c0_mode;
        a.nq = c.nq;
        a.nrows = top + 1 + c.kp;
        const uint32_t* seed = ks.a ? nullptr : ks.seed;
        CK(c.logn == 14 ? ks::dot_all_run<14>(&a, c.narrow, c.f64, seed, s)
                        : ks::dot_all_run<16>(&a, c.narrow, c.f64, seed, s));
    }
    return 0;
}

// Key inner products of K cts against up to KEYS_MAX keys at once (FP64 chains): key r's extended outputs go to
// the r-th batch of c.ext; the ModUp digits are read once for the whole group
int dot_group(PcbCtx& c, const KeySlot* const* keys, int n, const uint64_t* c1, const uint64_t* c0, int c0_mode,
              int top, int K, cudaStream_t s, uint64_t* dst = nullptr, uint64_t dst_stride = 0) {
    const LevelPlan& l = c.lv[top];
    const size_t cw = c.ct_words(), rn = (size_t)c.rows * c.n;
    if (!dst) {
        dst = c.ext;
        dst_stride = (uint64_t)c.k_max * cw;
    }
    PcbKsArgs a;
    memset(&a, 0, sizeof a);
    a.c1 = c1;
    a.modup = c.digits;
    a.c0 = c0;
    a.out0 = dst;
    a.out1 = dst + rn;
    a.rows = l.ks_rows;
    a.digit_of = c.digit_of;
    a.pmod = c.pmod;
    a.pmods = c.pmods;
    a.pr = c.pr;
    a.ct_stride = cw;
    a.mu_ct_stride = (uint64_t)c.dnum * rn;
    a.mu_digit_stride = rn;
    a.out_ct_stride = cw;
    a.out_rot_stride = dst_stride;
    a.key_digit_stride = rn;
    a.K = K;
    a.R = n;
    a.ndig = l.ndig;
    a.c0_mode = c0_mode;
    a.nq = c.nq;
    a.nrows = top + 1 + c.kp;
    ks::KeyGroup kg;
    memset(&kg, 0, sizeof kg);
    kg.n = n;
    for (int r = 0; r < n; ++r) {
        kg.kb[r] = keys[r]->b;
        kg.ka[r] = keys[r]->a;
        kg.seed[r] = keys[r]->a ? nullptr : keys[r]->seed;
        kg.autok[r] = (uint32_t)keys[r]->autok;
    }
    CK(c.logn == 14 ? ks::dot_keys_run<14>(&a, kg, s) : ks::dot_keys_run<16>(&a, kg, s));
    return 0;
}

// The inner products of up to SUM_KEYS_MAX keys against the same ModUp digits summed into c.ext (FP64 chains, the
// gather-form kernel): c0_mode 1 adds each key's P sigma(c0), | PCB_KS_ACC adds the batch already in c.ext
int dot_sum(PcbCtx& c, const KeySlot* const* keys, int n, const uint64_t* c1, const uint64_t* c0, int c0_mode, int top,
            int K, cudaStream_t s) {
    const LevelPlan& l = c.lv[top];
    const size_t cw = c.ct_words(), rn = (size_t)c.rows * c.n;
    PcbKsArgs a;
    memset(&a, 0, sizeof a);
    a.c1 = c1;
    a.modup = c.digits;
    a.c0 = c0;
    a.out0 = c.ext;
    a.out1 = c.ext + rn;
    a.rows = l.ks_rows;
    a.digit_of = c.digit_of;
    a.pmod = c.pmod;
    a.pmods = c.pmods;
    a.pr = c.pr;
    a.ct_stride = cw;
    a.mu_ct_stride = (uint64_t)c.dnum * rn;
    a.mu_digit_stride = rn;
    a.out_ct_stride = cw;
    a.key_digit_stride = rn;
    a.K = K;
    a.R = n;
    a.ndig = l.ndig;
    a.c0_mode = c0_mode;
    a.nq = c.nq;
    a.nrows = top + 1 + c.kp;
    ks::KeySum kg;
    memset(&kg, 0, sizeof kg);
    kg.n = n;
    for (int r = 0; r < n; ++r) {
        kg.kb[r] = keys[r]->b;
        kg.ka[r] = keys[r]->a;
        kg.seed[r] = keys[r]->a ? nullptr : keys[r]->seed;
        kg.g[r] = (uint32_t)keys[r]->galois;
    }
    CK(c.logn == 14 ? ks::dot_sum_run<14>(&a, kg, s) : ks::dot_sum_run<16>(&a, kg, s));
    return 0;
}

// ModDown of the K cts of one extended-output batch (c.ext by default) into out: epi 1 (out = (x - conv) P^-1) or
// 2 (out += ...)
// acc_src: out = acc_src + (x - conv) P^-1 (epi 2 reading acc_src, which may be out itself)
int moddown(PcbCtx& c, uint64_t* out, bool accumulate, int top, int K, cudaStream_t s, uint64_t* ext = nullptr,
            const uint64_t* acc_src = nullptr) {
    if (!ext) ext = c.ext;
    const LevelPlan& l = c.lv[top];
    PcbNttArgs a = ntt_args(c, ext, l.md_intt_roff, l.md_intt_rprime, K * 2 * c.kp);
    a.es = l.md_es;
    a.ess = l.md_ess;
    CK(ntt_inv(c, &a, s));
    PcbBconvArgs b;
    memset(&b, 0, sizeof b);
    b.src = ext;
    b.dst = c.conv;
    b.jobs = l.md_jobs;
    b.pool = l.md_pool;
    b.pr = c.pr;
    b.njobs = 2 * K;
    b.max_tgt = top + 1;
    CK(c.logn == 14 ? ks::bconv_run<14>(&b, c.narrow, c.f64, c.kp, s) : ks::bconv_run<16>(&b, c.narrow, c.f64, c.kp, s));
    PcbNttArgs f = ntt_args(c, c.conv, l.md_ntt_roff, l.md_ntt_rprime, K * 2 * (top + 1));
    f.epi = accumulate || acc_src ? 2 : 1;
    f.eout = out;
    f.ed = acc_src;
    f.ex = ext;
    f.es = c.pinv;
    f.ess = c.pinvs;
    CK(ntt_fwd(c, &f, s));
    return 0;
}

const KeySlot* key_of(const PcbCtx& c, uint64_t g) {
    for (int k = 0; k < c.nkeys_made; ++k)
        if (c.keys[k].galois == g) return &c.keys[k];
    return nullptr;
}

uint64_t rot_galois(const PcbCtx& c, int64_t step) {
    const int64_t h = (int64_t)c.n / 2;
    return hm::powmod(5, (uint64_t)(((step % h) + h) % h), 2 * c.n);
}

__global__ void dec_row0(const uint64_t* c0, const uint64_t* c1, const uint64_t* s, uint64_t* out, PcbPrimeConst pc) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    out[i] = add_mod(c0[i], mul_mod(c1[i], s[i], pc), pc.p);
}

// add_pt: part 0 += pt, part 1 copied (out may be x)
template <int LOGN>
__global__ void add_pt_k(PcbPolyRef out, PcbPolyRef x, const uint64_t* pt, const PcbPrimeConst* pr) {
    const int row = blockIdx.y, cc = blockIdx.z >> 1, part = blockIdx.z & 1;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t v = at_row(x, cc, part, row, LOGN)[i];
    at_row_w(out, cc, part, row, LOGN)[i] = part == 0 ? add_mod(v, pt[((size_t)row << LOGN) + i], pr[row].p) : v;
}

int launch_add_pt(PcbCtx& c, const uint64_t* x, const uint64_t* pt, uint64_t* out, int top, int K, cudaStream_t s) {
    const dim3 g((unsigned)(c.n / 256), top + 1, 2 * K);
    if (c.logn == 14) add_pt_k<14><<<g, 256, 0, s>>>(ct_ref(c, out), ct_ref(c, x), pt, c.pr);
    else add_pt_k<16><<<g, 256, 0, s>>>(ct_ref(c, out), ct_ref(c, x), pt, c.pr);
    return PCB_LAUNCH_RESULT();
}

// x * pt (or y +- x * pt) over Q rows 0..=top through the mul_table / mul_add launchers
int launch_mul_pt(PcbCtx& c, const uint64_t* x, const uint64_t* pt, const uint64_t* y, int sub, uint64_t* out, int top,
                  int K, cudaStream_t s) {
    PcbMulAddArgs a;
    memset(&a, 0, sizeof a);
    a.m.out = ct_ref(c, out);
    a.m.in = ct_ref(c, x);
    a.m.t = pt;
    a.m.pr = c.pr;
    a.m.n = top + 1;
    a.m.K = K;
    if (!y) return c.logn == 14 ? pt::mul_table_launch<14>(&a.m, s) : pt::mul_table_launch<16>(&a.m, s);
    a.y = ct_ref(c, y);
    a.sub = sub;
    return c.logn == 14 ? pt::mul_add_launch<14>(&a, s) : pt::mul_add_launch<16>(&a, s);
}

}  // namespace

// ================================================================================================ C API
extern "C" {

const char* pcb_last_error(void) { return g_err.c_str(); }

static int init_ctx(PcbCtx& c, const PcbParams* prm, int nkeys) {
    if (!prm) return fail(PCB_BAD_ARGS, "null params");
    if (prm->log_n != 14 && prm->log_n != 16) return fail(PCB_BAD_ARGS, "log_n %u (14 or 16)", prm->log_n);
    if (prm->nq < 1 || prm->kp < 1 || prm->dnum < 1 || prm->dnum > 16 || prm->dnum > prm->nq || !prm->q || !prm->p)
        return fail(PCB_BAD_ARGS, "nq %d, kp %d, dnum %d", prm->nq, prm->kp, prm->dnum);
    if (prm->k_max < 1 || prm->k_max > 256 || nkeys < 0) return fail(PCB_BAD_ARGS, "k_max %d, nkeys %d", prm->k_max, nkeys);
    c.logn = (int)prm->log_n;
    c.n = (size_t)1 << c.logn;
    c.nq = prm->nq;
    c.kp = prm->kp;
    c.rows = c.nq + c.kp;
    c.dnum = prm->dnum;
    c.alpha = (c.nq + c.dnum - 1) / c.dnum;
    if (c.nq <= c.alpha * (c.dnum - 1)) return fail(PCB_BAD_ARGS, "%d limbs do not split into %d digits", c.nq, c.dnum);
    if (c.alpha > 16 || c.kp > 16) return fail(PCB_BAD_ARGS, "digits of %d limbs / %d special primes (max 16)", c.alpha, c.kp);
    c.k_max = prm->k_max;
    c.nkeys = nkeys;
    if (prm->key_source != PCB_KEYS_DENSE && prm->key_source != PCB_KEYS_REGEN)
        return fail(PCB_BAD_ARGS, "key_source %d (0 dense, 1 regenerated)", prm->key_source);
    c.regen = prm->key_source == PCB_KEYS_REGEN;
    c.primes.assign(prm->q, prm->q + c.nq);
    c.primes.insert(c.primes.end(), prm->p, prm->p + c.kp);
    for (uint64_t p : c.primes)
        if (p < 3 || !(p & 1) || p >= (1ull << 61) || (p - 1) % (2 * c.n))
            return fail(PCB_BAD_ARGS, "prime %llu is not an odd NTT prime below 2^61 (p = 1 mod 2N)", (unsigned long long)p);
    c.tab = table_for(c.logn);
    c.narrow = c.f64 = true;
    for (uint64_t p : c.primes) {
        c.narrow = c.narrow && p < (1ull << 52);
        c.f64 = c.f64 && p < (1ull << 50);
    }
    return 0;
}

int64_t pcb_ctx_bytes(const PcbParams* prm, int32_t nkeys) {
    PcbCtx c;
    int rc = init_ctx(c, prm, nkeys);
    if (rc) return rc;
    c.arena.measure = true;
    rc = layout(c, nkeys, nullptr);
    if (rc) return rc;
    return (int64_t)c.arena.used + 256;
}

int pcb_ctx_create(const PcbParams* prm, int32_t nkeys, void* arena, size_t arena_bytes, cudaStream_t stream,
                   PcbCtx** out) {
    if (!out) return fail(PCB_BAD_ARGS, "null output");
    *out = nullptr;
    PcbCtx* c = new PcbCtx();
    int rc = init_ctx(*c, prm, nkeys);
    if (rc) {
        delete c;
        return rc;
    }
    const int64_t need = pcb_ctx_bytes(prm, nkeys);
    if (!arena || (int64_t)arena_bytes < need) {
        delete c;
        return fail(PCB_BAD_ARGS, "arena of %zu bytes, %lld needed", arena_bytes, (long long)need);
    }
    if (cudaGetDevice(&c->device) != cudaSuccess) {
        delete c;
        return fail(PCB_BAD_ARGS, "no current CUDA device");
    }
    c->arena.base = (char*)(((uintptr_t)arena + 255) & ~(uintptr_t)255);
    c->arena.cap = arena_bytes - (size_t)(c->arena.base - (char*)arena);
    c->arena.measure = false;
    c->enc = new hm::Encoder(c->n);
    rc = layout(*c, nkeys, stream);
    if (rc) {
        delete c;
        return rc;
    }
    *out = c;
    return 0;
}

void pcb_ctx_destroy(PcbCtx* ctx) { delete ctx; }
int pcb_ctx_rows(const PcbCtx* ctx) { return ctx ? ctx->rows : PCB_BAD_ARGS; }

int pcb_ctx_tables(const PcbCtx* c, const PcbPrimeConst** pr, const uint64_t** fw, const uint64_t** fws,
                   const uint64_t** iw, const uint64_t** iws, const uint64_t** ninv, const uint64_t** ninvs) {
    if (!c) return fail(PCB_BAD_ARGS, "null context");
    if (pr) *pr = c->pr;
    if (fw) *fw = c->fw;
    if (fws) *fws = c->fws;
    if (iw) *iw = c->iw;
    if (iws) *iws = c->iws;
    if (ninv) *ninv = c->ninv;
    if (ninvs) *ninvs = c->ninvs;
    return 0;
}

int pcb_keygen(PcbCtx* c, uint64_t seed, uint32_t h, double sigma, int32_t ngal, const uint64_t* galois,
               cudaStream_t s) {
    if (!c) return fail(PCB_BAD_ARGS, "null context");
    if (ngal < 0 || ngal > c->nkeys || (ngal && !galois))
        return fail(PCB_BAD_ARGS, "%d keys requested, the context holds %d", ngal, c->nkeys);
    if (!(sigma > 0.0 && sigma < 1e6)) return fail(PCB_BAD_ARGS, "sigma %g", sigma);
    const size_t n = c->n;
    const int rows = c->rows;
    const uint32_t key0[8] = {0x5e551013u, (uint32_t)seed, (uint32_t)(seed >> 32), 4, 5, 6, 7, 8};
    delete c->drbg;
    delete c->gauss;
    c->drbg = new hm::Drbg(key0, 0);
    c->gauss = new hm::Gauss(sigma);
    c->secret.assign(n, 0);
    if (h == 0) hm::ternary(*c->drbg, n, c->secret.data());
    else if (!hm::sparse_ternary(*c->drbg, n, h, c->secret.data()))
        return fail(PCB_BAD_ARGS, "Hamming weight %u > N", h);
    // the secret in evaluation form over every prime id
    std::vector<uint64_t> host((size_t)rows * n);
    for (int r = 0; r < rows; ++r)
        for (size_t i = 0; i < n; ++i)
            host[(size_t)r * n + i] = c->secret[i] < 0 ? c->primes[r] - 1 : (uint64_t)c->secret[i];
    CK(cudaMemcpyAsync(c->s_eval, host.data(), host.size() * 8, cudaMemcpyHostToDevice, s));
    PcbNttArgs a = ntt_args(*c, c->s_eval, c->id_roff, c->id_rprime, rows);
    CK(ntt_fwd(*c, &a, s));
    CK(cudaStreamSynchronize(s));
    c->nkeys_made = 0;
    std::vector<uint64_t> err((size_t)c->dnum * rows * n);
    for (int gi = 0; gi < ngal; ++gi) {
        KeySlot& k = c->keys[gi];
        k.galois = galois[gi] % (2 * n);
        if (!(k.galois & 1)) return fail(PCB_BAD_ARGS, "galois element %llu is even", (unsigned long long)galois[gi]);
        k.autok = hm::powmod(k.galois, (2 * n >> 2) - 1, 2 * n);
        uint32_t kseed[8], sub[8];
        c->drbg->seed8(kseed);
        c->drbg->seed8(sub);
        for (int d = 0; d < c->dnum; ++d) {
            hm::Drbg g(sub, (uint32_t)d);
            std::vector<int64_t> e(n);
            for (size_t i = 0; i < n; ++i) e[i] = c->gauss->draw(g);
            for (int r = 0; r < rows; ++r) {
                const int64_t p = (int64_t)c->primes[r];
                uint64_t* o = &err[((size_t)d * rows + r) * n];
                for (size_t i = 0; i < n; ++i) {
                    const int64_t v = e[i] % p;
                    o[i] = (uint64_t)(v < 0 ? v + p : v);
                }
            }
        }
        std::vector<uint32_t> sd(kseed, kseed + 8), ak{(uint32_t)k.autok};
        CK(upload(k.seed, sd, s));
        CK(upload(k.autok_dev, ak, s));
        CK(cudaMemcpyAsync(c->digits, err.data(), err.size() * 8, cudaMemcpyHostToDevice, s));
        PcbNttArgs e = ntt_args(*c, c->digits, c->key_roff, c->key_rprime, c->dnum * rows);
        CK(ntt_fwd(*c, &e, s));
        const uint64_t* s_new = c->s_eval;
        if (k.galois != 1) {
            // sigma_{g^-1}(s): the rotation key switches s to it (crates/pc-gpu/src/keygen.rs:235-256)
            PcbAutomorphArgs am;
            memset(&am, 0, sizeof am);
            am.out = ct_ref(*c, c->coef);
            am.in = ct_ref(*c, c->s_eval);
            am.rs.nq = rows;
            am.pr = c->pr;
            am.k = (uint32_t)k.autok;
            am.K = 1;
            am.nparts = 1;
            CK(c->tab->automorph(&am, s));
            s_new = c->coef;
        }
        PcbKskGenArgs g;
        memset(&g, 0, sizeof g);
        g.b = k.b;
        g.a = k.a;
        g.e = c->digits;
        g.s_new = s_new;
        g.s_old = c->s_eval;
        g.seed = k.seed;
        g.ids = c->id_rprime;
        g.digit_of = c->digit_of;
        g.pmod = c->pmod;
        g.pmods = c->pmods;
        g.pr = c->pr;
        g.nrows = rows;
        g.ndig = c->dnum;
        g.nq = c->nq;
        g.sq = k.galois == 1;
        CK(c->tab->ksk_gen(&g, s));
        CK(cudaStreamSynchronize(s));
        c->nkeys_made = gi + 1;
    }
    uint32_t es[8];
    c->drbg->seed8(es);
    std::vector<uint32_t> esv(es, es + 8);
    CK(upload(c->enc_seed, esv, s));
    c->nonce = 0;
    CK(cudaStreamSynchronize(s));
    return 0;
}

int pcb_key_ptrs(const PcbCtx* c, int32_t idx, const uint64_t** b, const uint64_t** a, uint64_t* galois) {
    if (!c || idx < 0 || idx >= c->nkeys_made) return fail(PCB_BAD_ARGS, "no key %d", idx);
    if (b) *b = c->keys[idx].b;
    if (a) *a = c->keys[idx].a;
    if (galois) *galois = c->keys[idx].galois;
    return 0;
}

int pcb_key_copy(const PcbCtx* c, int32_t idx, uint64_t* b_out, uint64_t* a_out, cudaStream_t s) {
    if (!c || idx < 0 || idx >= c->nkeys_made) return fail(PCB_BAD_ARGS, "no key %d", idx);
    const size_t bytes = (size_t)c->dnum * c->rows * c->n * 8;
    const KeySlot& k = c->keys[idx];
    if (b_out) CK(cudaMemcpyAsync(b_out, k.b, bytes, cudaMemcpyDeviceToDevice, s));
    if (a_out && k.a) CK(cudaMemcpyAsync(a_out, k.a, bytes, cudaMemcpyDeviceToDevice, s));
    if (a_out && !k.a) {  // a regenerated key: expand its `a` from the seed, every digit and prime id
        PcbKskExpandArgs e;
        memset(&e, 0, sizeof e);
        e.out = a_out;
        e.seed = k.seed;
        e.prime_ids = c->key_rprime;
        e.pr = c->pr;
        e.nmod = c->rows;
        e.dnum = c->dnum;
        CK(c->tab->ksk_expand(&e, s));
    }
    return 0;
}

int pcb_key_seed(const PcbCtx* c, int32_t idx, uint32_t* seed8) {
    if (!c || !seed8 || idx < 0 || idx >= c->nkeys_made) return fail(PCB_BAD_ARGS, "no key %d", idx);
    CK(cudaMemcpy(seed8, c->keys[idx].seed, 32, cudaMemcpyDeviceToHost));
    return 0;
}

int pcb_key_load(PcbCtx* c, int32_t idx, uint64_t galois, const uint64_t* b, const uint32_t* seed8, cudaStream_t s) {
    if (!c || !b || !seed8) return fail(PCB_BAD_ARGS, "null argument");
    if (idx < 0 || idx >= c->nkeys || idx > c->nkeys_made)
        return fail(PCB_BAD_ARGS, "key %d: the context holds %d, %d loaded", idx, c->nkeys, c->nkeys_made);
    const uint64_t two_n = 2 * (uint64_t)c->n;
    if (!(galois % two_n & 1)) return fail(PCB_BAD_ARGS, "galois element %llu is even", (unsigned long long)galois);
    for (int j = 0; j < c->nkeys_made; ++j)
        if (j != idx && c->keys[j].galois == galois % two_n)
            return fail(PCB_BAD_ARGS, "galois element %llu is key %d's", (unsigned long long)galois, j);
    KeySlot& k = c->keys[idx];
    k.galois = galois % two_n;
    k.autok = hm::powmod(k.galois, (two_n >> 2) - 1, two_n);
    const size_t bytes = (size_t)c->dnum * c->rows * c->n * 8;
    CK(cudaMemcpyAsync(k.b, b, bytes, cudaMemcpyDefault, s));
    std::vector<uint32_t> sd(seed8, seed8 + 8), ak{(uint32_t)k.autok};
    CK(upload(k.seed, sd, s));
    CK(upload(k.autok_dev, ak, s));
    if (k.a) {  // dense key source: `a` expanded from the seed once, here
        PcbKskExpandArgs e;
        memset(&e, 0, sizeof e);
        e.out = k.a;
        e.seed = k.seed;
        e.prime_ids = c->key_rprime;
        e.pr = c->pr;
        e.nmod = c->rows;
        e.dnum = c->dnum;
        CK(c->tab->ksk_expand(&e, s));
    }
    CK(cudaStreamSynchronize(s));  // the seed and autok staging vectors end here
    if (idx == c->nkeys_made) ++c->nkeys_made;
    return 0;
}

int pcb_ct_compress(PcbCtx* c, const uint64_t* ct, int32_t top, int32_t bits, uint32_t* out, cudaStream_t s) {
    if (!c || !ct || !out) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top, 1);
    if (rc) return rc;
    const int k = top + 1;
    int qbits = 0;
    for (int r = 0; r < k; ++r) qbits += 64 - __builtin_clzll(c->primes[r]);
    if (k > 2 || bits < 1 || bits > 64 || qbits + bits > 127)
        return fail(PCB_BAD_ARGS, "%d bits over %d limbs (%d bits of modulus; at most 127 together, 2 limbs)", bits, k,
                    qbits);
    const size_t n = c->n;
    // rows 0..top of both parts, coefficient form, in the workspace: part p row t at coef + (p k + t) N
    for (int part = 0; part < 2; ++part)
        CK(cudaMemcpyAsync(c->coef + (size_t)part * k * n, ct + (size_t)part * c->rows * n, (size_t)k * n * 8,
                           cudaMemcpyDeviceToDevice, s));
    std::vector<uint32_t> ro;
    std::vector<int32_t> rp;
    for (int part = 0; part < 2; ++part)
        for (int t = 0; t < k; ++t) {
            ro.push_back((uint32_t)(part * k + t));
            rp.push_back(t);
        }
    CK(upload(c->mr_roff, ro, s));
    CK(upload(c->mr_rprime, rp, s));
    PcbNttArgs a = ntt_args(*c, c->coef, c->mr_roff, c->mr_rprime, 2 * k);
    CK(ntt_inv(*c, &a, s));
    const uint64_t q0 = c->primes[0], q1 = k == 2 ? c->primes[1] : q0;
    const uint64_t inv01 = k == 2 ? hm::invmod(q0 % q1, q1) : 0;
    CK(pcb::wire_compress_launch(c->coef, k, n, hm::prime_const(q0), hm::prime_const(q1), inv01, bits, out, s));
    return 0;
}

int pcb_encode(PcbCtx* c, const double* vals, int32_t nvals, int32_t nslots, double scale, int32_t top,
               uint64_t* rows) {
    if (!c || !rows || (nvals && !vals)) return fail(PCB_BAD_ARGS, "null argument");
    if (nslots < 1 || (nslots & (nslots - 1)) || (size_t)nslots > c->n / 2 || nvals < 0 || nvals > nslots)
        return fail(PCB_BAD_ARGS, "%d values into %d slots", nvals, nslots);
    if (top < 0 || top >= c->nq) return fail(PCB_BAD_ARGS, "top %d", top);
    std::vector<hm::i128> co;
    if (!c->enc->encode(vals, nvals, nslots, scale, co)) return fail(-2, "scaled value exceeds 2^126");
    for (int r = 0; r <= top; ++r)
        for (size_t k = 0; k < c->n; ++k) rows[(size_t)r * c->n + k] = hm::mod_i128(co[k], c->primes[r]);
    return 0;
}

int pcb_encrypt(PcbCtx* c, const double* vals, int32_t nvals, int32_t nslots, double scale, int32_t top, uint64_t* ct,
                cudaStream_t s) {
    if (!c || !ct) return fail(PCB_BAD_ARGS, "null argument");
    if (!c->drbg) return fail(-3, "no session keys (pcb_keygen first)");
    int rc = check_top(*c, top, 1);
    if (rc) return rc;
    const size_t n = c->n;
    std::vector<uint64_t> m((size_t)(top + 1) * n);
    rc = pcb_encode(c, vals, nvals, nslots, scale, top, m.data());
    if (rc) return rc;
    std::vector<int64_t> e(n);
    for (size_t i = 0; i < n; ++i) e[i] = c->gauss->draw(*c->drbg);
    for (int r = 0; r <= top; ++r) {
        const int64_t p = (int64_t)c->primes[r];
        for (size_t i = 0; i < n; ++i) {
            const int64_t v = e[i] % p;
            const uint64_t ev = (uint64_t)(v < 0 ? v + p : v);
            uint64_t& x = m[(size_t)r * n + i];
            x = (x + ev) % (uint64_t)p;
        }
    }
    CK(cudaMemcpyAsync(ct, m.data(), m.size() * 8, cudaMemcpyHostToDevice, s));
    PcbNttArgs a = ntt_args(*c, ct, c->id_roff, c->id_rprime, top + 1);
    CK(ntt_fwd(*c, &a, s));
    PcbEncryptArgs ea;
    memset(&ea, 0, sizeof ea);
    ea.c0 = ct;
    ea.c1 = ct + (size_t)c->rows * n;
    ea.s = c->s_eval;
    ea.e = ct;
    ea.seed = c->enc_seed;
    ea.pr = c->pr;
    ea.nonce = c->nonce++;
    ea.nl = top + 1;
    CK(c->tab->encrypt(&ea, s));
    CK(cudaStreamSynchronize(s));  // the host staging rows go out of scope
    return 0;
}

int pcb_decrypt(PcbCtx* c, const uint64_t* ct, int32_t top, int32_t nslots, double scale, double* vals,
                cudaStream_t s) {
    if (!c || !ct || !vals) return fail(PCB_BAD_ARGS, "null argument");
    if (c->secret.empty()) return fail(-3, "no secret (pcb_keygen first)");
    if (nslots < 1 || (nslots & (nslots - 1)) || (size_t)nslots > c->n / 2) return fail(PCB_BAD_ARGS, "slots %d", nslots);
    int rc = check_top(*c, top, 1);
    if (rc) return rc;
    const size_t n = c->n;
    const PcbPrimeConst pc = hm::prime_const(c->primes[0]);
    dec_row0<<<(unsigned)(n / 256), 256, 0, s>>>(ct, ct + (size_t)c->rows * n, c->s_eval, c->row, pc);
    CK(PCB_LAUNCH_RESULT());
    PcbNttArgs a = ntt_args(*c, c->row, c->id_roff, c->id_rprime, 1);
    CK(ntt_inv(*c, &a, s));
    std::vector<uint64_t> m(n);
    CK(cudaMemcpyAsync(m.data(), c->row, n * 8, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    const uint64_t q0 = c->primes[0];
    std::vector<hm::i128> co(n);
    for (size_t k = 0; k < n; ++k) co[k] = m[k] > q0 / 2 ? -(hm::i128)(q0 - m[k]) : (hm::i128)m[k];
    c->enc->decode(co, nslots, scale, vals);
    return 0;
}

int pcb_pt_load(PcbCtx* c, const uint64_t* rows_host, int32_t top, uint64_t* pt, cudaStream_t s) {
    if (!c || !rows_host || !pt) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top, 1);
    if (rc) return rc;
    CK(cudaMemcpyAsync(pt, rows_host, (size_t)(top + 1) * c->n * 8, cudaMemcpyHostToDevice, s));
    PcbNttArgs a = ntt_args(*c, pt, c->id_roff, c->id_rprime, top + 1);
    CK(ntt_fwd(*c, &a, s));
    CK(cudaStreamSynchronize(s));
    return 0;
}

int pcb_encode_ext(PcbCtx* c, const double* vals, int32_t nvals, int32_t nslots, double scale, int32_t top,
                   uint64_t* rows) {
    if (!c || !rows || (nvals && !vals)) return fail(PCB_BAD_ARGS, "null argument");
    if (nslots < 1 || (nslots & (nslots - 1)) || (size_t)nslots > c->n / 2 || nvals < 0 || nvals > nslots)
        return fail(PCB_BAD_ARGS, "%d values into %d slots", nvals, nslots);
    if (top < 0 || top >= c->nq) return fail(PCB_BAD_ARGS, "top %d", top);
    std::vector<hm::i128> co;
    if (!c->enc->encode(vals, nvals, nslots, scale, co)) return fail(-2, "scaled value exceeds 2^126");
    for (int r = 0; r <= top + c->kp; ++r) {
        const uint64_t p = c->primes[r <= top ? r : c->nq + (r - top - 1)];
        for (size_t k = 0; k < c->n; ++k) rows[(size_t)r * c->n + k] = hm::mod_i128(co[k], p);
    }
    return 0;
}

int pcb_pt_load_ext(PcbCtx* c, const uint64_t* rows_host, int32_t top, uint64_t* pt, cudaStream_t s) {
    if (!c || !rows_host || !pt) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top, 1);
    if (rc) return rc;
    const int nr = top + 1 + c->kp;
    CK(cudaMemcpyAsync(pt, rows_host, (size_t)nr * c->n * 8, cudaMemcpyHostToDevice, s));
    PcbNttArgs a = ntt_args(*c, pt, c->id_roff, (const int32_t*)c->lv[top].ks_rows, nr);
    CK(ntt_fwd(*c, &a, s));
    CK(cudaStreamSynchronize(s));
    return 0;
}

static int ew_ct(PcbCtx* c, const uint64_t* a, const uint64_t* b, uint64_t* out, int top, int K, int sub,
                 cudaStream_t s) {
    if (!c || !a || !b || !out) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    PcbEwArgs e;
    memset(&e, 0, sizeof e);
    e.out = ct_ref(*c, out);
    e.a = ct_ref(*c, a);
    e.b = ct_ref(*c, b);
    e.rs.nq = top + 1;
    e.pr = c->pr;
    e.K = K;
    e.nparts = 2;
    e.sub = sub;
    CK(c->tab->ew_add(&e, s));
    return 0;
}
int pcb_add(PcbCtx* c, const uint64_t* a, const uint64_t* b, uint64_t* out, int32_t top, int32_t K, cudaStream_t s) {
    return ew_ct(c, a, b, out, top, K, 0, s);
}
int pcb_sub(PcbCtx* c, const uint64_t* a, const uint64_t* b, uint64_t* out, int32_t top, int32_t K, cudaStream_t s) {
    return ew_ct(c, a, b, out, top, K, 1, s);
}

int pcb_sum(PcbCtx* c, const uint64_t* const* ins, int32_t n, uint64_t* out, int32_t top, int32_t K, cudaStream_t s) {
    if (!c || !ins || !out) return fail(PCB_BAD_ARGS, "null argument");
    if (n < 1 || n > elem::SUM_MAX) return fail(PCB_BAD_ARGS, "%d inputs (1 .. %d)", n, elem::SUM_MAX);
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    elem::SumArgs a;
    memset(&a, 0, sizeof a);
    for (int m = 0; m < n; ++m) {
        if (!ins[m]) return fail(PCB_BAD_ARGS, "input %d is null", m);
        a.in[m] = ins[m];
    }
    a.out = out;
    a.pr = c->pr;
    a.ct_stride = c->ct_words();
    a.part_stride = (uint64_t)c->rows * c->n;
    a.n = n;
    a.nrows = top + 1;
    a.K = K;
    CK(c->logn == 14 ? elem::sum_launch<14>(&a, s) : elem::sum_launch<16>(&a, s));
    return 0;
}

int pcb_mult(PcbCtx* c, const uint64_t* a, const uint64_t* b, uint64_t* out, int32_t top, int32_t K, cudaStream_t s) {
    if (!c || !a || !b || !out) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    const KeySlot* k = key_of(*c, 1);
    if (!k) return fail(-3, "no relinearization key");
    // tensor: (c0, c1) into out, d2 into part 1 of the d2 workspace (ct layout), then out += KS(d2)
    PcbTensorArgs t;
    memset(&t, 0, sizeof t);
    t.out = ct_ref(*c, out);
    t.d2 = ct_ref(*c, c->dbuf);
    t.a0 = ct_ref(*c, a);
    t.b0 = ct_ref(*c, b);
    t.pr = c->pr;
    t.npairs = 1;
    t.n = top + 1;
    t.K = K;
    CK(c->tab->tensor(&t, s));
    const uint64_t* d2 = c->dbuf + (size_t)c->rows * c->n;
    rc = modup(*c, d2, top, K, s);
    if (rc) return rc;
    rc = dot(*c, *k, d2, nullptr, 0, top, K, s);
    if (rc) return rc;
    return moddown(*c, out, true, top, K, s);
}

int pcb_rescale(PcbCtx* c, uint64_t* ct, int32_t top, int32_t K, cudaStream_t s) {
    if (!c || !ct) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    if (top < 1) return fail(PCB_BAD_ARGS, "rescale at the bottom limb");
    const LevelPlan& l = c->lv[top];
    // INTT of the top rows (out of place into the conversion workspace)
    PcbNttArgs a = ntt_args(*c, c->conv, l.rs_intt_roff, l.rs_intt_rprime, 2 * K);
    a.src = ct;
    a.soff = l.rs_intt_roff;
    CK(ntt_inv(*c, &a, s));
    PcbRescaleArgs r;
    memset(&r, 0, sizeof r);
    r.x = ct_ref(*c, c->conv);
    r.tmp = ct_ref(*c, c->conv);
    r.A = l.rs_A;
    r.As = l.rs_As;
    r.qam = l.rs_qam;
    r.pr = c->pr;
    r.ca = r.cb = 1;
    r.top = top;
    r.nrows = top;
    r.K = K;
    r.ndrop = 1;
    CK(c->tab->rescale_coef(&r, s));
    // NTT of the correction rows; the epilogue combines x_i = alpha_i x_i + tmp_i (epi 3)
    PcbNttArgs f = ntt_args(*c, c->conv, l.rs_ntt_roff, l.rs_ntt_rprime, 2 * K * top);
    f.epi = 3;
    f.eout = ct;
    f.ex = ct;
    f.es = l.rs_alpha;
    f.ess = l.rs_alphas;
    CK(ntt_fwd(*c, &f, s));
    return 0;
}

int pcb_mod_raise(PcbCtx* c, uint64_t* ct, int32_t top_out, int32_t K, cudaStream_t s) {
    if (!c || !ct) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top_out, K);
    if (rc) return rc;
    if (top_out > 63) return fail(PCB_BAD_ARGS, "raise to %d limbs (the mod_raise entry takes 64)", top_out + 1);
    const LevelPlan& l0 = c->lv[0];
    // row 0 of both parts to coefficient form, in place
    PcbNttArgs a = ntt_args(*c, ct, l0.rs_intt_roff, l0.rs_intt_rprime, 2 * K);
    CK(ntt_inv(*c, &a, s));
    // rows 1..top_out: the centred lift of row 0 (one source row, qhatinv = qhat = 1)
    PcbModRaiseArgs m;
    memset(&m, 0, sizeof m);
    m.x = ct;
    m.pr = c->pr;
    m.ct_stride = c->ct_words();
    m.part_stride = (uint64_t)c->rows * c->n;
    m.qhatinv[0] = 1;
    for (int t = 0; t < 64; ++t) m.qhat[0][t] = 1;
    m.K = K;
    m.d = 1;
    m.r0 = 1;
    m.r1 = top_out + 1;
    m.nparts = 2;
    CK(c->tab->mod_raise(&m, s));
    // every row back to evaluation form
    std::vector<uint32_t> ro;
    std::vector<int32_t> rp;
    for (int cc = 0; cc < K; ++cc)
        for (int part = 0; part < 2; ++part)
            for (int t = 0; t <= top_out; ++t) {
                ro.push_back((uint32_t)((2 * cc + part) * c->rows + t));
                rp.push_back(t);
            }
    CK(upload(c->mr_roff, ro, s));
    CK(upload(c->mr_rprime, rp, s));
    PcbNttArgs f = ntt_args(*c, ct, c->mr_roff, c->mr_rprime, (int)ro.size());
    CK(ntt_fwd(*c, &f, s));
    return 0;
}

int pcb_keyswitch(PcbCtx* c, const uint64_t* d, const uint64_t* c0, int32_t c0_mode, int32_t kidx, uint32_t autok,
                  uint64_t* out, int32_t top, int32_t K, uint64_t in_stride, cudaStream_t s) {
    if (!c || !d || !out) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    if (in_stride != 0 && in_stride != c->ct_words())
        return fail(PCB_BAD_ARGS, "input polynomials must sit one ciphertext layout apart");
    if (kidx < 0 || kidx >= c->nkeys_made) return fail(-3, "no key %d", kidx);
    if ((c0_mode != 0 && c0_mode != 1) || (c0_mode && !c0)) return fail(PCB_BAD_ARGS, "c0 mode %d", c0_mode);
    KeySlot k = c->keys[kidx];
    if (autok != k.autok) return fail(PCB_BAD_ARGS, "autok %u differs from the key's %llu", autok, (unsigned long long)k.autok);
    rc = modup(*c, d, top, K, s);
    if (rc) return rc;
    rc = dot(*c, k, d, c0, c0_mode, top, K, s);
    if (rc) return rc;
    return moddown(*c, out, false, top, K, s);
}

int pcb_rotate(PcbCtx* c, const uint64_t* x, int64_t step, uint64_t* out, int32_t top, int32_t K, cudaStream_t s) {
    if (!c || !x || !out) return fail(PCB_BAD_ARGS, "null argument");
    if (x == out) return fail(PCB_BAD_ARGS, "rotate: out must not alias x");
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    const uint64_t g = rot_galois(*c, step);
    if (g == 1) {
        // rotation by a multiple of N/2 is the identity (crates/pc-gpu/src/rotate.rs:190-192): a copy
        PcbEwArgs e;
        memset(&e, 0, sizeof e);
        e.out = ct_ref(*c, out);
        e.a = ct_ref(*c, x);
        e.rs.nq = top + 1;
        e.K = K;
        e.nparts = 2;
        CK(c->tab->ew_copy(&e, s));
        return 0;
    }
    const KeySlot* k = key_of(*c, g);
    if (!k) return fail(-3, "no rotation key for step %lld (galois %llu)", (long long)step, (unsigned long long)g);
    const uint64_t* c1 = x + (size_t)c->rows * c->n;
    rc = modup(*c, c1, top, K, s);
    if (rc) return rc;
    rc = dot(*c, *k, c1, x, 1, top, K, s);
    if (rc) return rc;
    return moddown(*c, out, false, top, K, s);
}

// Hoisted rotations (crates/pc-gpu/src/rotate.rs:456): the ModUp of x's c1 is shared by every step, each step then
// runs its own inner product (output scattered by g^-1) and ModDown, so outs[i] is word for word pcb_rotate(x, steps[i]).
int pcb_rotate_hoisted(PcbCtx* c, const uint64_t* x, const int64_t* steps, int32_t nsteps, uint64_t* const* outs,
                       int32_t top, int32_t K, cudaStream_t s) {
    if (!c || !x || (nsteps > 0 && (!steps || !outs))) return fail(PCB_BAD_ARGS, "null argument");
    if (nsteps < 0) return fail(PCB_BAD_ARGS, "%d steps", nsteps);
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    std::vector<const KeySlot*> keys(nsteps, nullptr);
    bool any = false;
    for (int i = 0; i < nsteps; ++i) {
        if (!outs[i] || outs[i] == x) return fail(PCB_BAD_ARGS, "output %d is null or aliases the input", i);
        const uint64_t g = rot_galois(*c, steps[i]);
        if (g == 1) continue;
        keys[i] = key_of(*c, g);
        if (!keys[i])
            return fail(-3, "no rotation key for step %lld (galois %llu)", (long long)steps[i], (unsigned long long)g);
        any = true;
    }
    const uint64_t* c1 = x + (size_t)c->rows * c->n;
    if (any) {
        rc = modup(*c, c1, top, K, s);
        if (rc) return rc;
    }
    // FP64 chains of up to 4 digits at this level: the steps' inner products in groups sharing one read of the digits
    const bool grouped = c->ext_groups > 1 && c->lv[top].ndig <= 4;
    if (grouped) {
        std::vector<int> todo;
        for (int i = 0; i < nsteps; ++i)
            if (keys[i]) todo.push_back(i);
        for (size_t g0 = 0; g0 < todo.size(); g0 += c->ext_groups) {
            const int n = (int)std::min(todo.size() - g0, (size_t)c->ext_groups);
            const KeySlot* grp[ks::KEYS_MAX];
            for (int r = 0; r < n; ++r) grp[r] = keys[todo[g0 + r]];
            rc = dot_group(*c, grp, n, c1, x, 1, top, K, s);
            if (rc) return rc;
            for (int r = 0; r < n; ++r) {
                rc = moddown(*c, outs[todo[g0 + r]], false, top, K, s, c->ext + (size_t)r * c->k_max * c->ct_words());
                if (rc) return rc;
            }
        }
    }
    for (int i = 0; i < nsteps; ++i) {
        if (keys[i] && grouped) continue;
        if (!keys[i]) {
            PcbEwArgs e;
            memset(&e, 0, sizeof e);
            e.out = ct_ref(*c, outs[i]);
            e.a = ct_ref(*c, x);
            e.rs.nq = top + 1;
            e.K = K;
            e.nparts = 2;
            CK(c->tab->ew_copy(&e, s));
            continue;
        }
        rc = dot(*c, *keys[i], c1, x, 1, top, K, s);
        if (rc) return rc;
        rc = moddown(*c, outs[i], false, top, K, s);
        if (rc) return rc;
    }
    return 0;
}

int pcb_rotate_and_sum(PcbCtx* c, const uint64_t* x, int64_t start, int64_t stop, uint64_t* out, int32_t top, int32_t K,
                       cudaStream_t s) {
    if (!c || !x || !out) return fail(PCB_BAD_ARGS, "null argument");
    if (start == 0 || stop <= 0) return fail(PCB_BAD_ARGS, "start %lld must be non-zero, stop %lld positive", (long long)start, (long long)stop);
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    // out = x, then out += rot(out, sign g) for g = |start|, 2|start|, .. < stop; the rotation lands in dbuf
    if (out != x) {
        PcbEwArgs e;
        memset(&e, 0, sizeof e);
        e.out = ct_ref(*c, out);
        e.a = ct_ref(*c, x);
        e.rs.nq = top + 1;
        e.K = K;
        e.nparts = 2;
        CK(c->tab->ew_copy(&e, s));
    }
    const int64_t sign = start < 0 ? -1 : 1;
    for (int64_t g = start < 0 ? -start : start; g < stop; g *= 2) {
        rc = pcb_rotate(c, out, sign * g, c->dbuf, top, K, s);
        if (rc) return rc;
        rc = pcb_add(c, out, c->dbuf, out, top, K, s);
        if (rc) return rc;
    }
    return 0;
}

// out = x + sum_k rot(x, steps[k]) (the reference's rotate_sum, crates/pc-gpu/src/rotate.rs:690-775, the sum formed
// in the ModDown): one ModUp of x's c1, every key's inner product accumulated into one extended batch (c0 mode 1: each
// adds its own P sigma_k(c0)), one ModDown whose epilogue adds x. Steps of Galois element 1 are refused. out may be x.
int pcb_rotate_sum(PcbCtx* c, const uint64_t* x, const int64_t* steps, int32_t nsteps, uint64_t* out, int32_t top,
                   int32_t K, cudaStream_t s) {
    if (!c || !x || !out || !steps) return fail(PCB_BAD_ARGS, "null argument");
    if (nsteps < 1) return fail(PCB_BAD_ARGS, "%d steps", nsteps);
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    std::vector<const KeySlot*> keys(nsteps);
    for (int i = 0; i < nsteps; ++i) {
        const uint64_t g = rot_galois(*c, steps[i]);
        if (g == 1) return fail(PCB_BAD_ARGS, "rotate_sum: step %lld is the identity", (long long)steps[i]);
        keys[i] = key_of(*c, g);
        if (!keys[i])
            return fail(-3, "no rotation key for step %lld (galois %llu)", (long long)steps[i], (unsigned long long)g);
    }
    const uint64_t* c1 = x + (size_t)c->rows * c->n;
    rc = modup(*c, c1, top, K, s);
    if (rc) return rc;
    if (c->f64 && c->lv[top].ndig <= 4) {  // every key's products summed in registers, SUM_KEYS_MAX keys per launch
        for (int i0 = 0; i0 < nsteps; i0 += ks::SUM_KEYS_MAX) {
            const int n = std::min(nsteps - i0, ks::SUM_KEYS_MAX);
            rc = dot_sum(*c, keys.data() + i0, n, c1, x, i0 == 0 ? 1 : 1 | PCB_KS_ACC, top, K, s);
            if (rc) return rc;
        }
    } else {
        for (int i = 0; i < nsteps; ++i) {
            rc = dot(*c, *keys[i], c1, x, i == 0 ? 1 : 1 | PCB_KS_ACC, top, K, s);
            if (rc) return rc;
        }
    }
    return moddown(*c, out, false, top, K, s, nullptr, x);
}

// The rotate-and-sum ladder with radix groups (crates/pc-gpu/src/rotate.rs:924-992, radix_bits >= 2): the gaps
// |start|, 2|start|, .. below stop taken n = min(radix_bits, left) at a time; a group of n > 1 whose steps
// j g (j = 1 .. 2^n - 1) all have keys is one rotate_sum in place, the rest rung by rung. radix_bits < 2: the rungs.
int pcb_rotate_and_sum_radix(PcbCtx* c, const uint64_t* x, int64_t start, int64_t stop, int32_t radix_bits,
                             uint64_t* out, int32_t top, int32_t K, cudaStream_t s) {
    if (radix_bits < 2) return pcb_rotate_and_sum(c, x, start, stop, out, top, K, s);
    if (!c || !x || !out) return fail(PCB_BAD_ARGS, "null argument");
    if (start == 0 || stop <= 0) return fail(PCB_BAD_ARGS, "start %lld must be non-zero, stop %lld positive", (long long)start, (long long)stop);
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    if (out != x) {
        PcbEwArgs e;
        memset(&e, 0, sizeof e);
        e.out = ct_ref(*c, out);
        e.a = ct_ref(*c, x);
        e.rs.nq = top + 1;
        e.K = K;
        e.nparts = 2;
        CK(c->tab->ew_copy(&e, s));
    }
    const int64_t sign = start < 0 ? -1 : 1;
    std::vector<int64_t> gaps;
    for (int64_t g = start < 0 ? -start : start; g < stop; g *= 2) gaps.push_back(g);
    for (size_t i0 = 0; i0 < gaps.size();) {
        const size_t m = std::min((size_t)radix_bits, gaps.size() - i0);
        std::vector<int64_t> steps;
        bool keyed = m > 1;
        for (int64_t j = 1; keyed && j < ((int64_t)1 << m); ++j) {
            const uint64_t g = rot_galois(*c, sign * j * gaps[i0]);
            keyed = g != 1 && key_of(*c, g) != nullptr;
            steps.push_back(sign * j * gaps[i0]);
        }
        if (keyed) {
            rc = pcb_rotate_sum(c, out, steps.data(), (int32_t)steps.size(), out, top, K, s);
            if (rc) return rc;
            i0 += m;
            continue;
        }
        for (size_t r = 0; r < m; ++r) {
            rc = pcb_rotate(c, out, sign * gaps[i0 + r], c->dbuf, top, K, s);
            if (rc) return rc;
            rc = pcb_add(c, out, c->dbuf, out, top, K, s);
            if (rc) return rc;
        }
        i0 += m;
    }
    return 0;
}

int pcb_mult_pt(PcbCtx* c, const uint64_t* x, const uint64_t* pt, uint64_t* out, int32_t top, int32_t K,
                cudaStream_t s) {
    if (!c || !x || !pt || !out) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    CK(launch_mul_pt(*c, x, pt, nullptr, 0, out, top, K, s));
    return 0;
}

int pcb_mult_pt_add(PcbCtx* c, const uint64_t* x, const uint64_t* pt, const uint64_t* y, uint64_t* out, int32_t sub,
                    int32_t top, int32_t K, cudaStream_t s) {
    if (!c || !x || !pt || !y || !out) return fail(PCB_BAD_ARGS, "null argument");
    if (sub < 0 || sub > 2) return fail(PCB_BAD_ARGS, "sub %d outside [0, 2]", sub);
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    CK(launch_mul_pt(*c, x, pt, y, sub, out, top, K, s));
    return 0;
}

// out = sum_j xs[j] pts[j] in one pass of the table's mul_add_n (every ciphertext and plaintext read once, one write)
int pcb_mult_pt_sum(PcbCtx* c, const uint64_t* const* xs, const uint64_t* const* pts, int32_t n, uint64_t* out,
                    int32_t top, int32_t K, cudaStream_t s) {
    if (!c || !xs || !pts || !out) return fail(PCB_BAD_ARGS, "null argument");
    if (n < 1 || n > 8) return fail(PCB_BAD_ARGS, "%d terms (1..8)", n);
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    PcbMulAddNArgs a;
    memset(&a, 0, sizeof a);
    a.out = ct_ref(*c, out);
    for (int j = 0; j < n; ++j) {
        if (!xs[j] || !pts[j]) return fail(PCB_BAD_ARGS, "term %d is null", j);
        a.x[j] = ct_ref(*c, xs[j]);
        a.t[j] = pts[j];
    }
    a.pr = c->pr;
    a.n = top + 1;
    a.K = K;
    a.nterm = n;
    a.lazy = 1;
    CK(c->logn == 14 ? pt::mul_add_n_launch<14>(&a, s) : pt::mul_add_n_launch<16>(&a, s));
    return 0;
}

int pcb_add_pt(PcbCtx* c, const uint64_t* x, const uint64_t* pt, uint64_t* out, int32_t top, int32_t K,
               cudaStream_t s) {
    if (!c || !x || !pt || !out) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    CK(launch_add_pt(*c, x, pt, out, top, K, s));
    return 0;
}

// The BSGS plaintext-matrix product (the LT stage of crates/pc-gpu/src/bts/cts.rs and apply_linear of
// python/perseus/impl/linear.py, in the baby / giant split of FIDESlib's LTstep), for nw weights sharing the input
// (linear_multi of linear.py: the Q, K and V projections of one activation):
//   out[w] = sum_{j < gstep} rot(sum_{b < bstep} rot(x, b stride) pts[w npts + bstep j + b], bstep j stride)
// 1. the bstep - 1 baby rotations hoisted (one ModUp of x), x itself as baby 0, shared by every weight;
// 2. per weight, every giant step's baby sum in one pt_dot launch per 8 ciphertexts (each plaintext read once for
//    all of them), written as giant step j of batch member w: the nw weights' results of one giant step form one
//    batch of nw K ciphertexts;
// 3. the giant rotations over that batch: one ModUp and one key inner product per giant step, accumulated in the
//    extended basis, then one ModDown whose epilogue adds giant step 0 (which needs no rotation).
int pcb_linear_transform_multi(PcbCtx* c, const uint64_t* x, const uint64_t* const* pts, int32_t nw, int32_t npts,
                               int32_t bstep, int64_t stride, uint64_t* work, uint64_t* out, int32_t top, int32_t K,
                               cudaStream_t s) {
    if (!c || !x || !pts || !work || !out) return fail(PCB_BAD_ARGS, "null argument");
    if (nw < 1 || npts < 1 || bstep < 1 || bstep > 256 || stride == 0)
        return fail(PCB_BAD_ARGS, "nw %d, npts %d, bstep %d (1..256), stride %lld", nw, npts, bstep, (long long)stride);
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    const int KW = nw * K;  // the giant stage's batch
    if (KW > c->k_max) return fail(PCB_BAD_ARGS, "%d weights x %d ciphertexts exceed k_max %d", nw, K, c->k_max);
    const int gstep = (npts + bstep - 1) / bstep;
    const size_t cw = c->ct_words(), kw = (size_t)K * cw, gw = (size_t)KW * cw;
    uint64_t* baby = work;
    uint64_t* res = work + (size_t)bstep * kw;  // [gstep][nw][K]
    const uint64_t* wend = res + (size_t)gstep * gw;
    if (x >= work && x < wend) return fail(PCB_BAD_ARGS, "x inside the workspace");
    if (out + gw > work && out < wend) return fail(PCB_BAD_ARGS, "out overlaps the workspace");
    std::vector<const KeySlot*> giant(gstep, nullptr);
    for (int j = 1; j < gstep; ++j) {
        const int64_t st = (int64_t)j * bstep * stride;
        const uint64_t g = rot_galois(*c, st);
        if (g == 1) return fail(PCB_BAD_ARGS, "giant step %lld is the identity", (long long)st);
        giant[j] = key_of(*c, g);
        if (!giant[j]) return fail(-3, "no rotation key for giant step %lld (galois %llu)", (long long)st, (unsigned long long)g);
    }
    // 1. babies
    {
        PcbEwArgs e;
        memset(&e, 0, sizeof e);
        e.out = ct_ref(*c, baby);
        e.a = ct_ref(*c, x);
        e.rs.nq = top + 1;
        e.K = K;
        e.nparts = 2;
        CK(c->tab->ew_copy(&e, s));
    }
    if (bstep > 1) {
        std::vector<int64_t> steps(bstep - 1);
        std::vector<uint64_t*> bo(bstep - 1);
        for (int b = 1; b < bstep; ++b) {
            steps[b - 1] = (int64_t)b * stride;
            bo[b - 1] = baby + (size_t)b * kw;
        }
        rc = pcb_rotate_hoisted(c, x, steps.data(), bstep - 1, bo.data(), top, K, s);
        if (rc) return rc;
    }
    // 2. baby sums
    for (int w = 0; w < nw; ++w)
        for (int c0 = 0; c0 < K; c0 += 8) {
            PcbPtDotArgs a;
            memset(&a, 0, sizeof a);
            a.rot = ct_ref(*c, baby + (size_t)c0 * cw);
            a.res = ct_ref(*c, res + (size_t)w * kw + (size_t)c0 * cw);
            a.rot_stride = kw;
            a.res_stride = gw;
            a.pts = (const void* const*)(pts + (size_t)w * npts);
            a.pr = c->pr;
            a.rs.nq = top + 1;
            a.rs.qmax = top + 1;
            a.npts = npts;
            a.bstep = bstep;
            a.gstep = gstep;
            a.K = std::min(8, K - c0);
            a.ptw = (int32_t)c->n;
            a.enc = 0xFFFFFFFFu;
            CK(c->logn == 14 ? pt::pt_dot_launch<14>(&a, s) : pt::pt_dot_launch<16>(&a, s));
        }
    // 3. giant steps over the nw K batch
    if (gstep == 1) {
        PcbEwArgs e;
        memset(&e, 0, sizeof e);
        e.out = ct_ref(*c, out);
        e.a = ct_ref(*c, res);
        e.rs.nq = top + 1;
        e.K = KW;
        e.nparts = 2;
        CK(c->tab->ew_copy(&e, s));
        return 0;
    }
    for (int j = 1; j < gstep; ++j) {
        const uint64_t* rj = res + (size_t)j * gw;
        rc = modup(*c, rj + (size_t)c->rows * c->n, top, KW, s);
        if (rc) return rc;
        rc = dot(*c, *giant[j], rj + (size_t)c->rows * c->n, rj, j == 1 ? 1 : 1 | PCB_KS_ACC, top, KW, s);
        if (rc) return rc;
    }
    return moddown(*c, out, false, top, KW, s, nullptr, res);
}

int pcb_linear_transform(PcbCtx* c, const uint64_t* x, const uint64_t* const* pts, int32_t npts, int32_t bstep,
                         int64_t stride, uint64_t* work, uint64_t* out, int32_t top, int32_t K, cudaStream_t s) {
    return pcb_linear_transform_multi(c, x, pts, 1, npts, bstep, stride, work, out, top, K, s);
}

// The BSGS product with the babies kept in the extended basis (double hoisting; the sums of the reference's fused
// CoeffToSlot stage, crates/pc-gpu/src/bts/cts.rs with the cts_fused launcher, argument rules of args.cuh:325-352):
// 1. baby b = x rotated by (b + baby_offset) stride: P x on the Q rows and 0 on the special rows for the identity,
//    the others one ModUp of x, then each key's inner product with P c0 added, scattered by the automorphism, written
//    straight into its slot: no ModDown (a nonzero baby_offset folds a rotation of x before the product into them);
// 2. the baby sums res_j over the Q rows and the special rows (plaintexts with special rows: pcb_pt_load_ext);
// 3. res_j (j >= 1) brought down (ModDown) and rotated by its giant step, the extended outputs summed with res_0;
//    one ModDown. bstep - 1 ModDowns fewer than pcb_linear_transform_multi for gstep - 1 more.
int pcb_linear_transform_ext(PcbCtx* c, const uint64_t* x, const uint64_t* const* pts, int32_t nw, int32_t npts,
                             int32_t bstep, int64_t stride, int64_t baby_offset, uint64_t* work, uint64_t* out,
                             int32_t top, int32_t K, cudaStream_t s) {
    if (!c || !x || !pts || !work || !out) return fail(PCB_BAD_ARGS, "null argument");
    if (nw < 1 || npts < 1 || bstep < 1 || bstep > 256 || stride == 0)
        return fail(PCB_BAD_ARGS, "nw %d, npts %d, bstep %d (1..256), stride %lld", nw, npts, bstep, (long long)stride);
    int rc = check_top(*c, top, K);
    if (rc) return rc;
    const int KW = nw * K;
    if (KW > c->k_max) return fail(PCB_BAD_ARGS, "%d weights x %d ciphertexts exceed k_max %d", nw, K, c->k_max);
    const int gstep = (npts + bstep - 1) / bstep;
    const size_t cw = c->ct_words(), kw = (size_t)K * cw, gw = (size_t)KW * cw, rn = (size_t)c->rows * c->n;
    uint64_t* baby = work;
    uint64_t* res = work + (size_t)bstep * kw;  // [gstep][nw][K], extended
    const uint64_t* wend = res + (size_t)gstep * gw;
    if (x >= work && x < wend) return fail(PCB_BAD_ARGS, "x inside the workspace");
    if (out + gw > work && out < wend) return fail(PCB_BAD_ARGS, "out overlaps the workspace");
    std::vector<const KeySlot*> giant(gstep, nullptr), bk(bstep, nullptr);
    for (int j = 1; j < gstep; ++j) {
        const int64_t st = (int64_t)j * bstep * stride;
        const uint64_t g = rot_galois(*c, st);
        if (g == 1) return fail(PCB_BAD_ARGS, "giant step %lld is the identity", (long long)st);
        giant[j] = key_of(*c, g);
        if (!giant[j]) return fail(-3, "no rotation key for giant step %lld (galois %llu)", (long long)st, (unsigned long long)g);
    }
    // baby b is x rotated by (b + baby_offset) stride: the product of rot(x, baby_offset stride) without that rotation
    bool any = false;
    for (int b = 0; b < bstep; ++b) {
        const int64_t st = ((int64_t)b + baby_offset) * stride;
        const uint64_t g = rot_galois(*c, st);
        if (g == 1) continue;
        bk[b] = key_of(*c, g);
        if (!bk[b]) return fail(-3, "no rotation key for baby step %lld (galois %llu)", (long long)st, (unsigned long long)g);
        any = true;
    }
    PcbRowSet ext_rows;
    memset(&ext_rows, 0, sizeof ext_rows);
    ext_rows.nq = top + 1;
    ext_rows.np = c->kp;
    ext_rows.qmax = c->nq;
    // 1. babies: P x (the identity step), the others by the hoisted inner products
    for (int b = 0; b < bstep; ++b) {
        if (bk[b]) continue;
        PcbEwArgs e;
        memset(&e, 0, sizeof e);
        e.out = ct_ref(*c, baby + (size_t)b * kw);
        e.a = ct_ref(*c, x);
        e.rs = ext_rows;
        e.sc = c->pmod;
        e.scs = c->pmods;
        e.zero_p = 1;
        e.pr = c->pr;
        e.K = K;
        e.nparts = 2;
        CK(c->tab->ew_scale(&e, s));
    }
    if (any) {
        const uint64_t* c1 = x + rn;
        rc = modup(*c, c1, top, K, s);
        if (rc) return rc;
        const bool grouped = c->ext_groups > 1 && c->lv[top].ndig <= 4;
        std::vector<int> todo;
        for (int b = 0; b < bstep; ++b)
            if (bk[b]) todo.push_back(b);
        size_t g0 = 0;
        while (g0 < todo.size()) {
            // a group: consecutive baby slots (their outputs kw apart), up to ext_groups keys
            size_t n = 1;
            while (grouped && g0 + n < todo.size() && (int)n < c->ext_groups && todo[g0 + n] == todo[g0] + (int)n) ++n;
            uint64_t* dst = baby + (size_t)todo[g0] * kw;
            if (n > 1) {
                const KeySlot* grp[ks::KEYS_MAX];
                for (size_t r = 0; r < n; ++r) grp[r] = bk[todo[g0 + r]];
                rc = dot_group(*c, grp, (int)n, c1, x, 1, top, K, s, dst, kw);
            } else {
                rc = dot(*c, *bk[todo[g0]], c1, x, 1, top, K, s, dst);
            }
            if (rc) return rc;
            g0 += n;
        }
    }
    // 2. baby sums over the extended rows
    for (int w = 0; w < nw; ++w)
        for (int c0 = 0; c0 < K; c0 += 8) {
            PcbPtDotArgs a;
            memset(&a, 0, sizeof a);
            a.rot = ct_ref(*c, baby + (size_t)c0 * cw);
            a.res = ct_ref(*c, res + (size_t)w * kw + (size_t)c0 * cw);
            a.rot_stride = kw;
            a.res_stride = gw;
            a.pts = (const void* const*)(pts + (size_t)w * npts);
            a.pr = c->pr;
            a.rs = ext_rows;
            a.npts = npts;
            a.bstep = bstep;
            a.gstep = gstep;
            a.K = std::min(8, K - c0);
            a.ptw = (int32_t)c->n;
            a.pt_prow = top + 1;
            a.enc = 0xFFFFFFFFu;
            CK(c->logn == 14 ? pt::pt_dot_launch<14>(&a, s) : pt::pt_dot_launch<16>(&a, s));
        }
    if (gstep == 1) return moddown(*c, out, false, top, KW, s, res);
    // 3. giant steps over the nw K batch: res_j down, rotated, summed in c.ext with res_0, one ModDown
    for (int j = 1; j < gstep; ++j) {
        rc = moddown(*c, c->dbuf, false, top, KW, s, res + (size_t)j * gw);
        if (rc) return rc;
        rc = modup(*c, c->dbuf + rn, top, KW, s);
        if (rc) return rc;
        rc = dot(*c, *giant[j], c->dbuf + rn, c->dbuf, j == 1 ? 1 : 1 | PCB_KS_ACC, top, KW, s);
        if (rc) return rc;
    }
    {
        PcbEwArgs e;
        memset(&e, 0, sizeof e);
        e.out = ct_ref(*c, c->ext);
        e.a = ct_ref(*c, c->ext);
        e.b = ct_ref(*c, res);
        e.rs = ext_rows;
        e.pr = c->pr;
        e.K = KW;
        e.nparts = 2;
        CK(c->tab->ew_add(&e, s));
    }
    return moddown(*c, out, false, top, KW, s);
}

int pcb_ntt_batch(PcbCtx* c, uint64_t* x, int32_t nrows, int32_t inverse, cudaStream_t s) {
    if (!c || !x) return fail(PCB_BAD_ARGS, "null argument");
    if (nrows < 0 || nrows > c->k_max * 2 * c->rows)
        return fail(PCB_BAD_ARGS, "%d rows (row tables hold %d)", nrows, c->k_max * 2 * c->rows);
    PcbNttArgs a = ntt_args(*c, x, c->id_roff, c->id_rprime_q, nrows);
    CK(inverse ? ntt_inv(*c, &a, s) : ntt_fwd(*c, &a, s));
    return 0;
}

}  // extern "C"

// ================================================================================================ allocation-free rescale
// pcb_rescale_static: the rescale of one ciphertext with its working rows in a fixed device array that this library
// owns, for callers that cannot allocate device memory while they run: code that may only use memory set aside
// ahead of time (a host that has handed all of its device memory to an arena, or a caller whose allocator must
// not be entered from where it calls this). The context's arena still holds the tables; the op itself takes no
// workspace from it and allocates nothing.
#include <mutex>

namespace {

// Working rows of pcb_rescale_static: the inverse-transformed top row and the correction rows of both parts, in the
// ciphertext layout [2][nq + kp][N]. 2^21 words = 16 MiB, held on every GPU that loads the library until exit.
constexpr size_t STATIC_SCRATCH_WORDS = (size_t)1 << 21;
static __device__ __align__(256) uint64_t g_static_scratch[STATIC_SCRATCH_WORDS];

// The array's device address per device, looked up once per device with that device current (host code cannot
// use the symbol itself: on the host it names a stand-in, not device memory). The cached address belongs to the
// device's primary context as it was at the first call: after a cudaDeviceReset the library must be reloaded.
constexpr int MAX_DEVICES = 64;
std::mutex g_scratch_mu;
uint64_t* g_scratch_ptr[MAX_DEVICES] = {};

int static_scratch(const PcbCtx& c, uint64_t** out) {
    int dev = -1;
    CK(cudaGetDevice(&dev));
    // the array used is the current device's; the ciphertext and the tables are on the context's device
    if (dev != c.device)
        return fail(PCB_BAD_ARGS, "pcb_rescale_static: device %d is current, the context was created on device %d",
                    dev, c.device);
    if (dev < 0 || dev >= MAX_DEVICES) return fail(PCB_BAD_ARGS, "device %d beyond %d", dev, MAX_DEVICES);
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess)
            return fail((int)e, "cudaGetSymbolAddress of the static scratch failed on device %d: %s", dev,
                        cudaGetErrorString(e));
        g_scratch_ptr[dev] = (uint64_t*)p;
    }
    *out = g_scratch_ptr[dev];
    return 0;
}

}  // namespace

extern "C" {

int pcb_rescale_static(PcbCtx* c, uint64_t* ct, int32_t top, cudaStream_t s) {
    if (!c || !ct) return fail(PCB_BAD_ARGS, "null argument");
    int rc = check_top(*c, top, 1);
    if (rc) return rc;
    if (top < 1) return fail(PCB_BAD_ARGS, "rescale at the bottom limb");
    const size_t need = c->ct_words();
    if (need > STATIC_SCRATCH_WORDS)
        return fail(PCB_BAD_ARGS,
                    "pcb_rescale_static: a ciphertext of %d rows of N = %zu needs %zu scratch words, beyond the "
                    "maximum of %zu (2 (nq + kp) N <= 2^21); use pcb_rescale",
                    c->rows, c->n, need, STATIC_SCRATCH_WORDS);
    uint64_t* scratch = nullptr;
    rc = static_scratch(*c, &scratch);
    if (rc) return rc;
    // the same three launches as pcb_rescale with K = 1; every scratch word read is written first in this call
    const LevelPlan& l = c->lv[top];
    PcbNttArgs a = ntt_args(*c, scratch, l.rs_intt_roff, l.rs_intt_rprime, 2);
    a.src = ct;
    a.soff = l.rs_intt_roff;
    CK(ntt_inv(*c, &a, s));
    PcbRescaleArgs r;
    memset(&r, 0, sizeof r);
    r.x = ct_ref(*c, scratch);
    r.tmp = ct_ref(*c, scratch);
    r.A = l.rs_A;
    r.As = l.rs_As;
    r.qam = l.rs_qam;
    r.pr = c->pr;
    r.ca = r.cb = 1;
    r.top = top;
    r.nrows = top;
    r.K = 1;
    r.ndrop = 1;
    CK(c->tab->rescale_coef(&r, s));
    PcbNttArgs f = ntt_args(*c, scratch, l.rs_ntt_roff, l.rs_ntt_rprime, 2 * top);
    f.epi = 3;
    f.eout = ct;
    f.ex = ct;
    f.es = l.rs_alpha;
    f.ess = l.rs_alphas;
    CK(ntt_fwd(*c, &f, s));
    return 0;
}

}  // extern "C"
