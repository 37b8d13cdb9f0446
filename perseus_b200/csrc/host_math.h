// Host-side math of the evaluator: exact 64-bit modular arithmetic, prime constants, the sampler DRBG and samplers,
// and the CKKS slot encoder. Restates crates/pc-core/src/{modmul,keys,encode}.rs and
// crates/pc-core/src/params/nbtheory.rs; these run at setup (tables, keys) and at the encrypt / decrypt boundary.
#pragma once
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "../../include/pcb200.h"

namespace pcb {
namespace hm {

typedef unsigned __int128 u128;
typedef __int128 i128;

inline uint64_t mulmod(uint64_t a, uint64_t b, uint64_t p) { return (uint64_t)((u128)a * b % p); }
inline uint64_t powmod(uint64_t a, uint64_t e, uint64_t p) {
    uint64_t r = 1 % p;
    a %= p;
    for (; e; e >>= 1) {
        if (e & 1) r = mulmod(r, a, p);
        a = mulmod(a, a, p);
    }
    return r;
}
// extended Euclid (crates/pc-core/src/modmul.rs:55-75); 0 when not invertible
inline uint64_t invmod(uint64_t a, uint64_t m) {
    a %= m;
    if (!a) return 0;
    i128 r0 = a, r1 = m, s0 = 1, s1 = 0;
    while (r1) {
        const i128 q = r0 / r1, t = r0 - q * r1, u = s0 - q * s1;
        r0 = r1;
        r1 = t;
        s0 = s1;
        s1 = u;
    }
    if (r0 != 1) return 0;
    i128 v = s0 % (i128)m;
    return (uint64_t)(v < 0 ? v + m : v);
}
inline uint64_t shoup_of(uint64_t w, uint64_t p) { return (uint64_t)(((u128)w << 64) / p); }

// crates/pc-core/src/modmul.rs:371-413 at 64-bit words
inline PcbPrimeConst prime_const(uint64_t p) {
    PcbPrimeConst c;
    const u128 mu = (~(u128)0) / p;
    c.p = p;
    c.mu_lo = (uint64_t)mu;
    c.mu_hi = (uint64_t)(mu >> 64);
    c.bits = 64 - __builtin_clzll(p);
    c.neal_mu = (uint64_t)(((u128)1 << (2 * c.bits + 1)) / p);
    c.word_bits = 64;
    uint64_t inv = p;
    for (int i = 0; i < 6; ++i) inv *= 2 - p * inv;
    c.mont_pinv = 0 - inv;
    c.mont_r2 = (uint64_t)((~(u128)0 % p + 1) % p);
    c.split = 0;
    return c;
}

// the minimal primitive m-th root of unity (crates/pc-core/src/params/nbtheory.rs:105-140)
inline uint64_t min_root(uint64_t m, uint64_t p) {
    const uint64_t e = (p - 1) / m;
    uint64_t w = 0;
    for (uint64_t g = 2; g < p && !w; ++g) {
        const uint64_t c = powmod(g, e, p);
        if (powmod(c, m / 2, p) == p - 1) w = c;
    }
    if (!w) return 0;
    const uint64_t w2 = mulmod(w, w, p);
    uint64_t x = w, mn = w;
    for (uint64_t k = 1; k + 2 < m; k += 2) {
        x = mulmod(x, w2, p);
        if (x < mn && x != 1) mn = x;
    }
    return mn;
}

inline uint32_t bitrev(uint32_t x, int bits) {
    uint32_t r = 0;
    for (int i = 0; i < bits; ++i) r |= ((x >> i) & 1u) << (bits - 1 - i);
    return r;
}
inline uint32_t automorph_slot(uint32_t k, uint32_t o, int logn) {
    const uint32_t j = bitrev(o, logn);
    return bitrev((((j << 1) + 1) * k & ((2u << logn) - 1)) >> 1, logn);
}

// ------------------------------------------------------------------------------------------------ DRBG
// ChaCha20 sampler DRBG (crates/pc-core/src/keys.rs:119-207): 64-bit counter in state words 12..13, stream id in 14,
// the "DRBG" tag in 15
inline void chacha(const uint32_t k[8], uint32_t w12, uint32_t w13, uint32_t w14, uint32_t w15, int rounds,
                   uint32_t o[16]) {
    const uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, k[0], k[1], k[2], k[3],
                            k[4],        k[5],        k[6],        k[7],        w12,  w13,  w14,  w15};
    uint32_t x[16];
    memcpy(x, s, sizeof x);
    auto rl = [](uint32_t v, int r) { return (v << r) | (v >> (32 - r)); };
    auto q = [&](int a, int b, int c, int d) {
        x[a] += x[b]; x[d] = rl(x[d] ^ x[a], 16);
        x[c] += x[d]; x[b] = rl(x[b] ^ x[c], 12);
        x[a] += x[b]; x[d] = rl(x[d] ^ x[a], 8);
        x[c] += x[d]; x[b] = rl(x[b] ^ x[c], 7);
    };
    for (int r = 0; r < rounds; r += 2) {
        q(0, 4, 8, 12); q(1, 5, 9, 13); q(2, 6, 10, 14); q(3, 7, 11, 15);
        q(0, 5, 10, 15); q(1, 6, 11, 12); q(2, 7, 8, 13); q(3, 4, 9, 14);
    }
    for (int i = 0; i < 16; ++i) o[i] = x[i] + s[i];
}

class Drbg {
   public:
    Drbg(const uint32_t key[8], uint32_t stream) : stream_(stream) { memcpy(key_, key, sizeof key_); }
    uint32_t u32() {
        if (pos_ == 16) {
            chacha(key_, (uint32_t)ctr_, (uint32_t)(ctr_ >> 32), stream_, 0x47425244u, 20, buf_);
            ++ctr_;
            pos_ = 0;
        }
        return buf_[pos_++];
    }
    uint64_t u64() {
        const uint64_t lo = u32();
        return lo | (uint64_t)u32() << 32;
    }
    uint64_t below(uint64_t q) {
        const uint64_t rem = (UINT64_MAX % q + 1) % q;
        for (;;) {
            const uint64_t v = u64();
            if (v >= rem) return v % q;
        }
    }
    double unit() { return (double)(u64() >> 11) * (1.0 / 9007199254740992.0); }
    void seed8(uint32_t out[8]) {
        for (int i = 0; i < 8; ++i) out[i] = u32();
    }

   private:
    uint32_t key_[8];
    uint32_t stream_;
    uint64_t ctr_ = 0;
    uint32_t buf_[16];
    int pos_ = 16;
};

// uniform ternary (crates/pc-core/src/keys.rs:228-243) and sparse ternary of weight h (:245-260)
inline void ternary(Drbg& g, size_t n, int8_t* out) {
    size_t k = 0;
    while (k < n) {
        uint32_t w = g.u32();
        for (int i = 0; i < 16; ++i, w >>= 2)
            if ((w & 3) < 3 && k < n) out[k++] = (int8_t)((int)(w & 3) - 1);
    }
}
inline bool sparse_ternary(Drbg& g, size_t n, size_t h, int8_t* out) {
    if (h > n) return false;
    memset(out, 0, n);
    for (size_t placed = 0; placed < h;) {
        const size_t i = (size_t)g.below(n);
        if (!out[i]) {
            out[i] = (g.u32() & 1) ? -1 : 1;
            ++placed;
        }
    }
    return true;
}

// discrete Gaussian by inversion of the |x| cdf on |x| <= ceil(14 sigma) (crates/pc-core/src/keys.rs:267-325)
class Gauss {
   public:
    explicit Gauss(double sigma) {
        const size_t bound = (size_t)std::ceil(sigma * 14.0);
        std::vector<double> w(bound + 1);
        double tot = 0.0;
        for (size_t k = 0; k <= bound; ++k) {
            const double p = std::exp(-((double)(k * k)) / (2.0 * sigma * sigma));
            w[k] = k ? 2.0 * p : p;
        }
        for (double x : w) tot += x;
        double acc = 0.0;
        for (double x : w) {
            acc += x / tot;
            cdf_.push_back(acc);
        }
    }
    int64_t draw(Drbg& g) const {
        const double u = g.unit();
        size_t k = (size_t)(std::upper_bound(cdf_.begin(), cdf_.end(), u) - cdf_.begin());
        k = std::min(k, cdf_.size() - 1);
        if (!k) return 0;
        return (g.u32() & 1) ? -(int64_t)k : (int64_t)k;
    }

   private:
    std::vector<double> cdf_;
};

// ------------------------------------------------------------------------------------------------ encoder
// OpenFHE FFTSpecial / FFTSpecialInv over the rotation group of 5 (crates/pc-core/src/encode.rs:84-331): values are
// (re, im) pairs; encode rounds half away from zero into exact i128 coefficients at gap N / (2 slots) (real parts)
// and + N/2 (imaginary parts); decode reads the centred residues of the bottom prime.
class Encoder {
   public:
    explicit Encoder(size_t n) : n_(n) {
        const size_t m = 2 * n, nh = n / 2;
        std::vector<size_t> rot(nh);
        for (size_t j = 0, f = 1; j < nh; ++j, f = f * 5 % m) rot[j] = f;
        std::vector<double> kr(m + 1), ki(m + 1);
        for (size_t j = 0; j < m; ++j) {
            const double ang = 2.0 * M_PI * (double)j / (double)m;
            kr[j] = std::cos(ang);
            ki[j] = std::sin(ang);
        }
        kr[m] = kr[0];
        ki[m] = ki[0];
        for (size_t h = 1; h < nh; h *= 2) {
            const size_t q = 8 * h, gap = m / q;
            for (size_t k = 0; k < h; ++k) {
                twr_.push_back(kr[(rot[k] % q) * gap]);
                twi_.push_back(ki[(rot[k] % q) * gap]);
            }
            for (size_t k = 0; k < h; ++k) {
                itr_.push_back(kr[(q - rot[k] % q) * gap]);
                iti_.push_back(ki[(q - rot[k] % q) * gap]);
            }
        }
    }
    // false when a scaled value leaves the exact range (|x| >= 2^126)
    bool encode(const double* vals, int nvals, int slots, double scale, std::vector<i128>& c) const {
        std::vector<double> re(slots, 0.0), im(slots, 0.0);
        for (int i = 0; i < nvals && i < slots; ++i) {
            re[i] = vals[2 * i];
            im[i] = vals[2 * i + 1];
        }
        // FFTSpecialInv
        for (size_t len = (size_t)slots; len >= 2; len >>= 1) {
            const size_t h = len >> 1;
            for (size_t b = 0; b < (size_t)slots; b += len)
                for (size_t k = 0; k < h; ++k) {
                    const double ar = re[b + k], ai = im[b + k], br = re[b + k + h], bi = im[b + k + h];
                    const double ur = ar + br, ui = ai + bi, dr = ar - br, di = ai - bi;
                    const double wr = itr_[h - 1 + k], wi = iti_[h - 1 + k];
                    re[b + k] = ur;
                    im[b + k] = ui;
                    re[b + k + h] = dr * wr - di * wi;
                    im[b + k + h] = dr * wi + di * wr;
                }
        }
        bitrev_perm(re, im);
        const size_t gap = n_ / (2 * (size_t)slots);
        c.assign(n_, 0);
        const double lim = std::ldexp(1.0, 126);
        for (int i = 0; i < slots; ++i) {
            const double a = std::round(re[i] / (double)slots * scale), b = std::round(im[i] / (double)slots * scale);
            if (!std::isfinite(a) || !std::isfinite(b) || std::fabs(a) >= lim || std::fabs(b) >= lim) return false;
            c[gap * i] = (i128)a;
            c[gap * i + n_ / 2] = (i128)b;
        }
        return true;
    }
    void decode(const std::vector<i128>& c, int slots, double scale, double* out) const {
        const size_t gap = n_ / (2 * (size_t)slots);
        std::vector<double> re(slots), im(slots);
        auto f = [&](i128 x) {
            return (x >= (i128)INT64_MIN && x <= (i128)INT64_MAX) ? (double)(int64_t)x / scale : (double)x / scale;
        };
        for (int i = 0; i < slots; ++i) {
            re[i] = f(c[gap * i]);
            im[i] = f(c[gap * i + n_ / 2]);
        }
        bitrev_perm(re, im);
        // FFTSpecial
        for (size_t len = 2; len <= (size_t)slots; len <<= 1) {
            const size_t h = len >> 1;
            for (size_t b = 0; b < (size_t)slots; b += len)
                for (size_t k = 0; k < h; ++k) {
                    const double wr = twr_[h - 1 + k], wi = twi_[h - 1 + k];
                    const double br = re[b + k + h], bi = im[b + k + h];
                    const double vr = br * wr - bi * wi, vi = br * wi + bi * wr;
                    const double ur = re[b + k], ui = im[b + k];
                    re[b + k] = ur + vr;
                    im[b + k] = ui + vi;
                    re[b + k + h] = ur - vr;
                    im[b + k + h] = ui - vi;
                }
        }
        for (int i = 0; i < slots; ++i) {
            out[2 * i] = re[i];
            out[2 * i + 1] = im[i];
        }
    }

   private:
    static void bitrev_perm(std::vector<double>& re, std::vector<double>& im) {
        const size_t size = re.size();
        for (size_t i = 1, j = 0; i < size; ++i) {
            size_t bit = size >> 1;
            for (; j >= bit; bit >>= 1) j -= bit;
            j += bit;
            if (i < j) {
                std::swap(re[i], re[j]);
                std::swap(im[i], im[j]);
            }
        }
    }
    size_t n_;
    std::vector<double> twr_, twi_, itr_, iti_;
};

inline uint64_t mod_i128(i128 x, uint64_t q) {
    i128 r = x % (i128)q;
    return (uint64_t)(r < 0 ? r + q : r);
}

}  // namespace hm
}  // namespace pcb
