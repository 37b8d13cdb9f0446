// The versioned wire format of crates/pc-client/src/wire.rs: frames (magic, version, JSON header length, JSON
// header, payloads of little-endian u32 words each followed by its FNV-1a checksum), bit-packed rows, and the
// compressed ciphertext frame (each coefficient as round(x 2^bits / Q), x the CRT of its residues). The host functions
// move bytes; the JSON header is written and read by the caller (perseus_b200/wire.py). The compression runs on the
// device (`compress`, launched by pcb_ct_compress in evaluator.cu after the INTT of the frame's rows).
#include <cstring>

#include "arith.cuh"
#include "kernels.h"

namespace pcb {
namespace wire {

// ------------------------------------------------------------------------------------------------ 128-bit helpers
struct U128 {
    uint64_t lo, hi;
};
__device__ __forceinline__ U128 mul64(uint64_t a, uint64_t b) { return {a * b, __umul64hi(a, b)}; }
__device__ __forceinline__ U128 add(U128 a, U128 b) {
    const uint64_t lo = a.lo + b.lo;
    return {lo, a.hi + b.hi + (lo < a.lo)};
}
__device__ __forceinline__ U128 sub(U128 a, U128 b) { return {a.lo - b.lo, a.hi - b.hi - (a.lo < b.lo)}; }
__device__ __forceinline__ bool ge(U128 a, U128 b) { return a.hi != b.hi ? a.hi > b.hi : a.lo >= b.lo; }
__device__ __forceinline__ U128 shl(U128 a, int s) {  // 0 <= s < 128
    if (s == 0) return a;
    if (s >= 64) return {0, a.lo << (s - 64)};
    return {a.lo << s, (a.hi << s) | (a.lo >> (64 - s))};
}
__device__ __forceinline__ U128 shr1(U128 a) { return {(a.lo >> 1) | (a.hi << 63), a.hi >> 1}; }

// round(x 2^bits / Q) mod 2^bits for x < Q, Q < 2^(127 - bits): floor((x 2^bits + floor(Q / 2)) / Q) by restoring
// division over the bits + 1 quotient bits (the quotient is below 2^(bits + 1)), then masked: wire.rs pack_coeffs'
// `(((x << bits) + big / 2) / big) & mask`, bit for bit
__device__ __forceinline__ uint64_t round_scaled(U128 x, U128 Q, int bits) {
    U128 num = add(shl(x, bits), shr1(Q));
    uint64_t y = 0;
    U128 d = shl(Q, bits);
    for (int j = bits; j >= 0; --j) {
        if (ge(num, d)) {
            num = sub(num, d);
            if (j < 64) y |= 1ull << j;
        }
        d = shr1(d);
    }
    return bits == 64 ? y : (y & ((1ull << bits) - 1));
}

// One thread per 32 coefficients of one part (blockIdx.y): the CRT x of the k coefficient rows (k = 1: x = v0;
// k = 2: Garner, x = v0 + q0 ((v1 - v0) q0^-1 mod q1)), y = round(x 2^bits / Q), the 32 values packed LSB first into
// exactly `bits` u32 words at word (i / 32) bits of the part's stream (the part's stream: n bits / 32 words).
__global__ void __launch_bounds__(128) compress(const uint64_t* coef, int k, uint32_t n, PcbPrimeConst c0,
                                                PcbPrimeConst c1, uint64_t inv01, int bits, uint32_t* out) {
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;  // group of 32 coefficients
    if ((size_t)g * 32 >= n) return;
    const int part = blockIdx.y;
    const uint64_t* r0 = coef + (size_t)part * k * n;
    const uint64_t* r1 = r0 + n;
    const U128 Q = k == 1 ? U128{c0.p, 0} : mul64(c0.p, c1.p);
    uint32_t* o = out + (size_t)part * ((size_t)n * bits / 32) + (size_t)g * bits;
    uint64_t acc = 0;  // pending bits, LSB first
    int nb = 0, w = 0;
    for (int e = 0; e < 32; ++e) {
        const size_t i = (size_t)g * 32 + e;
        const uint64_t v0 = r0[i];
        U128 x = {v0, 0};
        if (k == 2) {
            const uint64_t v0m = v0 % c1.p;
            const uint64_t d = sub_mod(r1[i], v0m, c1.p);
            const uint64_t t = mul_mod(d, inv01, c1);
            x = add(x, mul64(c0.p, t));
        }
        const uint64_t y = round_scaled(x, Q, bits);
        // append `bits` bits of y
        int left = bits;
        uint64_t v = y;
        while (left > 0) {
            const int take = left < 64 - nb ? left : 64 - nb;
            const uint64_t part_bits = take == 64 ? v : (v & ((1ull << take) - 1));
            acc |= part_bits << nb;
            nb += take;
            v = take == 64 ? 0 : (v >> take);
            left -= take;
            while (nb >= 32) {
                o[w++] = (uint32_t)acc;
                acc >>= 32;
                nb -= 32;
            }
        }
    }
}

}  // namespace wire

namespace keys {
// Packed key rows -> dense u64 rows (the table's ksk_unpack, args.cuh:656-663): one thread per value; value i of row r
// sits at bits [i bits, (i + 1) bits) of the row's LSB-first u32 stream; up to three words hold it when bits > 32
// (the guard word keeps the reads of the last value inside the row).
template <int LOGN>
__global__ void __launch_bounds__(128) ksk_unpack(PcbKskUnpackArgs a) {
    const int r = blockIdx.y;
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t* in = a.in + (size_t)r * a.row_words;
    const uint64_t bit = (uint64_t)i * a.bits;
    const uint64_t w = bit >> 5;
    const int o = (int)(bit & 31);
    uint64_t x = ((uint64_t)in[w] | ((uint64_t)in[w + 1] << 32)) >> o;
    if (o + a.bits > 64) x |= (uint64_t)in[w + 2] << (64 - o);
    const uint64_t mask = a.bits == 64 ? ~0ull : ((1ull << a.bits) - 1);
    ((uint64_t*)a.out)[((size_t)r << LOGN) + i] = x & mask;
}

template <int LOGN>
int ksk_unpack_launch(const PcbKskUnpackArgs* ap, cudaStream_t s) {
    if (!ap) return -1;
    const PcbKskUnpackArgs& a = *ap;
    constexpr uint64_t N = 1ull << LOGN;
    // the reads of the last value end inside the row: ceil((N bits + 32) / 32) words (the guard word and, above 32
    // bits, one more), which packed_row_words always covers for bits <= 32
    const uint64_t need = (N * (uint64_t)a.bits + 31) / 32 + (a.bits > 32 ? 2 : 1);
    if (!a.out || !a.in || a.bits <= 0 || a.bits > 64 || a.nrows < 0 || a.row_words < need) return -1;
    if (a.nrows == 0) return 0;
    ksk_unpack<LOGN><<<dim3((unsigned)(N / 128), (unsigned)a.nrows), 128, 0, s>>>(a);
    return (int)cudaGetLastError();
}
template int ksk_unpack_launch<14>(const PcbKskUnpackArgs*, cudaStream_t);
template int ksk_unpack_launch<16>(const PcbKskUnpackArgs*, cudaStream_t);
}  // namespace keys

int wire_compress_launch(const uint64_t* coef, int k, size_t n, const PcbPrimeConst& c0, const PcbPrimeConst& c1,
                         uint64_t inv01, int bits, uint32_t* out, cudaStream_t s) {
    const unsigned groups = (unsigned)(n / 32);
    wire::compress<<<dim3((groups + 127) / 128, 2), 128, 0, s>>>(coef, k, (uint32_t)n, c0, c1, inv01, bits, out);
    return (int)cudaGetLastError();
}

}  // namespace pcb

// ================================================================================================ host (C ABI)
namespace {
constexpr uint32_t WIRE_VERSION = 1;  // wire.rs VERSION
}

extern "C" {

// FNV-1a over little-endian u64 words (a trailing odd u32 word widened): wire.rs sum64
uint64_t pcb_wire_sum64(const uint32_t* w, size_t n) {
    uint64_t h = 0xcbf29ce484222325ull;
    const uint64_t prime = 0x00000100000001b3ull;
    size_t i = 0;
    for (; i + 1 < n; i += 2) {
        h ^= (uint64_t)w[i] | ((uint64_t)w[i + 1] << 32);
        h *= prime;
    }
    if (i < n) {
        h ^= (uint64_t)w[i];
        h *= prime;
    }
    return h;
}

// u32 words of n values of `bits` bits, bit-packed: wire.rs packed_words
size_t pcb_wire_packed_words(size_t n, int32_t bits) { return (n * (size_t)bits + 31) / 32; }

// u32 words of one packed row (one zero guard word, padded to 16 bytes): wire.rs packed_row_words
size_t pcb_wire_packed_row_words(size_t n, int32_t bits) { return ((n * (size_t)bits / 32 + 1) + 3) / 4 * 4; }

// Values of `bits` bits (1..64) LSB first into pcb_wire_packed_words(n, bits) words: wire.rs pack_bits (for bits <= 32
// also the bit order of pack_row). Values are masked to `bits` bits.
int pcb_wire_pack_bits(const uint64_t* v, size_t n, int32_t bits, uint32_t* out) {
    if (!v || !out || bits < 1 || bits > 64) return -1;
    const uint64_t mask = bits == 64 ? ~0ull : ((1ull << bits) - 1);
    const size_t words = pcb_wire_packed_words(n, bits);
    memset(out, 0, words * 4);
    for (size_t i = 0; i < n; ++i) {
        const uint64_t x = v[i] & mask;
        const size_t bit = i * (size_t)bits;
        const size_t w = bit >> 5;
        const int o = (int)(bit & 31);
        // x << o spans up to 3 words
        out[w] |= (uint32_t)(x << o);
        if (o + bits > 32) out[w + 1] |= (uint32_t)(o == 0 ? (x >> 32) : (x >> (32 - o)));
        if (o + bits > 64) out[w + 2] |= (uint32_t)(x >> (64 - o));
    }
    return 0;
}

// Inverse of pcb_wire_pack_bits: n values of `bits` bits from `in` (in_words words; reads never pass them).
int pcb_wire_unpack_bits(const uint32_t* in, size_t in_words, size_t n, int32_t bits, uint64_t* out) {
    if (!in || !out || bits < 1 || bits > 64 || pcb_wire_packed_words(n, bits) > in_words) return -1;
    const uint64_t mask = bits == 64 ? ~0ull : ((1ull << bits) - 1);
    for (size_t i = 0; i < n; ++i) {
        const size_t bit = i * (size_t)bits;
        const size_t w = bit >> 5;
        const int o = (int)(bit & 31);
        uint64_t lo = in[w];
        if (w + 1 < in_words) lo |= (uint64_t)in[w + 1] << 32;
        uint64_t x = lo >> o;
        if (o + bits > 64 && w + 2 < in_words) x |= (uint64_t)in[w + 2] << (64 - o);
        out[i] = x & mask;
    }
    return 0;
}

// One packed row of n values (wire.rs pack_row, widened to values of up to 64 bits): the values bit-packed, the rest
// of out (out_words >= pcb_wire_packed_row_words(n, bits), guard word included) zero.
int pcb_wire_pack_row(const uint64_t* v, size_t n, int32_t bits, uint32_t* out, size_t out_words) {
    if (!out || bits < 1 || bits > 64 || out_words < pcb_wire_packed_row_words(n, bits)) return -1;
    memset(out, 0, out_words * 4);
    return pcb_wire_pack_bits(v, n, bits, out);
}

// Frame header: magic (4 bytes), version (u32 LE), JSON length (u64 LE), the JSON bytes. Returns the bytes written
// (16 + len), or -1 (null argument, out of room).
int64_t pcb_wire_write_header(const char* magic, const uint8_t* json, uint64_t len, uint8_t* out, uint64_t cap) {
    if (!magic || (!json && len) || !out || cap < 16 + len) return -1;
    memcpy(out, magic, 4);
    const uint32_t ver = WIRE_VERSION;
    memcpy(out + 4, &ver, 4);  // little-endian hosts only (x86-64, aarch64)
    memcpy(out + 8, &len, 8);
    if (len) memcpy(out + 16, json, len);
    return (int64_t)(16 + len);
}

// Parses a frame header (wire.rs read_header): returns the JSON's offset (16) with its length in *json_len, or
// -1 (short buffer), -2 (wrong magic), -3 (another version), -4 (a header above 1 GiB or past the buffer).
int64_t pcb_wire_read_header(const uint8_t* buf, uint64_t n, const char* magic, uint64_t* json_len) {
    if (!buf || !magic || !json_len || n < 16) return -1;
    if (memcmp(buf, magic, 4) != 0) return -2;
    uint32_t ver;
    memcpy(&ver, buf + 4, 4);
    if (ver != WIRE_VERSION) return -3;
    uint64_t len;
    memcpy(&len, buf + 8, 8);
    if (len > (1ull << 30) || 16 + len > n) return -4;
    *json_len = len;
    return 16;
}

// Client side of the compressed frame (wire.rs unpack_coeffs): residues mod each q[r] of round(y Q / 2^bits) for the
// n words y (one per coefficient); rows [nq][n]. nq 1..2, every q below 2^63, bits 1..64 with the sum of the primes'
// bits + bits <= 127.
int pcb_wire_unpack_coeffs(const uint64_t* q, int32_t nq, const uint64_t* y, size_t n, int32_t bits, uint64_t* rows) {
    if (!q || !y || !rows || nq < 1 || nq > 2 || bits < 1 || bits > 64) return -1;
    unsigned __int128 Q = 1;
    int qbits = 0;
    for (int r = 0; r < nq; ++r) {
        if (q[r] < 2 || (q[r] >> 63)) return -1;
        Q *= q[r];
        qbits += 64 - __builtin_clzll(q[r]);
    }
    if (qbits + bits > 127) return -1;
    for (size_t i = 0; i < n; ++i) {
        // (y Q + 2^(bits - 1)) >> bits, in 192 bits: y Q = (y Q_lo) + (y Q_hi) 2^64
        const uint64_t Qlo = (uint64_t)Q, Qhi = (uint64_t)(Q >> 64);
        const unsigned __int128 a = (unsigned __int128)y[i] * Qlo;
        const unsigned __int128 b = (unsigned __int128)y[i] * Qhi + (uint64_t)(a >> 64);
        // 192-bit value: words w0 = (uint64)a, w1 = (uint64)b, w2 = b >> 64
        uint64_t w0 = (uint64_t)a, w1 = (uint64_t)b, w2 = (uint64_t)(b >> 64);
        const unsigned __int128 half = (unsigned __int128)1 << (bits - 1);
        const unsigned __int128 lo = ((unsigned __int128)w1 << 64 | w0) + half;
        if (lo < half) ++w2;
        w0 = (uint64_t)lo;
        w1 = (uint64_t)(lo >> 64);
        // shift right by bits (1..64)
        unsigned __int128 x;
        if (bits == 64) {
            x = ((unsigned __int128)w2 << 64) | w1;
        } else {
            x = ((unsigned __int128)w2 << (128 - bits)) | ((((unsigned __int128)w1 << 64) | w0) >> bits);
        }
        x %= Q;
        for (int r = 0; r < nq; ++r) rows[(size_t)r * n + i] = (uint64_t)(x % q[r]);
    }
    return 0;
}

}  // extern "C"
