"""Test infrastructure: the reference's own references for its wire format, restated with Python integers
(crates/pc-client/src/wire.rs tests: pack_coeffs_ref :793-806 on its exact branch, pack_bits_ref :808-818,
unpack_bits_ref :820-829; sum64 :12-25; unpack_coeffs :405-410)."""


def sum64_ref(words):
    h = 0xCBF29CE484222325
    w = [int(x) for x in words]
    for i in range(0, len(w) - 1, 2):
        h = ((h ^ (w[i] | (w[i + 1] << 32))) * 0x100000001B3) & (2**64 - 1)
    if len(w) % 2:
        h = ((h ^ w[-1]) * 0x100000001B3) & (2**64 - 1)
    return h


def pack_coeffs_ref(q, rows, bits):
    """round(x 2^bits / Q) mod 2^bits of the CRT x in [0, Q) of each coefficient's residues (exact)."""
    big = 1
    for p in q:
        big *= int(p)
    out = []
    for i in range(len(rows[0])):
        x = 0
        for r, p in enumerate(q):
            m = big // int(p)
            x = (x + (int(rows[r][i]) % int(p)) * pow(m % int(p), -1, int(p)) * m) % big
        out.append((((x << bits) + big // 2) // big) & ((1 << bits) - 1))
    return out


def pack_bits_ref(v, bits):
    out = [0] * ((len(v) * bits + 31) // 32)
    for i, x in enumerate(v):
        bit = i * bits
        w, o = bit // 32, bit % 32
        x = (int(x) & ((1 << bits) - 1)) << o
        for k in range((o + bits + 31) // 32):
            out[w + k] |= (x >> (32 * k)) & 0xFFFFFFFF
    return out


def unpack_bits_ref(w, n, bits):
    out = []
    for i in range(n):
        bit = i * bits
        k, o = bit // 32, bit % 32
        x = 0
        for j in range((o + bits + 31) // 32):
            x |= int(w[k + j]) << (32 * j)
        out.append((x >> o) & ((1 << bits) - 1))
    return out


def unpack_coeffs_ref(q, words, bits):
    big = 1
    for p in q:
        big *= int(p)
    xs = [((int(y) * big) + (1 << (bits - 1))) >> bits for y in words]
    return [[x % big % int(p) for x in xs] for p in q]
