"""Pins the parity oracle against the reference's own known answers and the selftest's host formulas.

Sources (read as text into tests/golden/reference_pins.json by tests/golden/make_pins.py):
- crates/pc-core/tests/kskb_frozen.rs:13-52 — the frozen u64 KSKB expander, three pinned rows at n = 2^16;
- crates/pc-core/src/params/nbtheory.rs:170-180 — primality, prime search and the minimal 2N-th root;
- crates/pc-host/src/arith.rs:197-214 — the u64 double-word reduction at p = 2^59 - 55;
- crates/pc-kernels/src/bin/selftest/host.rs:119-186 — OpenFHE's bit-reversed negacyclic NTT and the automorphism
  slot map, checked here against direct polynomial evaluation on small rings.
"""
import json
import os

import numpy as np
import pytest

from tests import _oracle as O

PINS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_pins.json")))


def fnv(v):
    h = 0xCBF29CE484222325
    for x in v:
        h = ((h ^ int(x)) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def test_kskb_frozen_vectors():
    k = PINS["kskb_frozen"]
    for digit, (p, a0, a1, alast, h) in zip(k["digits"], k["pinned"]):
        row = O.expand_row(k["seed"], digit, p, O.TAG_KSKA, k["logn"])
        assert int(row[0]) == a0 and int(row[1]) == a1 and int(row[-1]) == alast
        assert fnv(row) == h
        assert (row < np.uint64(p)).all()


def test_nbtheory_known_answers():
    L = O.lib()
    nb = PINS["nbtheory"]
    assert L.orc_is_prime(nb["prime"]) == 1
    assert L.orc_is_prime(nb["composite"]) == 0
    assert L.orc_is_prime(nb["strong_pseudoprime"]) == 0
    m = nb["m"]
    assert L.orc_previous_prime(L.orc_first_prime(28, m), m) == nb["previous_of_first_28"]
    assert L.orc_root_of_unity(m, nb["root_prime"]) == nb["root"]


def test_u64_reduction_cases():
    L = O.lib()
    p = (1 << 59) - 55
    for a, b in [(p - 1, p - 1), (1 << 58, 3), (7, 9)]:
        assert L.orc_mulmod(a, b, p) == a * b % p
    m = (1 << 128) - 1
    assert L.orc_reduce128(m & ((1 << 64) - 1), m >> 64, p) == m % p
    pc = np.zeros(8, np.uint64)
    L.orc_prime_const(p, pc)
    mu = int(pc[1]) | int(pc[2]) << 64
    assert mu == ((1 << 128) - 1) // p
    assert (p * ((1 << 64) - int(pc[5]))) % (1 << 64) == 1  # mont_pinv = -p^-1 mod 2^64


def test_chacha20_block_rfc7539():
    # RFC 7539 section 2.3.2 block function test vector (the DRBG's block is standard ChaCha20)
    key = np.array([int.from_bytes(bytes(range(4 * i, 4 * i + 4)), "little") for i in range(8)], np.uint32)
    out = np.zeros(16, np.uint32)
    O.lib().orc_chacha_block(key, 1, 0x09000000, 0x4A000000, 0, 20, out)
    assert [int(x) for x in out[:4]] == [0xE4E7F110, 0x15593BD1, 0x1FDD0F50, 0xC47120A3]


def test_prng_uniform_below_and_sparse_secret():
    L = O.lib()
    g = L.orc_prng_new(np.array([3] * 8, np.uint32), 0)
    try:
        s = np.zeros(1 << 10, np.int8)
        assert L.orc_sample_sparse_ternary(g, 1 << 10, 32, s) == 0
        assert int((s != 0).sum()) == 32 and set(np.unique(s)) <= {-1, 0, 1}
        vals = [L.orc_prng_below(g, 97) for _ in range(2000)]
        assert min(vals) >= 0 and max(vals) < 97
    finally:
        L.orc_prng_free(g)


def _naive_eval(a, p, psi, logn):
    n = 1 << logn
    out = []
    for i in range(n):
        j = int("{:0{w}b}".format(i, w=logn)[::-1], 2)
        x = pow(psi, 2 * j + 1, p)
        acc = 0
        for c in reversed(a):
            acc = (acc * x + int(c)) % p
        out.append(acc)
    return out


@pytest.mark.parametrize("logn", [3, 5, 7])
def test_ntt_is_bitreversed_negacyclic_evaluation(logn):
    L = O.lib()
    (p,) = O.ntt_primes(50, logn, 1)
    psi = L.orc_root_of_unity(2 << logn, p)
    rng = np.random.default_rng(logn)
    a = rng.integers(0, p, 1 << logn, dtype=np.uint64)
    x = a.copy()
    L.orc_ntt_fwd(x, 1, np.array([p], np.uint64), logn)
    assert [int(v) for v in x] == _naive_eval(a, p, psi, logn)
    L.orc_ntt_inv(x, 1, np.array([p], np.uint64), logn)
    assert (x == a).all()


def test_automorph_slot_is_the_galois_map():
    L = O.lib()
    logn = 6
    n = 1 << logn
    (p,) = O.ntt_primes(50, logn, 1)
    rng = np.random.default_rng(1)
    a = rng.integers(0, p, n, dtype=np.uint64)
    for k in (5, 25, 2 * n - 1):
        # a(X^k) in coefficient form (crates/pc-kernels/src/bin/selftest/host.rs:170-186)
        b = np.zeros(n, np.uint64)
        for i in range(n):
            e = i * k % (2 * n)
            b[e % n] = a[i] if e < n else (p - int(a[i])) % p
        fa, fb = a.copy(), b.copy()
        L.orc_ntt_fwd(fa, 1, np.array([p], np.uint64), logn)
        L.orc_ntt_fwd(fb, 1, np.array([p], np.uint64), logn)
        gathered = np.array([fa[L.orc_automorph_slot(k, o, logn)] for o in range(n)], np.uint64)
        assert (gathered == fb).all()
