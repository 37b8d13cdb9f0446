"""The wire format's byte work on the host (perseus_b200/wire.py over pcb_wire_*), against the reference's own test
references restated in tests/_wire_ref.py and its test cases (crates/pc-client/src/wire.rs:759-1019)."""
import numpy as np
import pytest

from perseus_b200 import fhe
from perseus_b200 import wire as W
from tests import _wire_ref as R

GOLD32 = 2654435761
GOLD64 = 0x9E3779B97F4A7C15


def test_pack_row_roundtrip_and_guard():
    """wire.rs pack_roundtrip: 1024 values at 27, 28, 31 bits; the guard word stays zero."""
    n = 1024
    for bits in (27, 28, 31):
        vals = np.array([(i * GOLD32) % 2**32 & ((1 << bits) - 1) for i in range(n)], np.uint64)
        p = W.pack_row(vals, bits)
        assert p.size == W.packed_row_words(n, bits) and p[-1] == 0
        assert (W.unpack_row(p, n, bits) == vals).all()
    # 64-bit residues of these chains at 50 bits
    vals = np.array([(i * GOLD64) % 2**64 & ((1 << 50) - 1) for i in range(n)], np.uint64)
    assert (W.unpack_row(W.pack_row(vals, 50), n, 50) == vals).all()


@pytest.mark.parametrize("bits", [1, 7, 12, 20, 22, 26, 31, 32, 33, 46, 48, 50, 57, 64])
def test_pack_bits_matches_reference(bits):
    """wire.rs pack_matches_reference / pack_bits_roundtrip: word for word against pack_bits_ref, and back."""
    for n in (1, 3, 31, 33, 1000):
        v = np.array([(i * GOLD64) % 2**64 for i in range(n)], np.uint64)
        packed = W.pack_bits(v, bits)
        assert [int(x) for x in packed] == R.pack_bits_ref(v, bits)
        back = W.unpack_bits(packed, n, bits)
        assert [int(x) for x in back] == R.unpack_bits_ref(packed, n, bits)
        assert (back == (v & np.uint64((1 << bits) - 1) if bits < 64 else v)).all()


def test_sum64():
    for n in (0, 1, 2, 7, 1000):
        w = np.array([(i * GOLD32) % 2**32 for i in range(n)], np.uint32)
        assert W.sum64(w) == R.sum64_ref(w)


def test_unpack_coeffs_matches_reference():
    q = fhe.ntt_primes(50, 14, 2)
    rng = np.random.default_rng(3)
    for k, bits in ((1, 20), (1, 64), (2, 12), (2, 27)):
        y = rng.integers(0, 2**63, 257, dtype=np.uint64) & np.uint64((1 << bits) - 1 if bits < 64 else 2**64 - 1)
        got = W.unpack_coeffs(q[:k], y, bits)
        assert [[int(x) for x in r] for r in got] == R.unpack_coeffs_ref(q[:k], y, bits)
    with pytest.raises(W.WireError):
        W.unpack_coeffs(q, y, 28)  # 100 bits of modulus + 28 > 127


def test_frame_roundtrip_and_corruption():
    """wire.rs ct_frame_roundtrip_and_corruption: a frame reads back; a flipped payload bit, a wrong magic, another
    version and a truncated frame are refused."""
    h = W.CtHeader("x", 16, 2, 3, {"level": 4, "deg": 1, "nf": 2.0**54, "slots": 8, "tag": None})
    w = W.CtWire(h, np.arange(h.words(), dtype=np.uint32))
    b = w.to_bytes()
    r = W.CtWire.from_bytes(b)
    assert r.header == h and (r.data == w.data).all()
    bad = bytearray(b)
    bad[len(b) - 20] ^= 1
    with pytest.raises(W.WireError, match="checksum"):
        W.CtWire.from_bytes(bytes(bad))
    with pytest.raises(W.WireError, match="magic"):
        W.CtWire.from_bytes(b"PCKB" + b[4:])
    with pytest.raises(W.WireError, match="version"):
        W.CtWire.from_bytes(b[:4] + (2).to_bytes(4, "little") + b[8:])
    with pytest.raises(W.WireError):
        W.CtWire.from_bytes(b[:-3])
    # a frame of the reference's 32-bit sessions (no word_bits) is read, and refused by import as 32-bit words
    assert W.CtHeader.from_json({"params_hash": "x", "n": 16, "k": 1, "rows": 1, "meta": {}}).word_bits == 32


def test_params_hash():
    a, b = W.params_hash(fhe.config2_chain()), W.params_hash(fhe.config4_chain())
    assert len(a) == 16 and a != b and a == W.params_hash(fhe.config2_chain())
