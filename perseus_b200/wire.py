"""The versioned wire format (crates/pc-client/src/wire.rs) for this library's 64-bit chains: key bundles and
ciphertext frames, with the reference's framing (magic, version 1, JSON header, payloads of little-endian u32 words
each followed by its FNV-1a `sum64`), JSON field names and packing. The byte work (checksums, bit packing, frame
headers, the compressed frame's CRT and rounding on the device) is the C ABI's (pcb_wire_*, pcb_ct_compress); this
module writes and reads the JSON headers and moves the payloads, as crates/pc-py/src/client.rs's export_ct / import_ct
do for the reference's sessions.

What is the reference's, bit for bit: the framing and the checksum; `pack_bits` / `unpack_bits`; `pack_row`'s layout
(bits <= 32; wider values continue LSB first); the compressed frame (`bits`: each coefficient's CRT x in [0, Q) as
round(x 2^bits / Q), the exact path of `pack_coeffs`); `params_hash` (spec.rs:252-267) over this chain.
What is this library's (the reference defines these for 32-bit words only): a plain frame's residues are u64 words,
two u32 words each, marked `"word_bits": 64` in the header; a key bundle's `b` rows pack 64-bit residues at the
bundle's `bits` (50 for these chains, where the reference packs u32 residues at <= 32).
"""
import ctypes as C
import json
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib as L
from . import fhe

VERSION = 1
BUNDLE_MAGIC = b"PCKB"
CT_MAGIC = b"PCCT"


class WireError(ValueError):
    pass


def _u32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


def _p(a):
    return C.c_void_p(a.ctypes.data)


# ------------------------------------------------------------------------------------------------ primitives
def sum64(words):
    w = _u32(words)
    return int(L.lib().pcb_wire_sum64(_p(w), w.size))


def packed_words(n, bits):
    return int(L.lib().pcb_wire_packed_words(n, bits))


def packed_row_words(n, bits):
    return int(L.lib().pcb_wire_packed_row_words(n, bits))


def pack_bits(values, bits):
    v = np.ascontiguousarray(np.asarray(values, dtype=np.uint64))
    out = np.zeros(packed_words(v.size, bits), np.uint32)
    if L.lib().pcb_wire_pack_bits(_p(v), v.size, bits, _p(out)):
        raise WireError(f"pack_bits: {bits} bits")
    return out


def unpack_bits(words, n, bits):
    w = _u32(words)
    out = np.zeros(n, np.uint64)
    if L.lib().pcb_wire_unpack_bits(_p(w), w.size, n, bits, _p(out)):
        raise WireError(f"unpack_bits: {n} values of {bits} bits from {w.size} words")
    return out


def pack_row(values, bits, row_words=None):
    """One packed row (zero guard word, padded to 16 bytes): wire.rs pack_row."""
    v = np.ascontiguousarray(np.asarray(values, dtype=np.uint64))
    rw = row_words or packed_row_words(v.size, bits)
    out = np.zeros(rw, np.uint32)
    if L.lib().pcb_wire_pack_row(_p(v), v.size, bits, _p(out), rw):
        raise WireError(f"pack_row: {v.size} values of {bits} bits into {rw} words")
    return out


def unpack_row(packed, n, bits):
    return unpack_bits(packed, n, bits)


def unpack_coeffs(q, words, bits):
    """The client's side of a compressed frame (wire.rs unpack_coeffs): residue rows [len(q)][n]."""
    qa = np.ascontiguousarray(np.asarray(q, np.uint64))
    y = np.ascontiguousarray(np.asarray(words, np.uint64))
    rows = np.zeros((qa.size, y.size), np.uint64)
    if L.lib().pcb_wire_unpack_coeffs(_p(qa), qa.size, _p(y), y.size, bits, _p(rows)):
        raise WireError(f"unpack_coeffs: {bits} bits over {qa.size} primes")
    return rows


def write_header(magic, header):
    js = json.dumps(header, separators=(",", ":")).encode()
    out = np.zeros(16 + len(js), np.uint8)
    jb = np.frombuffer(js, np.uint8) if js else np.zeros(1, np.uint8)
    n = L.lib().pcb_wire_write_header(magic, _p(jb), len(js), _p(out), out.size)
    if n < 0:
        raise WireError("write_header")
    return out.tobytes()


def read_header(buf, magic):
    """(header dict, offset of the payload) of a frame."""
    b = np.frombuffer(buf, np.uint8)
    ln = C.c_uint64()
    off = L.lib().pcb_wire_read_header(_p(b), b.size, magic, C.byref(ln))
    if off < 0:
        why = {-1: "short frame", -2: "wrong magic", -3: f"version; this build reads version {VERSION}",
               -4: "header length"}[off]
        raise WireError(f"frame header: {why}")
    return json.loads(bytes(b[off:off + ln.value])), off + ln.value


def fnv1a64(data):
    h = 0xCBF29CE484222325
    for x in data:
        h = ((h ^ x) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def params_hash(chain):
    """spec.rs:252-267 over this chain: N, the Q then P primes, the digits (contiguous, alpha = ceil(nq / dnum) limbs
    each), level_unit 1, word_bits 64."""
    b = bytearray(np.uint64(chain.n).tobytes())
    for p in tuple(chain.q) + tuple(chain.p):
        b += np.uint64(p).tobytes()
    nq = len(chain.q)
    alpha = -(-nq // chain.dnum)
    for d in range(chain.dnum):
        ids = list(range(d * alpha, min((d + 1) * alpha, nq)))
        b += np.uint64(len(ids)).tobytes()
        for i in ids:
            b += np.uint64(i).tobytes()
    b += np.uint64(1).tobytes() + np.uint32(64).tobytes()
    return f"{fnv1a64(bytes(b)):016x}"


# ------------------------------------------------------------------------------------------------ ciphertext frame
@dataclass
class CtHeader:
    """wire.rs CtHeader (meta: level = primes dropped, deg, nf = the scale, slots, tag)."""

    params_hash: str
    n: int
    k: int
    rows: int
    meta: dict
    bits: int = None
    word_bits: int = 64

    def to_json(self):
        h = {"params_hash": self.params_hash, "n": self.n, "k": self.k, "rows": self.rows, "meta": self.meta}
        if self.bits is not None:
            h["bits"] = self.bits
        else:
            h["word_bits"] = self.word_bits
        return h

    @staticmethod
    def from_json(h):
        for f in ("seeded", "regen", "sparse", "coeff0", "coeff1"):
            if h.get(f):
                raise WireError(f"a {f} frame: not produced for 64-bit chains")
        for f in ("bits1", "drop", "sub1"):
            if h.get(f) is not None:
                raise WireError(f"a frame with {f}: not produced for 64-bit chains")
        return CtHeader(h["params_hash"], h["n"], h["k"], h["rows"], h["meta"], h.get("bits"), h.get("word_bits", 32))

    def words(self):
        """u32 payload words (wire.rs CtWire::words, u64 residues as two words each)."""
        if self.bits is not None:
            return self.k * 2 * packed_words(self.n, self.bits)
        return self.k * 2 * self.rows * self.n * (self.word_bits // 32)


@dataclass
class CtWire:
    header: CtHeader
    data: np.ndarray = field(repr=False)  # u32 words

    def to_bytes(self):
        if self.data.size != self.header.words():
            raise WireError(f"ciphertext data has {self.data.size} words, the header needs {self.header.words()}")
        d = _u32(self.data)
        return write_header(CT_MAGIC, self.header.to_json()) + d.tobytes() + np.uint64(sum64(d)).tobytes()

    @staticmethod
    def from_bytes(buf):
        h, off = read_header(buf, CT_MAGIC)
        hd = CtHeader.from_json(h)
        nw = hd.words()
        end = off + 4 * nw
        if len(buf) != end + 8:
            raise WireError(f"frame of {len(buf)} bytes, its header describes {end + 8}")
        data = np.frombuffer(buf, np.uint32, nw, off).copy()
        if int(np.frombuffer(buf, np.uint64, 1, end)[0]) != sum64(data):
            raise WireError("ciphertext checksum mismatch")
        return CtWire(hd, data)


def _meta(s, ct):
    return {"level": s.nq - 1 - ct.top, "deg": 1, "nf": float(ct.scale), "slots": int(ct.slots), "tag": None}


def export_ct(s, ct, bits=None):
    """A frame of ct (every member of a batch; crates/pc-py/src/client.rs:575-625 export_ct): the residues of rows
    0..top (evaluation form, u64 words), or with `bits` the compressed frame of a ciphertext at one or two limbs
    (coefficient form, round(x 2^bits / Q) per coefficient, packed on the device) for the client to decrypt."""
    k, rows = ct.k, ct.top + 1
    if bits is None:
        d = ct.data[:, :, :rows].contiguous().cpu().numpy().view(np.uint32).ravel()
    else:
        per = 2 * packed_words(s.n, bits)
        out = torch.zeros(k * per, dtype=torch.int32, device=s.device)
        for c in range(k):
            L.check(L.lib().pcb_ct_compress(s.ctx, C.c_void_p(ct.data[c].data_ptr()), ct.top, bits,
                                            C.c_void_p(out.data_ptr() + 4 * c * per), s._stream()),
                    "pcb_ct_compress")
        d = out.cpu().numpy().view(np.uint32)
    h = CtHeader(params_hash(s.chain), s.n, k, rows, _meta(s, ct), bits)
    return CtWire(h, d).to_bytes()


def import_ct(s, frame):
    """A plain frame (crates/pc-py/src/client.rs:861-940 import_ct) into a ciphertext of this session: the chain must
    be the frame's (params_hash), the rows its level's."""
    w = CtWire.from_bytes(frame)
    h = w.header
    if h.bits is not None:
        raise WireError("a compressed frame (export_ct bits=) is for a client to decrypt")
    if h.word_bits != 64:
        raise WireError(f"a frame of {h.word_bits}-bit words; this session's residues are 64-bit")
    if h.params_hash != params_hash(s.chain) or h.n != s.n:
        raise WireError(f"frame for params {h.params_hash} n {h.n}; this session runs {params_hash(s.chain)} n {s.n}")
    top = s.nq - 1 - int(h.meta["level"])
    if h.rows != top + 1 or not 0 <= top < s.nq:
        raise WireError(f"{h.rows} rows at level {h.meta['level']}")
    res = w.data.view(np.uint64).reshape(h.k, 2, h.rows, h.n)
    out = s.empty(h.k)
    out[:, :, : h.rows].copy_(torch.from_numpy(res.view(np.int64)))
    return fhe.Ct(out, top, float(h.meta["nf"]), int(h.meta["slots"]))


def decompress(s, frame):
    """The client's side of a compressed frame: its coefficient-form residues ([k][2][rows][n]) and metadata (the
    client decrypts c0 + c1 s with its secret; here they are re-imported for tests)."""
    w = CtWire.from_bytes(frame)
    h = w.header
    if h.bits is None:
        raise WireError("not a compressed frame")
    q = list(s.chain.q[: h.rows])
    per = packed_words(h.n, h.bits)
    out = np.zeros((h.k, 2, h.rows, h.n), np.uint64)
    for c in range(h.k):
        for part in range(2):
            seg = w.data[(2 * c + part) * per:(2 * c + part + 1) * per]
            out[c, part] = unpack_coeffs(q, unpack_bits(seg, h.n, h.bits), h.bits)
    return out, h


# ------------------------------------------------------------------------------------------------ key bundle
_STEPS = {}


def _role(s, g):
    """spec.rs Role of the key of galois element g: relin (1), conj (2N - 1), rot (5^step mod 2N), else auto."""
    if g == 1:
        return {"role": "relin"}
    if g == 2 * s.n - 1:
        return {"role": "conj"}
    steps = _STEPS.get(s.n)
    if steps is None:  # the discrete logs of the group generated by 5 mod 2N
        steps, x = {}, 1
        for st in range(s.n // 2):
            steps[x] = st
            x = x * 5 % (2 * s.n)
        _STEPS[s.n] = steps
    if g in steps:
        return {"role": "rot", "step": steps[g], "galois": g}
    return {"role": "auto", "galois": g}


def _galois(s, entry):
    r = entry["role"]
    if r == "relin":
        return 1
    if r == "conj":
        return 2 * s.n - 1
    if r in ("rot", "auto"):
        return int(entry["galois"])
    raise WireError(f"a {r} key: not a key of this library's sessions")


def export_keys(s, contract="perseus-b200"):
    """The session's switching keys as a key bundle (wire.rs BundleHeader + Ksk entries): per key its role, shape, the
    8-word seed of `a` and `b` packed at the bundle's bits ([digit][row][row_words])."""
    bits = max(int(p).bit_length() for p in tuple(s.chain.q) + tuple(s.chain.p))
    rw = packed_row_words(s.n, bits)
    shape = {"q_top": s.nq - 1, "ndig": s.chain.dnum, "nq": s.nq, "kp": s.kp}
    entries, payloads = [], []
    for idx, g in enumerate(s.galois):
        seed = np.zeros(8, np.uint32)
        L.check(L.lib().pcb_key_seed(s.ctx, idx, _p(seed)), "pcb_key_seed")
        b, _ = s.key_tensors(idx)
        rows = b.cpu().numpy().view(np.uint64).reshape(-1, s.n)
        words = np.concatenate([pack_row(r, bits, rw) for r in rows])
        entries.append({"kind": "ksk", **_role(s, g), "shape": shape, "seed": [int(x) for x in seed],
                        "words": int(words.size)})
        payloads.append(words)
    header = {"chain": f"n{s.n}q{s.nq}p{s.kp}d{s.chain.dnum}", "params_hash": params_hash(s.chain),
              "contract": contract, "n": s.n, "bits": bits, "row_words": rw, "entries": entries}
    out = [write_header(BUNDLE_MAGIC, header)]
    for wds in payloads:
        out.append(wds.tobytes() + np.uint64(sum64(wds)).tobytes())
    return b"".join(out)


def read_bundle(buf):
    """(header, [payload words]) of a bundle, every entry's checksum verified (wire.rs BundleReader)."""
    h, off = read_header(buf, BUNDLE_MAGIC)
    payloads = []
    for i, e in enumerate(h["entries"]):
        n = int(e["words"])
        end = off + 4 * n
        if end + 8 > len(buf):
            raise WireError(f"entry {i} runs past the bundle")
        w = np.frombuffer(buf, np.uint32, n, off)
        if int(np.frombuffer(buf, np.uint64, 1, end)[0]) != sum64(w):
            raise WireError(f"entry {i} ({e['kind']}): checksum mismatch")
        payloads.append(w)
        off = end + 8
    if off != len(buf):
        raise WireError(f"bundle is {len(buf)} bytes, its header describes {off}")
    return h, payloads


def import_keys(s, buf):
    """A client's key bundle into a session's key slots (pcb_key_load, in the bundle's order): the rows unpacked on
    the device by the table's ksk_unpack, `a` from each key's seed."""
    h, payloads = read_bundle(buf)
    if h["params_hash"] != params_hash(s.chain) or h["n"] != s.n:
        raise WireError(f"bundle for params {h['params_hash']}; this session runs {params_hash(s.chain)}")
    bits, rw = int(h["bits"]), int(h["row_words"])
    nrows = s.chain.dnum * s.rows
    tab = L.kernel_table(s.log_n)
    for idx, (e, w) in enumerate(zip(h["entries"], payloads)):
        if e["kind"] != "ksk":
            raise WireError(f"a {e['kind']} entry: this session loads switching keys")
        if w.size != nrows * rw:
            raise WireError(f"key {idx}: {w.size} words, {nrows} rows of {rw} expected")
        packed = torch.from_numpy(w.view(np.int32).copy()).to(s.device)
        b = torch.empty((nrows, s.n), dtype=torch.int64, device=s.device)
        a = L.KskUnpackArgs(b.data_ptr(), packed.data_ptr(), rw, nrows, bits)
        L.check(tab.ksk_unpack(C.cast(C.pointer(a), C.c_void_p), s._stream()), "ksk_unpack")
        seed = np.asarray(e["seed"], np.uint32)
        L.check(L.lib().pcb_key_load(s.ctx, idx, _galois(s, e), C.c_void_p(b.data_ptr()), _p(seed), s._stream()),
                "pcb_key_load")
    s.galois = [_galois(s, e) for e in h["entries"]]
