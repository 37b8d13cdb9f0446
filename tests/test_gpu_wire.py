"""The wire format on the GPU (perseus_b200/wire.py):

- the compressed frame (pcb_ct_compress: INTT, CRT, exact rounding, packing on the device) equals the reference's
  pack_coeffs + pack_bits formula word for word, over one and two limbs at several widths, and decompresses to within
  the rounding;
- client and server: a server session without a secret loads the client's key bundle (ksk_unpack + pcb_key_load),
  both key sources; its keys equal the client's word for word; a ciphertext crosses as a frame, the server's rotation
  and relinearized product equal the client's own word for word and decrypt on the client;
- a compressed frame of a bottom-level ciphertext decrypts after the client's decompression.
"""
import numpy as np
import pytest
import torch

from perseus_b200 import _lib as L
from perseus_b200 import fhe
from perseus_b200 import wire as W
from tests import _oracle as O
from tests import _wire_ref as R

pytestmark = pytest.mark.gpu

LOGN = 14


def chain():
    return fhe.Chain(LOGN, tuple(fhe.ntt_primes(50, LOGN, 6)), tuple(fhe.ntt_primes(50, LOGN, 3, skip=6)), 2)


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


def coeff_rows(ch, ct, c, part):
    rows = np.ascontiguousarray(host(ct.data[c, part])[: ct.top + 1]).copy()
    O.lib().orc_ntt_inv(rows, ct.top + 1, np.asarray(ch.q[: ct.top + 1], np.uint64), LOGN)
    return rows


@pytest.mark.parametrize("top,bits", [(0, 1), (0, 30), (0, 50), (0, 64), (1, 12), (1, 27)])
def test_compressed_frame_matches_reference(top, bits):
    ch = chain()
    s = fhe.Session(ch, k_max=2, seed=0)
    rng = np.random.default_rng(top * 100 + bits)
    ct = s.stack([s.encrypt(rng.uniform(-1, 1, 64), top=top, scale=2.0**30) for _ in range(2)])
    frame = W.export_ct(s, ct, bits=bits)
    w = W.CtWire.from_bytes(frame)
    assert w.header.bits == bits and w.header.rows == top + 1 and w.header.k == 2
    per = W.packed_words(ch.n, bits)
    q = list(ch.q[: top + 1])
    for c in range(2):
        for part in range(2):
            rows = coeff_rows(ch, ct, c, part)
            want = R.pack_bits_ref(R.pack_coeffs_ref(q, rows, bits), bits)
            got = w.data[(2 * c + part) * per:(2 * c + part + 1) * per]
            assert [int(x) for x in got] == want, (c, part)
    # the client's decompression: every coefficient within the rounding of its CRT value
    back, h = W.decompress(s, frame)
    Q = 1
    for p in q:
        Q *= p
    rows = coeff_rows(ch, ct, 1, 1)
    x = [sum(int(rows[r][i]) * (Q // p) * pow(Q // p % p, -1, p) for r, p in enumerate(q)) % Q for i in range(64)]
    xb = [sum(int(back[1, 1, r, i]) * (Q // p) * pow(Q // p % p, -1, p) for r, p in enumerate(q)) % Q for i in range(64)]
    tol = Q // 2**bits + 1
    assert all(min((a - b) % Q, (b - a) % Q) <= tol for a, b in zip(x, xb))


@pytest.mark.parametrize("key_source", ["dense", "regen"])
def test_client_server_roundtrip(key_source):
    ch = chain()
    steps = [1, 3]
    client = fhe.Session(ch, rot_steps=steps, k_max=1, seed=5, key_source=key_source)
    server = fhe.Session(ch, rot_steps=steps, k_max=1, key_source=key_source, keygen=False)
    bundle = W.export_keys(client)
    W.import_keys(server, bundle)
    assert server.galois == client.galois
    for idx in range(len(client.galois)):
        for a, b in zip(client.key_tensors(idx), server.key_tensors(idx)):
            assert torch.equal(a, b), idx
    rng = np.random.default_rng(9)
    z = rng.uniform(-1, 1, 64)
    ct = client.encrypt(z, top=ch.rows - len(ch.p) - 1, scale=2.0**40)
    x = W.import_ct(server, W.export_ct(client, ct))
    assert torch.equal(x.data[:, :, : x.top + 1], ct.data[:, :, : ct.top + 1])
    for op in (lambda s_, c_: s_.rotate(c_, 3), lambda s_, c_: s_.rescale_one(s_.mult(c_, c_))):
        y_server = op(server, x)
        y_client = op(client, ct)
        back = W.import_ct(client, W.export_ct(server, y_server))
        assert back.top == y_client.top and back.scale == y_client.scale
        assert torch.equal(back.data[:, :, : back.top + 1], y_client.data[:, :, : y_client.top + 1])
    got = client.decrypt_slots(W.import_ct(client, W.export_ct(server, server.rotate(x, 3)))).real[:64]
    assert np.abs(got - np.roll(z, -3)).max() < 1e-5
    # a corrupted bundle is refused
    bad = bytearray(bundle)
    bad[-100] ^= 1
    with pytest.raises(W.WireError, match="checksum"):
        W.import_keys(server, bytes(bad))


def test_compressed_bottom_level_decrypts():
    ch = chain()
    s = fhe.Session(ch, k_max=1, seed=2)
    z = np.random.default_rng(4).uniform(-1, 1, 64)
    ct = s.encrypt(z, top=0, scale=2.0**40)
    back, h = W.decompress(s, W.export_ct(s, ct, bits=32))
    buf = torch.zeros((2 * s.nq, s.n), dtype=torch.int64, device=s.device)
    buf[0] = torch.from_numpy(back[0, 0, 0].view(np.int64))
    buf[s.nq] = torch.from_numpy(back[0, 1, 0].view(np.int64))
    s.ntt_batch(buf, 2 * s.nq)  # row r under prime r mod nq: rows 0 and nq under q_0
    x = s.empty(1)
    x[0, 0, 0] = buf[0]
    x[0, 1, 0] = buf[s.nq]
    got = s.decrypt_slots(fhe.Ct(x, 0, h.meta["nf"], h.meta["slots"])).real[:64]
    # rounding to q_0 / 2^33 per coefficient, times the secret's weight: about 2^17 2^8 against the scale 2^40
    assert np.abs(got - z).max() < 1e-3
