"""The attention decode step on the oracle (no GPU): decrypt(attend(enc(Q), enc(K), enc(V))) matches fp64 attention
with the same degree-7 polynomial softmax within 1e-3 (BASELINE config 1 shapes, smaller ring to keep it fast)."""
import numpy as np

from perseus_b200 import attention as A
from perseus_b200 import fhe
from tests import _oracle as O
from tests._oracle_ops import OracleOps


def test_attention_decode_on_oracle():
    ch = fhe.Chain(12, tuple(fhe.ntt_primes(50, 12, 8)), tuple(fhe.ntt_primes(60, 12, 1)), 8)
    lay = A.Layout(head_dim=64, tokens=32, slots=ch.n // 2)
    gal = [1] + sorted({fhe.rotation_galois(s, ch.log_n) for s in lay.rot_steps()} - {1}, key=lambda g: g)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(0, 192, 3.2, gal)
    ops = OracleOps(o)
    rng = np.random.default_rng(0)
    q, K, V = rng.normal(0, 1, 64) / 8, rng.normal(0, 1, (32, 64)) / 8, rng.normal(0, 1, (32, 64)) / 8
    coeffs = A.softmax_poly(32)
    top = len(ch.q) - 1
    cache = A.KVCache(ops, lay, top)
    cache.load(K, V)
    qc = A.encrypt_query(ops, q, lay, top, ch.q[top])
    out = A.attend(ops, qc, cache, coeffs, ch.q)
    got = ops.decrypt_slots(out).real[:64]
    want = A.plain_attention(q, K, V, coeffs)
    assert out.top == top - 6
    assert np.abs(got - want).max() < 1e-3, np.abs(got - want).max()
    # the polynomial stands in for softmax: close to the true softmax attention for these small scores
    s = K @ q / 8
    w = np.exp(s) / np.exp(s).sum()
    assert np.abs(want - w @ V).max() < 5e-3


def test_softmax_poly_accuracy():
    c = A.softmax_poly(32)
    x = np.linspace(-1, 1, 201)
    assert np.abs(A.poly_eval(c, x) - np.exp(x) / 32).max() < 1e-6
