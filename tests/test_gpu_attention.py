"""The encrypted attention decode step on the CUDA path vs the oracle (N = 2^14, 8 x 50-bit
limbs + one 60-bit special prime, head_dim 64, 32 cached tokens, degree-7 polynomial softmax, seed 0): the output
ciphertext bit-exact on every residue, its decryption within 1e-3 of fp64 attention."""
import numpy as np
import pytest
import torch

from perseus_b200 import attention as A
from perseus_b200 import fhe
from tests import _oracle as O
from tests._oracle_ops import OracleOps

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair():
    ch = fhe.config1_chain()
    lay = A.Layout(head_dim=64, tokens=32, slots=ch.n // 2)
    s = fhe.Session(ch, rot_steps=lay.rot_steps(), k_max=1, seed=0, h=192, sigma=3.2)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(0, 192, 3.2, s.galois)
    return ch, lay, s, OracleOps(o)


def run(ops, ch, lay, q, K, V, push):
    top = len(ch.q) - 1
    cache = A.KVCache(ops, lay, top)
    if push:
        for t in range(K.shape[0]):
            cache.push(K[t], V[t])
    else:
        cache.load(K, V)
    qc = A.encrypt_query(ops, q, lay, top, ch.q[top])
    return A.attend(ops, qc, cache, A.softmax_poly(lay.tokens), ch.q)


@pytest.mark.parametrize("push", [False, True])
def test_attention_decode_bit_exact(pair, push):
    ch, lay, s, oo = pair
    rng = np.random.default_rng(7 + push)
    n = 32 if not push else 5  # a partly filled cache when pushing token by token
    q, K, V = rng.normal(0, 1, 64) / 8, rng.normal(0, 1, (n, 64)) / 8, rng.normal(0, 1, (n, 64)) / 8
    g = run(s, ch, lay, q, K, V, push)
    want_ct = run(oo, ch, lay, q, K, V, push)
    torch.cuda.synchronize()
    assert g.top == want_ct.top == len(ch.q) - 7
    gh = g.data[0].cpu().numpy().view(np.uint64)
    assert (gh[:, : g.top + 1] == want_ct.data[:, : g.top + 1]).all()
    got = s.decrypt_slots(g).real[:64]
    want = A.plain_attention(q, K, V, A.softmax_poly(lay.tokens))
    assert np.abs(got - want).max() < 1e-3


def test_decode_graph_replays_eager_step(pair):
    """The captured decode step gives, token after token, the eager step's ciphertext word for word."""
    ch, lay, s, oo = pair
    rng = np.random.default_rng(21)
    top = len(ch.q) - 1
    cache = A.KVCache(s, lay, top)
    cache.load(rng.normal(0, 1, (lay.tokens, 64)) / 8, rng.normal(0, 1, (lay.tokens, 64)) / 8)
    coeffs = A.softmax_poly(lay.tokens)
    qs = [A.encrypt_query(s, rng.normal(0, 1, 64) / 8, lay, top, ch.q[top]) for _ in range(3)]
    g = A.DecodeGraph(s, cache, coeffs, ch.q, qs[0])
    for q in qs:
        got = g(q).data.clone()
        want = A.attend(s, q, cache, coeffs, ch.q)
        assert torch.equal(got[:, :, : want.top + 1], want.data[:, :, : want.top + 1])


@pytest.fixture(scope="module")
def pair3():
    """Config 1 with the radix ladder (groups of 3 gaps summed by rotate_sum; 38 rotation keys)."""
    ch = fhe.config1_chain()
    lay = A.Layout(head_dim=64, tokens=32, slots=ch.n // 2, radix_bits=3)
    s = fhe.Session(ch, rot_steps=lay.rot_steps(), k_max=1, seed=0, h=192, sigma=3.2)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(0, 192, 3.2, s.galois)
    return ch, lay, s, OracleOps(o)


def test_attention_decode_radix_bit_exact(pair3):
    """The decode step with radix-3 ladders, the CUDA path against the oracle word for word, and replayed as a graph."""
    ch, lay, s, oo = pair3
    rng = np.random.default_rng(31)
    q, K, V = rng.normal(0, 1, 64) / 8, rng.normal(0, 1, (32, 64)) / 8, rng.normal(0, 1, (32, 64)) / 8
    g = run(s, ch, lay, q, K, V, False)
    want_ct = run(oo, ch, lay, q, K, V, False)
    torch.cuda.synchronize()
    gh = g.data[0].cpu().numpy().view(np.uint64)
    assert (gh[:, : g.top + 1] == want_ct.data[:, : g.top + 1]).all()
    got = s.decrypt_slots(g).real[:64]
    assert np.abs(got - A.plain_attention(q, K, V, A.softmax_poly(lay.tokens))).max() < 1e-3
    top = len(ch.q) - 1
    cache = A.KVCache(s, lay, top)
    cache.load(K, V)
    qc = A.encrypt_query(s, q, lay, top, ch.q[top])
    graph = A.DecodeGraph(s, cache, A.softmax_poly(lay.tokens), ch.q, qc)
    eager = A.attend(s, qc, cache, A.softmax_poly(lay.tokens), ch.q)
    assert torch.equal(graph(qc).data[:, :, : eager.top + 1], eager.data[:, :, : eager.top + 1])
