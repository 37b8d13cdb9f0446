"""Sessions whose switching keys are stored as `b` + seed, `a` regenerated inside every inner product (the reference's
Regen key source, crates/pc-gpu/src/ks.rs:57 and :1315-1400), against sessions with dense keys and the oracle.

The same seed gives the same keys, so every result must be the same words: relinearization and single rotations
(dot_all / dot_all_f), hoisted rotations in groups of up to four keys (dot_keys_f), rotate_sum in the extended basis
(dot_sum_f for batches, dot_sum1_f for one ciphertext), the radix ladder and the BSGS linear transform — on the FP64
chains of config 2 (N = 2^16) and of N = 2^14, and on config 1's integer chain (a 60-bit special prime).
"""
import numpy as np
import pytest
import torch

from perseus_b200 import fhe
from tests import _oracle as O

pytestmark = pytest.mark.gpu

SEED, H, SIGMA = 5, 192, 3.2


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


def chain(which):
    if which == "config2":
        return fhe.config2_chain()
    if which == "fp64_14":
        return fhe.Chain(14, tuple(fhe.ntt_primes(50, 14, 8)), tuple(fhe.ntt_primes(50, 14, 2, skip=8)), 4)
    return fhe.config1_chain()


STEPS = (1, 3, 5, 7, 2, 4, 6, -1)  # every step the radix-3 ladder over gaps 1, 2, 4 needs


@pytest.fixture(scope="module", params=["config2", "fp64_14", "config1"])
def pair(request):
    ch = chain(request.param)
    k_max = 3
    dense = fhe.Session(ch, rot_steps=STEPS, k_max=k_max, seed=SEED, h=H, sigma=SIGMA)
    regen = fhe.Session(ch, rot_steps=STEPS, k_max=k_max, seed=SEED, h=H, sigma=SIGMA, key_source="regen")
    return request.param, dense, regen


def same(x, y, top):
    return torch.equal(x.data[:, :, : top + 1], y.data[:, :, : top + 1])


def test_regen_keys_are_the_dense_keys_and_half_the_arena(pair):
    which, dense, regen = pair
    assert regen.arena.numel() < dense.arena.numel()
    key_words = len(dense.galois) * dense.chain.dnum * dense.rows * dense.n * 8
    assert dense.arena.numel() - regen.arena.numel() >= key_words  # every key's `a` is gone from the arena
    for idx in range(len(dense.galois)):
        b, a = dense.key_tensors(idx)
        rb, ra = regen.key_tensors(idx)  # `a` expanded from the seed
        assert torch.equal(b, rb) and torch.equal(a, ra), idx
        assert regen.key(idx)[1] in (None, 0)  # no stored `a`


def _enc(s, rng, top, k=1):
    cts = [s.encrypt(rng.normal(0, 1, 512) / 8, top=top) for _ in range(k)]
    return cts[0] if k == 1 else s.stack(cts)


def test_regen_ops_equal_dense(pair):
    which, dense, regen = pair
    for top in (dense.top(), dense.top() // 2):
        for k in (1, 3):
            rng1, rng2 = np.random.default_rng(top + k), np.random.default_rng(top + k)
            a, ra = _enc(dense, rng1, top, k), _enc(regen, rng2, top, k)
            b, rb = _enc(dense, rng1, top, k), _enc(regen, rng2, top, k)
            assert same(a, ra, top) and same(b, rb, top)  # the same encryptions (the same session randomness)
            assert same(dense.mult(a, b), regen.mult(ra, rb), top), (top, k, "mult")
            assert same(dense.rotate(a, 3), regen.rotate(ra, 3), top), (top, k, "rotate")
            for d, r in zip(dense.rotate_hoisted(a, STEPS), regen.rotate_hoisted(ra, STEPS)):
                assert same(d, r, top), (top, k, "hoisted")
            assert same(dense.rotate_sum(a, [1, 5, 7, 2, 3]), regen.rotate_sum(ra, [1, 5, 7, 2, 3]), top), \
                (top, k, "rotate_sum")
            assert same(dense.rotate_and_sum(a, 1, 8, radix_bits=3), regen.rotate_and_sum(ra, 1, 8, radix_bits=3),
                        top), (top, k, "radix ladder")


def test_regen_linear_transform_equals_dense(pair):
    which, dense, regen = pair
    rng = np.random.default_rng(31)
    top = dense.top()
    slots = 256
    diags = [rng.normal(0, 1, slots) for _ in range(6)]
    ld = dense.diagonals(diags, bstep=3, top=top, slots=slots)
    lr = regen.diagonals(diags, bstep=3, top=top, slots=slots)
    x = rng.normal(0, 1, slots) / 8
    a = dense.encrypt(x, top=top, slots=slots)
    ra = regen.encrypt(x, top=top, slots=slots)
    assert same(dense.linear_transform(a, ld), regen.linear_transform(ra, lr), top)


def test_regen_rotation_equals_oracle(pair):
    which, dense, regen = pair
    o = O.Ctx(regen.log_n, regen.chain.q, regen.chain.p, regen.chain.dnum)
    o.keygen(SEED, H, SIGMA, regen.galois)
    rng = np.random.default_rng(41)
    top = regen.top()
    x = rng.normal(0, 1, 512) / 8
    ct = regen.encrypt(x, top=top)
    oc = host(ct.data[0]).copy()  # the session's own encryption (its nonce has moved on past the oracle's)
    got = host(regen.rotate(ct, 5).data[0])
    want = o.rotate(oc, 5, top)
    assert (got[:, : top + 1] == want[:, : top + 1]).all()
    assert np.abs(regen.decrypt_slots(regen.rotate(ct, 5)).real[:507] - x[5:]).max() < 1e-4


def test_key_source_is_checked():
    with pytest.raises(ValueError, match="key_source"):
        fhe.Session(fhe.config1_chain(), key_source="packed")
