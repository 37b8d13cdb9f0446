"""The allocation-free rescale, pcb_rescale_static, against pcb_rescale.

Some callers cannot allocate device memory at the point where they rescale (everything they may touch was set aside
beforehand), so pcb_rescale_static keeps its working rows in a fixed array inside the library instead of the
context's workspace. Its output must be the same words as pcb_rescale's (residues are exact integers, so the
tolerance is zero) on two calls in a row — the second one sees the first one's leftovers in the shared array — and it
must refuse a chain too large for the array. This file is collected last so a failure here comes after every other
test has run.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from perseus_b200 import _lib as L
from perseus_b200 import fhe

pytestmark = pytest.mark.gpu


def _chain(which):
    if which == "config1":  # integer kernels (a 60-bit special prime)
        return fhe.config1_chain()
    if which == "fp64":  # every prime below 2^50: the FP64 transforms
        return fhe.Chain(14, tuple(fhe.ntt_primes(50, 14, 8)), tuple(fhe.ntt_primes(50, 14, 2, skip=8)), 4)
    # 48 + 16 rows at N = 2^14: 2 (nq + kp) N = 2^21 words, the array exactly full
    return fhe.Chain(14, tuple(fhe.ntt_primes(50, 14, 48)), tuple(fhe.ntt_primes(50, 14, 16, skip=48)), 3)


@pytest.fixture(scope="module", params=["config1", "fp64", "full"])
def sess(request):
    return fhe.Session(_chain(request.param), rot_steps=(), k_max=1, seed=3, h=192, sigma=3.2)


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_static_rescale_equals_rescale_twice(sess):
    s = sess
    rng = np.random.default_rng(21)
    for call in range(2):
        top = s.top() - call  # two different levels, back to back
        x, y = rng.normal(0, 1, 256) / 8, rng.normal(0, 1, 256) / 8
        a = s.drop_to(s.encrypt(x), top)
        b = s.drop_to(s.encrypt(y), top)
        m = s.mult(a, b)
        want = m.data.clone()
        got = m.data.clone()
        L.check(L.lib().pcb_rescale(s.ctx, C.c_void_p(want.data_ptr()), top, 1, _stream()), "pcb_rescale")
        L.check(L.lib().pcb_rescale_static(s.ctx, C.c_void_p(got.data_ptr()), top, _stream()), "pcb_rescale_static")
        torch.cuda.synchronize()
        assert torch.equal(got[:, :, :top], want[:, :, :top]), f"call {call}"
        r = fhe.Ct(got, top - 1, m.scale / s.chain.q[top], m.slots)
        assert np.abs(s.decrypt_slots(r).real[:256] - x * y).max() < 1e-5


def test_static_rescale_refuses_large_chains():
    ch = fhe.config2_chain()  # 2 * 32 rows * 2^16 words exceeds the 2^21-word array
    s = fhe.Session(ch, rot_steps=(), k_max=1, seed=0)
    ct = s.empty(1)
    rc = L.lib().pcb_rescale_static(s.ctx, C.c_void_p(ct.data_ptr()), s.top(), _stream())
    assert rc == -1
    assert "maximum" in L.lib().pcb_last_error().decode()
