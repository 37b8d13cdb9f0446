"""CKKS bootstrapping on the CUDA path (perseus_b200/bootstrap.py over the session's ops: ModRaise, CoeffToSlot,
conjugation, EvalMod, SlotToCoeff):

- at N = 2^14 (8192 slots, 20 + 5 limbs) the refreshed ciphertext equals the oracle's word for word, both run on the
  same level-0 ciphertext with the same keys, and decrypts to the input slots;
- BASELINE config 4 at its size: N = 2^16 with full slots (2^15), uniform [-1, 1] slot values (seeded) at level 0,
  refreshed to 12 usable levels (29 + 11 limbs of 50 bits, secret of Hamming weight 192), decrypting within 1e-3
  absolute of the input slots; one product of the refreshed ciphertext with itself within 1e-3 of z^2.
"""
import os

import numpy as np
import pytest
import torch

from perseus_b200 import bootstrap as BS
from perseus_b200 import fhe
from tests import _oracle as O
from tests._oracle_ops import OCt, OracleOps

pytestmark = pytest.mark.gpu


def host(t):
    return t.detach().cpu().numpy().view(np.uint64)


def session(ch, prm, h):
    s = fhe.Session(ch, rot_steps=BS.rot_steps(prm), k_max=2, seed=0, h=h, sigma=3.2,
                    galois_extra=(BS.conj_galois(ch.n),))
    return ch, s


def test_bootstrap_bit_exact_with_the_oracle():
    logn = 14
    prm = BS.Params(1 << logn, K=24, r=3, per_group=5)
    ch = fhe.Chain(logn, tuple(fhe.ntt_primes(50, logn, 20)), tuple(fhe.ntt_primes(50, logn, 6, skip=20)), 4)
    ch, s = session(ch, prm, h=64)
    O.lib().orc_set_threads(os.cpu_count() or 1)
    o = O.Ctx(ch.log_n, ch.q, ch.p, ch.dnum)
    o.keygen(0, 64, 3.2, s.galois)
    oo = OracleOps(o)
    rng = np.random.default_rng(40)
    z = rng.uniform(-1, 1, prm.slots)
    ct = s.encrypt(z, top=0, scale=2.0**40, slots=prm.slots)
    oc = OCt(host(ct.data[0]).copy(), 0, ct.scale, ct.slots)
    top = len(ch.q) - 1
    out = BS.Bootstrapper(s, prm, ch.q, ch.q[0])(ct, top)
    oout = BS.Bootstrapper(oo, prm, ch.q, ch.q[0])(oc, top)
    torch.cuda.synchronize()
    oout = oout.cts[0] if hasattr(oout, "cts") else oout
    assert out.top == oout.top == top - 16
    assert (host(out.data[0])[:, : out.top + 1] == oout.data[:, : out.top + 1]).all()
    got = s.decrypt_slots(out)
    assert np.abs(got.real - z).max() < 1e-4


def test_bootstrap_config4():
    logn = 16
    prm = BS.Params(1 << logn, K=24, r=3, per_group=5)
    ch, s = session(fhe.config4_chain(), prm, h=192)
    rng = np.random.default_rng(4)
    z = rng.uniform(-1, 1, prm.slots)
    ct = s.encrypt(z, top=0, scale=2.0**40, slots=prm.slots)
    bt = BS.Bootstrapper(s, prm, ch.q, ch.q[0])
    out = bt(ct, len(ch.q) - 1)
    assert out.top == 12  # 12 usable levels above the bottom limb
    again = bt(ct, len(ch.q) - 1)  # the input is left as it was; the refresh is deterministic
    assert ct.top == 0 and torch.equal(again.data[:, :, : out.top + 1], out.data[:, :, : out.top + 1])
    got = s.decrypt_slots(out)
    assert np.abs(got.real - z).max() < 1e-3 and np.abs(got.imag).max() < 1e-3
    sq = s.rescale_one(s.mult(out, out))
    assert np.abs(s.decrypt_slots(sq).real - z * z).max() < 1e-3
