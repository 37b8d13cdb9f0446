"""perseus-b200: a B200-native (sm_100a) CKKS encrypted-attention hot path with the reference's C ABI.

The compute path is perseus_b200/libpcb200.so (built in-tree by perseus_b200/build.py); this package holds the
Python side of the evaluator API (fhe.Session, mirroring the reference's Fhe) and the attention driver.
"""
from .fhe import Chain, Ct, Fhe, Session, config1_chain, config2_chain, ntt_primes, rotation_galois  # noqa: F401
