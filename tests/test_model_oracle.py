"""The multi-layer encrypted decode (perseus_b200/model.py: LayerNorm, attention over the layer's cache, MLP with the
polynomial GELU, residuals, a refresh before every stage that needs more levels than are left) on the oracle at a
small ring: two layers, two tokens decoded one after the other (the second reads the first's pushed K and V rows),
each decrypted within 1e-3 of the fp64 decode with the same polynomials."""
import numpy as np
import pytest

from perseus_b200 import attention as A
from perseus_b200 import bootstrap as BS
from perseus_b200 import fhe
from perseus_b200 import linear as LIN
from perseus_b200 import model as M
from tests import _oracle as O
from tests._oracle_ops import OracleOps

LOGN = 10
N = 1 << LOGN


@pytest.fixture(scope="module")
def setup():
    # 24 real elements in a 32-wide layout, the MLP's 64 hidden units in two full blocks of 32 (GPT-2's proportions)
    cfg = M.ModelCfg(layers=2, d=24, width=32, heads=3, head_dim=8, mlp=64, tokens=32, radix_bits=2)
    prm = BS.Params(N, K=24, r=3, per_group=5)
    q = O.ntt_primes(50, LOGN, 25)  # a refresh spends 14 levels and leaves top 10
    p = O.ntt_primes(50, LOGN, 6, skip=25)  # P one prime larger than a digit of 5
    lay = M.B.layout(N // 2, cfg.width, cfg.heads, cfg.head_dim, cfg.tokens, cfg.radix_bits)
    steps = sorted(set(BS.rot_steps(prm)) | set(lay.rot_steps()))
    gal = list(dict.fromkeys([1] + [fhe.rotation_galois(s, LOGN) for s in steps] + [BS.conj_galois(N)]))
    O.lib().orc_set_threads(8)
    c = O.Ctx(LOGN, q, p, 5)
    c.keygen(seed=0, h=64, sigma=3.2, galois=gal)
    return cfg, prm, c


def test_two_layer_decode_matches_fp64(setup):
    cfg, prm, c = setup
    ops = OracleOps(c)
    rng = np.random.default_rng(50)
    weights = [M.random_layer(rng, d=cfg.d, mlp=cfg.mlp, std=0.1) for _ in range(cfg.layers)]
    pre = 20
    Ks = [rng.normal(0, 1, (pre, cfg.d)) / 8 for _ in range(cfg.layers)]
    Vs = [rng.normal(0, 1, (pre, cfg.d)) / 8 for _ in range(cfg.layers)]
    bt = BS.Bootstrapper(ops, prm, c.q, c.q[0])
    dec = M.Decoder(ops, cfg, weights, c.q, bt)
    assert (dec.out_top, dec.cache_top) == (10, 8)
    dec.load(Ks, Vs)
    plain = [[K.copy(), V.copy()] for K, V in zip(Ks, Vs)]
    for tok in range(2):
        x = rng.normal(0, 1, cfg.d)
        xc = ops.encrypt(LIN.input_vector(x, dec.lay.geo), 0, 2.0**40, dec.lay.slots)
        y = dec.decode(xc)
        want = M.plain_decode(x, weights, plain, cfg, dec.coeffs)
        got = LIN.output_values(ops.decrypt_slots(y).real, dec.lay.geo, cfg.d)
        assert np.abs(got - want).max() < 1e-3, (tok, np.abs(got - want).max())
        assert all(cc.count == pre + tok + 1 for cc in dec.caches)


def test_gelu_poly_and_levels():
    cfg = M.ModelCfg()
    u = np.linspace(-1, 1, 1001)
    assert np.abs(A.poly_eval(M.gelu_poly(cfg.gelu_bound), u) - M.gelu(cfg.gelu_bound * u)).max() < 0.015
    # config 4's chain: a refresh spends 16 levels and leaves 12, the attention stage's 10 fit
    ch = fhe.config4_chain()
    assert len(ch.q) - 1 - (3 + 7 + 3 + 3) == 12


def test_two_sequences_decode_together(setup):
    """seqs = 2: one step decodes both sequences' tokens (every op on their batch, refreshes included); each output
    matches its own fp64 decode, and each sequence's caches grow by its own token."""
    cfg, prm, c = setup
    cfg = M.ModelCfg(layers=1, d=cfg.d, width=cfg.width, heads=cfg.heads, head_dim=cfg.head_dim, mlp=cfg.mlp,
                     tokens=cfg.tokens, radix_bits=cfg.radix_bits)
    ops = OracleOps(c)
    rng = np.random.default_rng(51)
    weights = [M.random_layer(rng, d=cfg.d, mlp=cfg.mlp, std=0.1)]
    pre, S = 10, 2
    Ks = [[rng.normal(0, 1, (pre, cfg.d)) / 8 for _ in range(S)]]
    Vs = [[rng.normal(0, 1, (pre, cfg.d)) / 8 for _ in range(S)]]
    dec = M.Decoder(ops, cfg, weights, c.q, BS.Bootstrapper(ops, prm, c.q, c.q[0]), seqs=S)
    dec.load(Ks, Vs)
    xs = [rng.normal(0, 1, cfg.d) for _ in range(S)]
    xc = ops.stack([ops.encrypt(LIN.input_vector(x, dec.lay.geo), 0, 2.0**40, dec.lay.slots) for x in xs])
    y = dec.decode(xc)
    for q in range(S):
        want = M.plain_decode(xs[q], weights, [[Ks[0][q].copy(), Vs[0][q].copy()]], cfg, dec.coeffs)
        got = LIN.output_values(ops.decrypt_slots(y, q).real, dec.lay.geo, cfg.d)
        assert np.abs(got - want).max() < 1e-3, q
