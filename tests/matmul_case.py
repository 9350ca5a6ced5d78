"""A small BERT-shaped matmul case for the BSGS tests: the SMALL ring
(N=2^12, 2048 slots, Q = 50 + 6 x 40 bits, P = 3 x 55 bits, three digits),
T=32 tokens, F=64 features per ciphertext, d_in = d_out = 128 (two input and
two output ciphertexts), B = G = 8 by default.  Activations N(0,1) and
weights N(0,0.02) from seed 4, as config 5 draws them; the diagonals are
encoded by the oracle at scale 2^40."""
import functools

import numpy as np

from comp390project_b200 import matmul
from tests.ksparams import SMALL, oracle_for

SCALE = 2.0 ** 40
TOKENS, D_IN, D_OUT = 32, 128, 128


@functools.lru_cache(maxsize=None)
def case(n_baby=None):
    """n_baby=None: B = G = 8; n_baby=64: G = 1 and 128 plaintext terms per
    output (more than one pass of the product kernel)."""
    o = oracle_for("small")
    lay = matmul.layout(o.N // 2, TOKENS, D_IN, D_OUT, n_baby=n_baby)
    rng = np.random.default_rng(4)
    X = rng.normal(0.0, 1.0, (TOKENS, D_IN))
    W = rng.normal(0.0, 0.02, (D_IN, D_OUT))
    s = o.secret(4)
    Ql = len(SMALL["qbits"])
    xs = [o.encrypt(s, o.encode(v, SCALE, Ql), Ql, 40 + i)
          for i, v in enumerate(matmul.pack(X, lay))]
    pts = [o.encode(d, SCALE, Ql) for d in matmul.diagonals(W, lay)]
    keys = {st: o.keygen_galois(s, o.galois_elt(st), 500 + k)
            for k, st in enumerate(lay.baby_steps() + lay.giant_steps())}
    return dict(o=o, lay=lay, X=X, W=W, s=s, Ql=Ql, xs=xs, pts=pts, keys=keys)


def decode_outputs(c, ys):
    """Decrypt, rescale-free decode of y [n_out][2][Ql][N] at scale 2^80."""
    o, lay, Ql = c["o"], c["lay"], c["Ql"]
    vecs = [o.decode(o.decrypt(c["s"], y, Ql), Ql, SCALE * SCALE) for y in ys]
    return matmul.unpack(np.real(np.array(vecs)), lay)


def split_reference(c, world):
    """The oracle's product summed over the giant-step ranges of `world`
    ranks (matmul.giant_ranges), each range evaluated by one call (one
    ModDown per range), as matmul_giant_parallel computes it."""
    o, lay, Ql = c["o"], c["lay"], c["Ql"]
    args = (c["xs"], Ql, lay.unit, lay.n_baby, lay.n_giant, c["pts"], c["keys"])
    q = np.array([int(o.moduli[j]) for j in range(Ql)], dtype=np.uint64)[None, None, :, None]
    acc = None
    for r in matmul.giant_ranges(lay.n_giant, world):
        if r[1] <= r[0]:
            continue
        p = o.bsgs_matmul(*args, g_range=r)
        acc = p if acc is None else (acc + p) % q
    return acc
