"""BSGS ciphertext x plaintext matmul, host side and oracle (no GPU):
the packing and the pre-rotated diagonals reproduce X W in the clear, the
work partition covers every baby and giant step exactly once, the oracle's
encrypted product decodes to X W, and partial products over giant-step
ranges add up (mod q) to the same product.  The giant steps of one call
share one ModDown, so a split into ranges rounds once per range: the sum of
the parts decodes to X W like the whole call, without being the same words."""
import numpy as np
import pytest

from comp390project_b200 import matmul
from tests.matmul_case import case, decode_outputs


def _rot(v, k):
    """CKKS left rotation of a slot vector: out[j] = v[(j + k) mod S]."""
    return np.roll(v, -k)


@pytest.mark.parametrize("shape", [(4096, 64, 128, 128), (32768, 128, 768, 768),
                                   (1024, 16, 64, 192)])
def test_bsgs_identity_in_the_clear(shape):
    slots, T, d_in, d_out = shape
    lay = matmul.layout(slots, T, d_in, d_out)
    assert lay.n_baby * lay.n_giant == lay.feats
    rng = np.random.default_rng(7)
    X = rng.normal(size=(T, d_in))
    W = rng.normal(size=(d_in, d_out))
    xs = matmul.pack(X, lay)
    assert np.array_equal(matmul.unpack(xs, lay.__class__(**{**lay.__dict__, "n_out": lay.n_in})), X)
    if slots > 8192:
        return  # packing only: the full config-5 diagonals take ~600 MB
    d = matmul.diagonals(W, lay).reshape(lay.n_out, lay.n_in, lay.n_giant, lay.n_baby, slots)
    B, u = lay.n_baby, lay.unit
    ys = []
    for o in range(lay.n_out):
        acc = np.zeros(slots)
        for g in range(lay.n_giant):
            inner = sum(d[o, i, g, b] * _rot(xs[i], b * u)
                        for i in range(lay.n_in) for b in range(B))
            acc += _rot(inner, g * B * u)
        ys.append(acc)
    assert np.allclose(matmul.unpack(np.array(ys), lay), X @ W, atol=1e-9)


def test_config5_layout():
    lay = matmul.layout(1 << 15, 128, 768, 768)
    assert (lay.feats, lay.n_in, lay.n_out, lay.unit, lay.n_baby, lay.n_giant) == \
        (256, 3, 3, 128, 16, 16)
    assert lay.n_diagonals == 2304
    # 45 hoisted baby-step rotations + 45 giant-step rotations per layer
    assert lay.n_in * len(lay.baby_steps()) + lay.n_out * len(lay.giant_steps()) == 90


def test_layout_rejects_bad_shapes():
    with pytest.raises(ValueError):
        matmul.layout(4096, 48, 128, 128)       # 4096 / 48 not an integer
    with pytest.raises(ValueError):
        matmul.layout(4096, 64, 100, 128)       # d_in not a multiple of F
    with pytest.raises(ValueError):
        matmul.layout(4096, 64, 128, 128, n_baby=3)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8, 20])
def test_partition_covers_every_step_once(world):
    lay = matmul.layout(1 << 15, 128, 768, 768)
    gr = matmul.giant_ranges(lay.n_giant, world)
    assert gr[0][0] == 0 and gr[-1][1] == lay.n_giant
    assert all(a[1] == b[0] for a, b in zip(gr, gr[1:]))
    sizes = [hi - lo for lo, hi in gr]
    assert max(sizes) - min(sizes) <= 1
    pairs = [p for r in range(world) for p in matmul.baby_assignment(lay, world, r)]
    want = [(i, b) for i in range(lay.n_in) for b in range(1, lay.n_baby)]
    assert pairs == want
    c = matmul.baby_chunk(lay, world)
    assert all(len(matmul.baby_assignment(lay, world, r)) <= c for r in range(world))


def test_sum_bound():
    matmul.check_sum_fits((1 << 60) - 1, 8)
    with pytest.raises(ValueError):
        matmul.check_sum_fits((1 << 61) - 1, 8)


@pytest.mark.parametrize("n_baby", [None, 64])
def test_oracle_bsgs_matmul_decodes_to_product(n_baby):
    c = case(n_baby)
    o, lay = c["o"], c["lay"]
    ys = o.bsgs_matmul(c["xs"], c["Ql"], lay.unit, lay.n_baby, lay.n_giant, c["pts"], c["keys"])
    Y = decode_outputs(c, ys)
    ref = c["X"] @ c["W"]
    assert np.abs(Y - ref).max() < 1e-4, np.abs(Y - ref).max()
    # and after a rescale by the last prime
    y2 = o.rescale(ys[0], c["Ql"])
    v = o.decode(o.decrypt(c["s"], y2, c["Ql"] - 1), c["Ql"] - 1,
                 2.0 ** 80 / float(o.moduli[c["Ql"] - 1]))
    col = np.real(v).reshape(lay.feats, lay.tokens).T
    assert np.abs(col - ref[:, :lay.feats]).max() < 1e-4


def test_oracle_partial_products_add_up():
    c = case()
    o, lay, Ql = c["o"], c["lay"], c["Ql"]
    args = (c["xs"], Ql, lay.unit, lay.n_baby, lay.n_giant, c["pts"], c["keys"])
    full = o.bsgs_matmul(*args)
    parts = [o.bsgs_matmul(*args, g_range=r) for r in matmul.giant_ranges(lay.n_giant, 3)]
    q = np.array([int(o.moduli[j]) for j in range(Ql)], dtype=np.uint64)[None, None, :, None]
    acc = np.zeros_like(full)
    for p in parts:
        acc = (acc + p) % q
    ref = c["X"] @ c["W"]
    for y in (full, acc):
        assert np.abs(decode_outputs(c, y) - ref).max() < 1e-4
    # each part's rounding is its own ModDown's: the sum differs from the
    # whole call, which rounds once
    assert not np.array_equal(acc, full)


def test_bsgs_identity_for_random_shapes():
    """Property: for any power-of-two packing the pre-rotated diagonals and the
    BSGS formula reproduce X W in the clear (slots 64..1024, any B dividing F)."""
    from hypothesis import given, settings, strategies as st

    @settings(max_examples=40, deadline=None)
    @given(log_s=st.integers(6, 10), log_t=st.integers(0, 4), n_in=st.integers(1, 3),
           n_out=st.integers(1, 3), log_b=st.integers(0, 6), seed=st.integers(0, 2 ** 31))
    def check(log_s, log_t, n_in, n_out, log_b, seed):
        slots, T = 1 << log_s, 1 << log_t
        F = slots // T
        B = 1 << min(log_b, F.bit_length() - 1)
        lay = matmul.layout(slots, T, n_in * F, n_out * F, n_baby=B)
        rng = np.random.default_rng(seed)
        X = rng.normal(size=(T, n_in * F))
        W = rng.normal(size=(n_in * F, n_out * F))
        xs = matmul.pack(X, lay)
        d = matmul.diagonals(W, lay).reshape(n_out, n_in, lay.n_giant, B, slots)
        ys = []
        for o in range(n_out):
            acc = np.zeros(slots)
            for g in range(lay.n_giant):
                inner = sum(d[o, i, g, b] * _rot(xs[i], b * lay.unit)
                            for i in range(n_in) for b in range(B))
                acc = acc + _rot(inner, g * B * lay.unit)
            ys.append(acc)
        assert np.allclose(matmul.unpack(np.array(ys), lay), X @ W, atol=1e-8)

    check()
