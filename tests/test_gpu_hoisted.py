"""Hoisted rotations and the hoisted linear transform through the C ABI
(ks_rotate_hoisted, ks_linear_transform_hoisted): one ModUp of c1 shared by
all rotations, the extended digits permuted inside the inner product.  The
rotations must equal the CPU oracle's hoisting (ork_rotate_hoisted: ModUp,
then the automorphism of every extended limb) word for word; the linear
transform (one ModDown for all rotations) must equal the oracle's
ork_linear_transform_hoisted word for word and decode to
sum_i diag_i * roll(z, step_i) within the reference's 1e-3 MAE."""
import numpy as np
import pytest

from tests.ksparams import SMALL, oracle_for, split

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

STEPS = [1, 2, 5, 7, 16]


def _ctx(o, s, steps, max_batch=4):
    from comp390project_b200 import KS_KEY_GALOIS, KsContext
    log_n, q, p = split(SMALL)
    ctx = KsContext(log_n, q, p, device=0, max_batch=max_batch)
    keys = {}
    for st in steps:
        e = o.galois_elt(st)
        keys[st] = o.keygen_galois(s, e, 70 + st)
        ctx.key_upload(KS_KEY_GALOIS, e, keys[st])
    return ctx, keys


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64).copy()).cuda()


def _host(t):
    return t.cpu().numpy().view(np.uint64)


@pytest.mark.parametrize("drop", [0, 2])
def test_rotate_hoisted_matches_oracle(drop, cuda_device):
    o = oracle_for("small")
    s = o.secret(3, 64)
    ctx, keys = _ctx(o, s, STEPS)
    Ql = o.L - drop
    rng = np.random.default_rng(5 + drop)
    ct = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                             for j in range(Ql)]) for _ in range(2)])
    d = _dev(ct)
    outs = [torch.zeros_like(d) for _ in STEPS]
    ctx.rotate_hoisted(d, Ql, STEPS, outs)
    torch.cuda.synchronize()
    want = o.rotate_hoisted(ct, Ql, [o.galois_elt(st) for st in STEPS], [keys[st] for st in STEPS])
    assert np.array_equal(_host(d), ct), "input modified"
    for i, out in enumerate(outs):
        assert np.array_equal(_host(out), want[i]), "rotation %d differs" % STEPS[i]
    ctx.close()


def _ext_basis(o, Ql):
    return list(range(Ql)) + [o.L + i for i in range(o.alpha)]


@pytest.mark.parametrize("drop", [0, 3])
def test_linear_transform_hoisted_matches_oracle(drop, cuda_device):
    o = oracle_for("small")
    s = o.secret(4, 64)
    ctx, keys = _ctx(o, s, STEPS)
    Ql = o.L - drop
    rng = np.random.default_rng(11 + drop)
    ct = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                             for j in range(Ql)]) for _ in range(2)])
    diags = [np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                       for j in _ext_basis(o, Ql)]) for _ in STEPS]
    d = _dev(ct)
    out = torch.zeros_like(d)
    ctx.linear_transform_hoisted(d, Ql, STEPS, [_dev(x) for x in diags], out)
    torch.cuda.synchronize()
    want = o.linear_transform_hoisted(ct, Ql, [o.galois_elt(st) for st in STEPS],
                                      [keys[st] for st in STEPS], diags)
    assert np.array_equal(_host(out), want)
    ctx.close()


def test_linear_transform_hoisted_decodes(cuda_device):
    o = oracle_for("small")
    s = o.secret(6, 64)
    ctx, keys = _ctx(o, s, STEPS)
    Ql = o.L
    n = o.N // 2
    rng = np.random.default_rng(3)
    z = rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)
    ct = o.encrypt(s, o.encode(z, 2.0 ** 40, Ql), Ql, 17)
    dz = [rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n) for _ in STEPS]
    diags = [o.encode_basis(x, 2.0 ** 40, _ext_basis(o, Ql)) for x in dz]
    out = torch.zeros((2, Ql, o.N), dtype=torch.int64, device="cuda")
    ctx.linear_transform_hoisted(_dev(ct), Ql, STEPS, [_dev(x) for x in diags], out)
    torch.cuda.synchronize()
    dec = o.decode(o.decrypt(s, _host(out), Ql), Ql, 2.0 ** 80)
    want = sum(x * np.roll(z, -st) for x, st in zip(dz, STEPS))
    assert np.abs(dec - want).mean() < 1e-3
    ctx.close()


def test_config4_hoisted_bitexact(cuda_device):
    """Config 4's ring (N = 2^16, alpha = 5) at level 24 (Ql = 25, five full
    digits): hoisted rotations and the hoisted linear transform over baby and
    giant steps, word for word against the oracle."""
    from comp390project_b200 import KS_KEY_GALOIS, KsContext
    from tests.ksparams import CFG3
    o = oracle_for("cfg3")
    log_n, q, p = split(CFG3)
    ctx = KsContext(log_n, q, p, device=0, max_batch=2)
    s = o.secret(7, 192)
    steps = [1, 5, 32, 64]
    keys = {}
    for st in steps:
        e = o.galois_elt(st)
        keys[st] = o.keygen_galois(s, e, 300 + st)
        ctx.key_upload(KS_KEY_GALOIS, e, keys[st])
    Ql = 25
    rng = np.random.default_rng(21)
    ct = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                             for j in range(Ql)]) for _ in range(2)])
    elts = [o.galois_elt(st) for st in steps]
    d = _dev(ct)
    outs = [torch.zeros_like(d) for _ in steps]
    ctx.rotate_hoisted(d, Ql, steps, outs)
    torch.cuda.synchronize()
    want = o.rotate_hoisted(ct, Ql, elts, [keys[st] for st in steps])
    for i, out in enumerate(outs):
        assert np.array_equal(_host(out), want[i]), "rotation %d differs" % steps[i]
    diags = [np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                       for j in _ext_basis(o, Ql)]) for _ in steps]
    out = torch.zeros_like(d)
    ctx.linear_transform_hoisted(d, Ql, steps, [_dev(x) for x in diags], out)
    torch.cuda.synchronize()
    want = o.linear_transform_hoisted(ct, Ql, elts, [keys[st] for st in steps], diags)
    assert np.array_equal(_host(out), want)
    ctx.close()
