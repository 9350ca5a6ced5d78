"""GPU parity: the CUDA path through the C ABI against the CPU oracle, bit-exact."""
import numpy as np
import pytest

from tests.ksparams import CFG1, CFG3, MANYDIG, SMALL, oracle_for, split

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _ctx(cfg, **kw):
    from comp390project_b200 import KsContext
    log_n, q, p = split(cfg)
    return KsContext(log_n, q, p, device=0, **kw)


def _to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()


def _to_host(t):
    return t.cpu().numpy().view(np.uint64)


@pytest.mark.parametrize("name,cfg", [("cfg1", CFG1), ("small", SMALL), ("cfg3", CFG3)])
def test_ntt_roundtrip_bitexact(name, cfg, cuda_device):
    o = oracle_for(name)
    ctx = _ctx(cfg)
    K = o.L + o.alpha
    rng = np.random.default_rng(1)
    x = np.stack([rng.integers(0, int(m), size=o.N, dtype=np.uint64) for m in o.moduli])
    d = _to_dev(x)
    ctx.ntt_forward(d, K, 0, 1)
    fwd = _to_host(d)
    ref = o.ntt(x, list(range(K)))
    assert np.array_equal(fwd, ref)
    ctx.ntt_inverse(d, K, 0, 1)
    assert np.array_equal(_to_host(d), x)


@pytest.mark.parametrize("name", ["n14", "n15"])
def test_other_ring_sizes_bitexact(name, cuda_device):
    """N = 2^14 and 2^15 (2^7-point column pass): NTT round trip and a
    rotation key switch against the oracle, and the rotation decodes."""
    from tests.ksparams import N14, N15
    cfg = {"n14": N14, "n15": N15}[name]
    o = oracle_for(name)
    ctx = _ctx(cfg)
    K = o.L + o.alpha
    rng = np.random.default_rng(3)
    x = np.stack([rng.integers(0, int(m), size=o.N, dtype=np.uint64) for m in o.moduli])
    d = _to_dev(x)
    ctx.ntt_forward(d, K, 0, 1)
    assert np.array_equal(_to_host(d), o.ntt(x, list(range(K))))
    ctx.ntt_inverse(d, K, 0, 1)
    assert np.array_equal(_to_host(d), x)
    s = o.secret(5)
    step = 7
    elt = o.galois_elt(step)
    key = o.keygen_galois(s, elt, 17)
    ctx.key_upload(1, elt, key)
    Ql = o.L
    z, ct = _encrypted(o, Ql, 9, s)
    ref = o.apply_galois(ct, Ql, elt, key)
    d = _to_dev(ct)
    ctx.rotate(d, Ql, step)
    out = _to_host(d).reshape(2, Ql, o.N)
    assert np.array_equal(out, ref)
    dec = o.decode(o.decrypt(s, out, Ql), Ql, 2.0 ** 40)
    assert np.abs(dec - np.roll(z, -step)).mean() < 1e-3


@pytest.mark.parametrize("pattern", ["max", "zero", "alt", "one", "ramp"])
def test_ntt_extreme_inputs(pattern, cuda_device):
    """Inputs at the ends of [0, q) stress the lazy-reduction bounds of every
    butterfly path (FP64 for 42-bit primes, integer Shoup for 58/60-bit)."""
    o = oracle_for("cfg3")
    ctx = _ctx(CFG3)
    K = o.L + o.alpha
    x = np.empty((K, o.N), dtype=np.uint64)
    for i, m in enumerate(o.moduli):
        m = int(m)
        if pattern == "max":
            x[i] = m - 1
        elif pattern == "zero":
            x[i] = 0
        elif pattern == "alt":
            x[i] = np.where(np.arange(o.N) % 2 == 0, m - 1, 0)
        elif pattern == "one":
            x[i] = 1
        else:
            x[i] = (np.arange(o.N, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15 % m)) % np.uint64(m)
    d = _to_dev(x)
    ctx.ntt_forward(d, K, 0, 1)
    assert np.array_equal(_to_host(d), o.ntt(x, list(range(K))))
    d = _to_dev(x)
    ctx.ntt_inverse(d, K, 0, 1)
    assert np.array_equal(_to_host(d), o.ntt(x, list(range(K)), inverse=True))


def test_ntt_batch_prime_pattern(cuda_device):
    o = oracle_for("small")
    ctx = _ctx(SMALL)
    rng = np.random.default_rng(2)
    batch, nl, first = 3, 4, 2
    x = np.stack([rng.integers(0, int(o.moduli[first + (i % nl)]), size=o.N, dtype=np.uint64)
                  for i in range(batch * nl)])
    d = _to_dev(x)
    ctx.ntt_forward(d, nl, first, batch)
    ref = o.ntt(x, [first + (i % nl) for i in range(batch * nl)])
    assert np.array_equal(_to_host(d), ref)


def _encrypted(o, Ql, seed, s):
    rng = np.random.default_rng(seed)
    z = rng.uniform(-1, 1, o.N // 2)
    pt = o.encode(z, 2.0 ** 40, Ql)
    return z, o.encrypt(s, pt, Ql, seed + 100)


@pytest.mark.parametrize("name,cfg,Ql,step", [("cfg1", CFG1, 3, 1), ("small", SMALL, 7, 5),
                                              ("small", SMALL, 5, -3), ("small", SMALL, 1, 2),
                                              ("manydig", MANYDIG, 34, 3),
                                              ("manydig", MANYDIG, 33, -1)])
def test_rotate_bitexact(name, cfg, Ql, step, cuda_device):
    o = oracle_for(name)
    ctx = _ctx(cfg)
    s = o.secret(0)
    elt = o.galois_elt(step)
    assert ctx.galois_elt(step) == elt
    key = o.keygen_galois(s, elt, 11)
    ctx.key_upload(1, elt, key)
    z, ct = _encrypted(o, Ql, 3, s)
    ref = o.apply_galois(ct, Ql, elt, key)
    d = _to_dev(ct)
    ctx.rotate(d, Ql, step)
    out = _to_host(d).reshape(2, Ql, o.N)
    assert np.array_equal(out, ref)
    dec = o.decode(o.decrypt(s, out, Ql), Ql, 2.0 ** 40)
    assert np.abs(dec - np.roll(z, -step)).mean() < 1e-3


def test_conjugate_bitexact(cuda_device):
    """Complex conjugation: Galois element 2N - 1 (Phantom's conjugate), on
    complex slots."""
    o = oracle_for("small")
    ctx = _ctx(SMALL)
    s = o.secret(0)
    elt = 2 * o.N - 1
    key = o.keygen_galois(s, elt, 13)
    ctx.key_upload(1, elt, key)
    rng = np.random.default_rng(8)
    Ql = o.L
    z = rng.uniform(-1, 1, o.N // 2) + 1j * rng.uniform(-1, 1, o.N // 2)
    ct = o.encrypt(s, o.encode(z, 2.0 ** 40, Ql), Ql, 108)
    ref = o.apply_galois(ct, Ql, elt, key)
    d = _to_dev(ct)
    ctx.apply_galois(d, Ql, elt)
    out = _to_host(d).reshape(2, Ql, o.N)
    assert np.array_equal(out, ref)
    dec = o.decode(o.decrypt(s, out, Ql), Ql, 2.0 ** 40)
    assert np.abs(dec - np.conj(z)).mean() < 1e-3


@pytest.mark.parametrize("name,cfg,Ql", [("cfg1", CFG1, 3), ("small", SMALL, 7), ("small", SMALL, 4),
                                         ("cfg3", CFG3, 35)])
def test_relinearize_bitexact(name, cfg, Ql, cuda_device):
    o = oracle_for(name)
    ctx = _ctx(cfg)
    s = o.secret(1)
    key = o.keygen_relin(s, 21)
    ctx.key_upload(0, 0, key)
    z1, c1 = _encrypted(o, Ql, 5, s)
    z2, c2 = _encrypted(o, Ql, 6, s)
    m = o.multiply(c1, c2, Ql)
    ref = o.relinearize(m, Ql, key)
    d = _to_dev(m)
    ctx.relinearize(d, Ql)
    out = _to_host(d).reshape(3, Ql, o.N)[:2]
    assert np.array_equal(out, ref)
    if Ql >= 2:
        dec = o.decode(o.decrypt(s, out, Ql), Ql, 2.0 ** 80)
        assert np.abs(dec - z1 * z2).mean() < 1e-3


def test_relinearize_on_the_reference_test_parameters(cuda_device):
    """The reference's own correctness test (multi_gpu_keyswitch_test.cu:186-332):
    N=8192, {60,40,40,40,60}, inputs (rand() % 1000) / 100 - 5; the GPU result
    must equal the oracle bit for bit and decode to the product (MAE < 1e-3)."""
    from tests.ksparams import REFTEST, reference_test_values
    o = oracle_for("reftest")
    ctx = _ctx(REFTEST)
    Ql = o.L
    s = o.secret(42)
    key = o.keygen_relin(s, 42)
    ctx.key_upload(0, 0, key)
    z1 = reference_test_values(o.N // 2, 42)
    z2 = reference_test_values(o.N // 2, 43)
    c1 = o.encrypt(s, o.encode(z1, 2.0 ** 40, Ql), Ql, 1)
    c2 = o.encrypt(s, o.encode(z2, 2.0 ** 40, Ql), Ql, 2)
    m = o.multiply(c1, c2, Ql)
    ref = o.relinearize(m, Ql, key)
    d = _to_dev(m)
    ctx.relinearize(d, Ql)
    out = _to_host(d).reshape(3, Ql, o.N)[:2]
    assert np.array_equal(out, ref)
    dec = o.decode(o.decrypt(s, out, Ql), Ql, 2.0 ** 80)
    assert np.abs(dec - z1 * z2).mean() < 1e-3


@pytest.mark.parametrize("name,cfg,kind", [("cfg1", CFG1, 1), ("small", SMALL, 1), ("small", SMALL, 0)])
def test_gpu_keygen_matches_oracle(name, cfg, kind, cuda_device):
    o = oracle_for(name)
    ctx = _ctx(cfg)
    from comp390project_b200 import secret_generate
    s = secret_generate(o.log_n, 7, 0)
    assert np.array_equal(s, o.secret(7))
    elt = o.galois_elt(3) if kind == 1 else 0
    ctx.key_generate(kind, elt, s, 99)
    torch.cuda.synchronize()
    got = ctx.key_download(kind, elt)
    ref = o.keygen_galois(s, elt, 99) if kind == 1 else o.keygen_relin(s, 99)
    assert np.array_equal(got, ref)


def test_config3_rotation_bitexact(cuda_device):
    o = oracle_for("cfg3")
    ctx = _ctx(CFG3)
    from comp390project_b200 import secret_generate
    s = secret_generate(o.log_n, 3, 192)
    assert np.array_equal(s, o.secret(3, 192))
    step = 5
    elt = o.galois_elt(step)
    ctx.key_generate(1, elt, s, 17)
    z, ct = _encrypted(o, 35, 9, s)
    d = _to_dev(ct)
    ctx.rotate(d, 35, step)
    out = _to_host(d).reshape(2, 35, o.N)
    key = o.keygen_galois(s, elt, 17)
    ref = o.apply_galois(ct, 35, elt, key)
    assert np.array_equal(out, ref)
    dec = o.decode(o.decrypt(s, out, 35), 35, 2.0 ** 40)
    assert np.abs(dec - np.roll(z, -step)).mean() < 1e-3


@pytest.mark.parametrize("lanes", [1, 3])
def test_rotate_batch_lanes(lanes, cuda_device):
    """Batched rotations spread over several execution lanes (streams with
    their own scratch) give the same words as the oracle for every member."""
    o = oracle_for("small")
    ctx = _ctx(SMALL, max_batch=lanes)
    s = o.secret(4)
    steps = [1, 2, 3, -1, 5]
    keys = {}
    for st in steps:
        elt = o.galois_elt(st)
        keys[st] = o.keygen_galois(s, elt, 40 + st)
        ctx.key_upload(1, elt, keys[st])
    cts = [_encrypted(o, 7, 50 + i, s)[1] for i in range(len(steps))]
    devs = [_to_dev(ct) for ct in cts]
    ctx.rotate_batch(devs, steps, 7)
    torch.cuda.synchronize()
    for ct, d, st in zip(cts, devs, steps):
        ref = o.apply_galois(ct, 7, o.galois_elt(st), keys[st])
        assert np.array_equal(_to_host(d).reshape(2, 7, o.N), ref)


@pytest.mark.parametrize("name,lanes,group,n", [("small", 1, 2, 5), ("small", 2, 3, 7),
                                                 ("small", 3, 8, 8), ("cfg3", 2, 2, 3)])
def test_rotate_batch_groups(name, lanes, group, n, cuda_device):
    """Groups of rotations pushed through every launch together (grid z =
    member), over one or more lanes, a short last group included: every
    member equals the oracle word for word."""
    cfg = {"small": SMALL, "cfg3": CFG3}[name]
    o = oracle_for(name)
    ctx = _ctx(cfg, max_batch=lanes, batch_group=group)
    s = o.secret(6, 192 if name == "cfg3" else 0)
    steps = [1, 2, 3, -1, 5, 1, 2, 4][:n] if name == "small" else [1, 2, 1]
    keys = {}
    for st in sorted(set(steps)):
        elt = o.galois_elt(st)
        keys[st] = o.keygen_galois(s, elt, 60 + st)
        ctx.key_upload(1, elt, keys[st])
    Ql = o.L
    rng = np.random.default_rng(31)
    cts = [np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                               for j in range(Ql)]) for _ in range(2)]) for _ in steps]
    devs = [_to_dev(ct) for ct in cts]
    ctx.rotate_batch(devs, steps, Ql)
    torch.cuda.synchronize()
    for ct, d, st in zip(cts, devs, steps):
        ref = o.apply_galois(ct, Ql, o.galois_elt(st), keys[st])
        assert np.array_equal(_to_host(d).reshape(2, Ql, o.N), ref)
    # a lower level through the same group scratch
    Ql2 = Ql - 2
    devs2 = [_to_dev(ct[:, :Ql2]) for ct in cts]
    ctx.rotate_batch(devs2, steps, Ql2)
    torch.cuda.synchronize()
    for ct, d, st in zip(cts, devs2, steps):
        ref = o.apply_galois(np.ascontiguousarray(ct[:, :Ql2]), Ql2, o.galois_elt(st), keys[st])
        assert np.array_equal(_to_host(d).reshape(2, Ql2, o.N), ref)
    ctx.close()


@pytest.mark.parametrize("lanes,group,n", [(2, 2, 5), (1, 1, 3), (2, 8, 21), (3, 4, 13)])
def test_rotate_batch_host_matches_device_batch(lanes, group, n, cuda_device):
    """ks_rotate_batch_host (host ciphertexts, copies pipelined over lanes)
    returns the words of ks_rotate_batch on device copies: a single staging
    buffer per lane (group 1), and double-buffered staging with the tapered
    group sizes, several groups per lane and each half reused."""
    from comp390project_b200 import KS_KEY_GALOIS, KsContext
    o = oracle_for("small")
    log_n, q, p = split(SMALL)
    ctx = KsContext(log_n, q, p, device=0, max_batch=lanes, batch_group=group)
    s = o.secret(8, 64)
    steps = [1 + i % 3 for i in range(n)]
    for st in sorted(set(steps)):
        e = o.galois_elt(st)
        ctx.key_upload(KS_KEY_GALOIS, e, o.keygen_galois(s, e, 80 + st))
    rng = np.random.default_rng(21)
    Ql = o.L
    cts = [np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                               for j in range(Ql)]) for _ in range(2)]) for _ in steps]
    dev = [torch.from_numpy(c.view(np.int64).copy()).cuda() for c in cts]
    ctx.rotate_batch(dev, steps, Ql)
    host = [torch.from_numpy(c.view(np.int64).copy()).pin_memory() for c in cts[:3]]
    host += [c.copy() for c in cts[3:]]  # pageable numpy arrays work too
    ctx.rotate_batch_host(host, steps, Ql)
    torch.cuda.synchronize()
    for d, h in zip(dev, host):
        hv = h.numpy().view(np.uint64) if isinstance(h, torch.Tensor) else h
        assert np.array_equal(d.cpu().numpy().view(np.uint64), hv)
    ctx.close()


@pytest.mark.parametrize("name,Ql", [("small", 7), ("small", 4), ("small", 2), ("cfg1", 3),
                                     ("cfg3", 35)])
def test_rescale_matches_oracle(name, Ql, cuda_device):
    """ks_rescale (divide by the last prime and round) equals the oracle word
    for word at several levels."""
    from comp390project_b200 import KsContext
    cfg = {"small": SMALL, "cfg1": CFG1, "cfg3": CFG3}[name]
    o = oracle_for(name)
    log_n, q, p = split(cfg)
    ctx = KsContext(log_n, q, p, device=0)
    rng = np.random.default_rng(40 + Ql)
    ct = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                             for j in range(Ql)]) for _ in range(2)])
    d = torch.from_numpy(ct.view(np.int64).copy()).cuda()
    out = torch.zeros((2, Ql - 1, o.N), dtype=torch.int64, device="cuda")
    ctx.rescale(d, Ql, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint64), o.rescale(ct, Ql))
    ctx.close()


def test_key_upload_from_wire_blob(cuda_device):
    """A Galois key shipped as a wire blob rotates like the uploaded array."""
    from comp390project_b200 import KsContext, wire
    o = oracle_for("small")
    log_n, q, p = split(SMALL)
    ctx = KsContext(log_n, q, p, device=0)
    s = o.secret(9, 64)
    elt = o.galois_elt(5)
    key = o.keygen_galois(s, elt, 55)
    ctx.key_upload_wire(wire.pack_key(log_n, q, p, key, galois_elt=elt))
    rng = np.random.default_rng(56)
    Ql = o.L
    ct = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                             for j in range(Ql)]) for _ in range(2)])
    d = torch.from_numpy(ct.view(np.int64).copy()).cuda()
    ctx.apply_galois(d, Ql, elt)
    torch.cuda.synchronize()
    assert np.array_equal(d.cpu().numpy().view(np.uint64), o.apply_galois(ct, Ql, elt, key))
    ctx.close()


def test_python_evaluator_rescale_and_hoisted(cuda_device):
    """keyswitching.Evaluator (the reference-named Python API): rescale_to_next
    and rotate_hoisted return the oracle's words and the right metadata."""
    from comp390project_b200.keyswitching import Ciphertext, Evaluator
    o = oracle_for("small")
    ctx = _ctx(SMALL, max_batch=2)
    s = o.secret(3, 64)
    steps = [1, 4]
    keys = {}
    for st in steps:
        e = o.galois_elt(st)
        keys[st] = o.keygen_galois(s, e, 40 + st)
        ctx.key_upload(1, e, keys[st])
    Ql = o.L
    z, ct = _encrypted(o, Ql, 12, s)
    ev = Evaluator(ctx)
    c = Ciphertext(_to_dev(ct), Ql, o.N, 2.0 ** 40)
    r = ev.rescale_to_next(c)
    assert r.coeff_modulus_size == Ql - 1 and r.scale == 2.0 ** 40 / float(o.moduli[Ql - 1])
    assert np.array_equal(_to_host(r.data).reshape(2, Ql - 1, o.N), o.rescale(ct, Ql))
    rots = ev.rotate_hoisted(c, steps)
    want = o.rotate_hoisted(ct, Ql, [o.galois_elt(st) for st in steps], [keys[st] for st in steps])
    for i, rc in enumerate(rots):
        assert np.array_equal(_to_host(rc.data).reshape(2, Ql, o.N), want[i])
    ctx.close()
