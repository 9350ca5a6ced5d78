"""CPU oracle against the reference's golden vectors and independent checks
(naive negacyclic transforms, big-integer CRT, decode-level semantics)."""
import json
import os

import numpy as np
import pytest

from oracle.oracle import Oracle, gen_primes, prng
from tests.ksparams import CFG1, SMALL, oracle_for, split

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _brev(i, bits):
    return int(format(i, "0%db" % bits)[::-1], 2) if bits else 0


@pytest.fixture(scope="module")
def kat():
    with open(os.path.join(GOLDEN, "prime_kat.json")) as f:
        return json.load(f)


def test_prime_kat_matches_reference_logs(kat):
    """Every modulus chain the reference logged (ckks_bench.txt) is regenerated."""
    assert len(kat) >= 10
    for rec in kat:
        got = [int(x) for x in gen_primes(rec["log_n"], rec["bits"])]
        assert got == rec["primes"], rec["source"]


def test_config_primes_properties():
    for cfg in (CFG1, SMALL):
        log_n, q, p = split(cfg)
        for x in list(q) + list(p):
            assert int(x) % (2 << log_n) == 1
    log_n, q, p = split(dict(log_n=16, qbits=(58,) + (42,) * 34, pbits=(60,) * 5))
    assert len(set(map(int, q)) | set(map(int, p))) == 40
    assert all(int(x).bit_length() == 42 for x in q[1:])
    assert int(q[0]).bit_length() == 58 and all(int(x).bit_length() == 60 for x in p)


@pytest.mark.parametrize("log_n", [3, 4, 6])
def test_ntt_matches_naive_evaluation(log_n):
    """Slot i of the forward transform holds a(psi^(2 brev(i) + 1)), psi the
    minimal primitive 2N-th root (checked by brute force)."""
    N = 1 << log_n
    qs = gen_primes(log_n, [30, 31])
    o = Oracle(log_n, qs[:1], qs[1:])
    q = int(qs[0])
    psi = o.psi(0)
    assert pow(psi, N, q) == q - 1
    roots = [pow(psi, 2 * k + 1, q) for k in range(N)]
    assert psi == min(roots)
    rng = np.random.default_rng(log_n)
    a = rng.integers(0, q, size=N, dtype=np.uint64)
    A = o.ntt(a.reshape(1, N), [0])[0]
    for i in range(N):
        e = 2 * _brev(i, log_n) + 1
        assert int(A[i]) == sum(int(a[k]) * pow(psi, e * k, q) for k in range(N)) % q
    assert np.array_equal(o.ntt(A.reshape(1, N), [0], inverse=True)[0], a)


def test_ntt_negacyclic_convolution():
    log_n = 6
    N = 1 << log_n
    qs = gen_primes(log_n, [40, 50])
    o = Oracle(log_n, qs[:1], qs[1:])
    q = int(qs[0])
    rng = np.random.default_rng(7)
    a = rng.integers(0, q, size=N, dtype=np.uint64)
    b = rng.integers(0, q, size=N, dtype=np.uint64)
    A = o.ntt(a.reshape(1, N), [0])[0]
    B = o.ntt(b.reshape(1, N), [0])[0]
    C = np.array([(int(x) * int(y)) % q for x, y in zip(A, B)], dtype=np.uint64)
    c = o.ntt(C.reshape(1, N), [0], inverse=True)[0]
    ref = [0] * N
    for i in range(N):
        for j in range(N):
            k = i + j
            v = int(a[i]) * int(b[j])
            if k >= N:
                ref[k - N] -= v
            else:
                ref[k] += v
    assert [int(x) for x in c] == [r % q for r in ref]


def test_bconv_matches_bigint_definition():
    """Fast base conversion: y = sum_i [x_i (B/b_i)^-1]_{b_i} (B/b_i) mod c, which
    equals X + u*B mod c for the CRT value X and one u in [0, n) per coefficient."""
    o = oracle_for("small")
    src = [1, 2, 3]
    dst = [0, 4, 7, 8, 9]
    rng = np.random.default_rng(3)
    x = np.stack([rng.integers(0, int(o.moduli[i]), size=o.N, dtype=np.uint64) for i in src])
    y = o.bconv(x, src, dst)
    B = 1
    for i in src:
        B *= int(o.moduli[i])
    for k in range(0, o.N, 97):
        vals = [int(x[t, k]) for t in range(len(src))]
        X = 0
        terms = []
        for t, i in enumerate(src):
            bi = int(o.moduli[i])
            bhat = B // bi
            v = vals[t] * pow(bhat % bi, -1, bi) % bi
            terms.append(v * bhat)
            X += v * bhat
        u = X // B
        assert 0 <= u < len(src)
        for jj, j in enumerate(dst):
            c = int(o.moduli[j])
            assert int(y[jj, k]) == X % c
            assert int(y[jj, k]) == (X % B + u * B) % c


def test_galois_ntt_equals_coefficient_automorphism():
    o = oracle_for("cfg1")
    rng = np.random.default_rng(11)
    a = np.stack([rng.integers(0, int(m), size=o.N, dtype=np.uint64) for m in o.moduli[:3]])
    for step in (1, 5, -2):
        elt = o.galois_elt(step)
        lhs = o.ntt(o.galois_coeff(a, elt, [0, 1, 2]), [0, 1, 2])
        rhs = o.galois_ntt(o.ntt(a, [0, 1, 2]), elt)
        assert np.array_equal(lhs, rhs)


def test_moddown_divides_exact_multiples_of_P():
    """ModDown of P*a (exactly divisible) returns a on every Q limb."""
    o = oracle_for("small")
    Ql = 5
    rng = np.random.default_rng(5)
    P = 1
    for p in o.p:
        P *= int(p)
    a = rng.integers(-(1 << 30), 1 << 30, size=o.N)
    idx = list(range(Ql)) + [o.L + i for i in range(o.alpha)]
    coeff = np.stack([np.array([(int(v) * P) % int(o.moduli[j]) for v in a], dtype=np.uint64)
                      for j in idx])
    cx = o.ntt(coeff, idx)
    out = o.moddown(cx, Ql)
    ref = np.stack([np.array([int(v) % int(o.moduli[j]) for v in a], dtype=np.uint64)
                    for j in range(Ql)])
    assert np.array_equal(out, o.ntt(ref, list(range(Ql))))


def test_modup_extends_each_digit_consistently():
    """Every ModUp digit, back in coefficient form, is X_d + u*Q_d on all limbs."""
    o = oracle_for("small")
    Ql = 7
    rng = np.random.default_rng(9)
    c = np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64) for j in range(Ql)])
    t = o.modup(c, Ql)
    idx = list(range(Ql)) + [o.L + i for i in range(o.alpha)]
    coef_in = o.ntt(c, list(range(Ql)), inverse=True)
    for d in range(o.digits(Ql)):
        D = list(range(d * o.alpha, min((d + 1) * o.alpha, Ql)))
        td = o.ntt(t[d], idx, inverse=True)
        Qd = 1
        for j in D:
            Qd *= int(o.moduli[j])
        for k in range(0, o.N, 211):
            X = 0
            for j in D:
                qj = int(o.moduli[j])
                X += int(coef_in[j, k]) * (Qd // qj) * pow((Qd // qj) % qj, -1, qj)
            X %= Qd
            us = set()
            for jj, j in enumerate(idx):
                m = int(o.moduli[j])
                v = int(td[jj, k])
                found = [u for u in range(len(D)) if (X + u * Qd) % m == v]
                assert found, (d, j, k)
                us.update(found)
            assert len(us) >= 1


@pytest.mark.parametrize("step", [1, 3, -1, 100])
def test_rotation_decodes_to_rolled_slots(step):
    o = oracle_for("cfg1")
    s = o.secret(0)
    elt = o.galois_elt(step)
    key = o.keygen_galois(s, elt, 11)
    rng = np.random.default_rng(step & 0xFFFF)
    z = rng.uniform(-1, 1, o.N // 2) + 1j * rng.uniform(-1, 1, o.N // 2)
    ct = o.encrypt(s, o.encode(z, 2.0 ** 40, 3), 3, 5)
    r = o.apply_galois(ct, 3, elt, key)
    dec = o.decode(o.decrypt(s, r, 3), 3, 2.0 ** 40)
    assert np.abs(dec - np.roll(z, -step)).mean() < 1e-3


def test_conjugation_decodes_to_conjugate_slots():
    """Galois element 2N - 1 (X -> X^-1) conjugates every slot."""
    o = oracle_for("cfg1")
    s = o.secret(0)
    elt = 2 * o.N - 1
    key = o.keygen_galois(s, elt, 12)
    rng = np.random.default_rng(9)
    z = rng.uniform(-1, 1, o.N // 2) + 1j * rng.uniform(-1, 1, o.N // 2)
    ct = o.encrypt(s, o.encode(z, 2.0 ** 40, 3), 3, 6)
    dec = o.decode(o.decrypt(s, o.apply_galois(ct, 3, elt, key), 3), 3, 2.0 ** 40)
    assert np.abs(dec - np.conj(z)).mean() < 1e-3


def test_relinearisation_decodes_to_product():
    o = oracle_for("cfg1")
    s = o.secret(1)
    key = o.keygen_relin(s, 3)
    rng = np.random.default_rng(2)
    z1, z2 = rng.uniform(-1, 1, o.N // 2), rng.uniform(-1, 1, o.N // 2)
    c1 = o.encrypt(s, o.encode(z1, 2.0 ** 40, 3), 3, 1)
    c2 = o.encrypt(s, o.encode(z2, 2.0 ** 40, 3), 3, 2)
    r = o.relinearize(o.multiply(c1, c2, 3), 3, key)
    dec = o.decode(o.decrypt(s, r, 3), 3, 2.0 ** 80)
    assert np.abs(dec - z1 * z2).mean() < 1e-3


def test_relinearisation_on_the_reference_test_parameters():
    """The reference's multi_gpu_keyswitch_test (src/benchmarks/
    multi_gpu_keyswitch_test.cu:186-332): N=8192, {60,40,40,40,60}, inputs
    (rand() % 1000) / 100 - 5, multiply + relinearise, decode MAE < 1e-3."""
    from tests.ksparams import reference_test_values
    o = oracle_for("reftest")
    Ql = o.L
    s = o.secret(42)
    key = o.keygen_relin(s, 42)
    z1 = reference_test_values(o.N // 2, 42)
    z2 = reference_test_values(o.N // 2, 43)
    c1 = o.encrypt(s, o.encode(z1, 2.0 ** 40, Ql), Ql, 1)
    c2 = o.encrypt(s, o.encode(z2, 2.0 ** 40, Ql), Ql, 2)
    r = o.relinearize(o.multiply(c1, c2, Ql), Ql, key)
    dec = o.decode(o.decrypt(s, r, Ql), Ql, 2.0 ** 80)
    assert np.abs(dec - z1 * z2).mean() < 1e-3


def test_keyswitch_noise_is_small():
    o = oracle_for("small")
    s = o.secret(2)
    elt = o.galois_elt(2)
    key = o.keygen_galois(s, elt, 8)
    rng = np.random.default_rng(4)
    for Ql in (7, 4, 1):
        c = np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                      for j in range(Ql)])
        ks = o.keyswitch(c, Ql, key)
        snew = o.galois_ntt(o.secret_ntt(s, Ql), elt)
        assert o.ks_noise_log2(s, c, snew, ks, Ql) < 24


def test_hoisted_rotations_decode():
    o = oracle_for("cfg1")
    s = o.secret(6)
    steps = [1, 2, 7]
    elts = [o.galois_elt(st) for st in steps]
    keys = [o.keygen_galois(s, e, 30 + i) for i, e in enumerate(elts)]
    rng = np.random.default_rng(8)
    z = rng.uniform(-1, 1, o.N // 2)
    ct = o.encrypt(s, o.encode(z, 2.0 ** 40, 3), 3, 9)
    outs = o.rotate_hoisted(ct, 3, elts, keys)
    for st, out in zip(steps, outs):
        dec = o.decode(o.decrypt(s, out, 3), 3, 2.0 ** 40)
        assert np.abs(dec - np.roll(z, -st)).mean() < 1e-3


def test_hoisted_linear_transform_decodes():
    """Double hoisting (one ModUp, products accumulated in the extended basis,
    one ModDown) decodes to sum_r d_r * roll(z, r)."""
    o = oracle_for("small")
    s = o.secret(12, 64)
    steps = [1, 3, 8]
    elts = [o.galois_elt(st) for st in steps]
    keys = [o.keygen_galois(s, e, 60 + i) for i, e in enumerate(elts)]
    Ql = o.L
    n = o.N // 2
    rng = np.random.default_rng(13)
    z = rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)
    ct = o.encrypt(s, o.encode(z, 2.0 ** 40, Ql), Ql, 19)
    dz = [rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n) for _ in steps]
    basis = list(range(Ql)) + [o.L + i for i in range(o.alpha)]
    diags = [o.encode_basis(x, 2.0 ** 40, basis) for x in dz]
    out = o.linear_transform_hoisted(ct, Ql, elts, keys, diags)
    dec = o.decode(o.decrypt(s, out, Ql), Ql, 2.0 ** 80)
    want = sum(x * np.roll(z, -st) for x, st in zip(dz, steps))
    assert np.abs(dec - want).mean() < 1e-3


def test_encode_basis_matches_encode_on_q_limbs():
    o = oracle_for("small")
    z = np.random.default_rng(2).uniform(-1, 1, o.N // 2)
    basis = list(range(o.L)) + [o.L + i for i in range(o.alpha)]
    ext = o.encode_basis(z, 2.0 ** 40, basis)
    assert np.array_equal(ext[:o.L], o.encode(z, 2.0 ** 40, o.L))


def test_rescale_decodes_to_product_at_lower_scale():
    """multiply + relinearise + rescale decodes to the product at scale
    2^80 / q_last (the reference's rescale_to_next_inplace semantics)."""
    o = oracle_for("small")
    s = o.secret(14, 64)
    Ql = o.L
    rng = np.random.default_rng(15)
    z1 = rng.uniform(-1, 1, o.N // 2)
    z2 = rng.uniform(-1, 1, o.N // 2)
    c1 = o.encrypt(s, o.encode(z1, 2.0 ** 40, Ql), Ql, 31)
    c2 = o.encrypt(s, o.encode(z2, 2.0 ** 40, Ql), Ql, 32)
    rk = o.keygen_relin(s, 33)
    r = o.relinearize(o.multiply(c1, c2, Ql), Ql, rk)
    rs = o.rescale(r, Ql)
    scale = 2.0 ** 80 / float(o.moduli[Ql - 1])
    dec = o.decode(o.decrypt(s, rs, Ql - 1), Ql - 1, scale)
    assert np.abs(dec - z1 * z2).mean() < 1e-3


def test_secret_hamming_weight_and_gaussian_support():
    o = oracle_for("small")
    s = o.secret(3, 64)
    assert np.count_nonzero(s) == 64 and set(np.unique(s)) <= {-1, 0, 1}
    u = o.secret(3, 0)
    assert set(np.unique(u)) == {-1, 0, 1}
    from oracle.oracle import lib
    vals = [lib().ork_gauss(prng(1, 4, i)) for i in range(20000)]
    assert max(abs(v) for v in vals) <= 19
    assert abs(np.std(vals) - 3.2) < 0.15
