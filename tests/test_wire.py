"""Wire format of keys and ciphertexts (host functions of the C ABI)."""
import numpy as np
import pytest

from tests.ksparams import SMALL, oracle_for, split


@pytest.fixture(scope="module")
def small():
    return oracle_for("small"), split(SMALL)


def test_key_round_trip(small):
    from comp390project_b200 import wire
    o, (log_n, q, p) = small
    s = o.secret(2, 64)
    elt = o.galois_elt(3)
    key = o.keygen_galois(s, elt, 5)
    blob = wire.pack_key(log_n, q, p, key, galois_elt=elt)
    assert len(blob) == 64 + key.size * 8
    obj, e, words = wire.unpack(log_n, q, p, blob)
    assert obj == wire.KS_WIRE_GALOIS_KEY and e == elt
    assert np.array_equal(words, key.reshape(words.shape))
    rk = o.keygen_relin(s, 6)
    obj, e, words = wire.unpack(log_n, q, p, wire.pack_key(log_n, q, p, rk))
    assert obj == wire.KS_WIRE_RELIN_KEY and e == 0 and np.array_equal(words, rk.reshape(words.shape))


def test_ciphertext_round_trip_and_file(small, tmp_path):
    from comp390project_b200 import wire
    o, (log_n, q, p) = small
    rng = np.random.default_rng(3)
    Ql = 5
    ct = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                             for j in range(Ql)]) for _ in range(2)])
    path = str(tmp_path / "ct.ksb")
    wire.save(path, wire.pack_ciphertext(log_n, q, p, ct))
    obj, _, words = wire.unpack(log_n, q, p, wire.load(path))
    assert obj == wire.KS_WIRE_CIPHERTEXT and words.shape == ct.shape
    assert np.array_equal(words, ct)


def test_rejects_corruption_other_parameters_and_bad_residues(small):
    from comp390project_b200 import KsError, wire
    o, (log_n, q, p) = small
    s = o.secret(2, 64)
    key = o.keygen_relin(s, 7)
    blob = bytearray(wire.pack_key(log_n, q, p, key))
    bad = bytearray(blob)
    bad[64 + 1000] ^= 0x01  # payload bit flip: digest mismatch
    with pytest.raises(KsError):
        wire.unpack(log_n, q, p, bytes(bad))
    with pytest.raises(KsError):  # another prime chain
        wire.unpack(log_n, list(q[:-1]) + [int(p[0])], list(p[:-1]) + [int(q[-1])], bytes(blob))
    with pytest.raises(KsError):  # truncated
        wire.unpack(log_n, q, p, bytes(blob[:-8]))
    noncanon = key.copy()
    noncanon.reshape(-1)[0] = int(o.moduli[0])  # word == q_0 is not a residue
    with pytest.raises(KsError):
        wire.unpack(log_n, q, p, wire.pack_key(log_n, q, p, noncanon))


@pytest.mark.parametrize("kind", ["ciphertext", "galois_key"])
def test_every_header_bit_flip_is_rejected(small, kind):
    """Every one of the 512 header bits is covered: flipping it makes unpack
    fail (the Galois element and the reserved word included)."""
    from comp390project_b200 import KsError, wire
    o, (log_n, q, p) = small
    if kind == "ciphertext":
        rng = np.random.default_rng(8)
        ct = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                                 for j in range(2)]) for _ in range(2)])
        blob = wire.pack_ciphertext(log_n, q, p, ct)
    else:
        elt = o.galois_elt(5)
        blob = wire.pack_key(log_n, q, p, o.keygen_galois(o.secret(2, 64), elt, 5), galois_elt=elt)
    wire.unpack(log_n, q, p, blob)
    for pos in range(64):
        for bit in range(8):
            bad = bytearray(blob)
            bad[pos] ^= 1 << bit
            with pytest.raises(KsError):
                wire.unpack(log_n, q, p, bytes(bad))


def test_pack_rejects_a_bad_galois_element(small):
    from comp390project_b200 import KsError, wire
    o, (log_n, q, p) = small
    key = o.keygen_galois(o.secret(2, 64), o.galois_elt(3), 5)
    for elt in (0, 2, 2 * o.N + 1):
        with pytest.raises(KsError):
            wire.pack_key(log_n, q, p, key, galois_elt=elt)


def test_any_single_bit_flip_is_rejected(small):
    """Property: flipping any one bit of a ciphertext blob (header or payload)
    makes unpack fail; the untouched blob still unpacks."""
    from hypothesis import given, settings, strategies as st

    from comp390project_b200 import KsError, wire
    o, (log_n, q, p) = small
    rng = np.random.default_rng(8)
    Ql = 3
    ct = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                             for j in range(Ql)]) for _ in range(2)])
    blob = wire.pack_ciphertext(log_n, q, p, ct)
    wire.unpack(log_n, q, p, blob)

    @settings(max_examples=200, deadline=None)
    @given(pos=st.integers(0, len(blob) - 1), bit=st.integers(0, 7))
    def check(pos, bit):
        bad = bytearray(blob)
        bad[pos] ^= 1 << bit
        with pytest.raises(KsError):
            wire.unpack(log_n, q, p, bytes(bad))

    check()
