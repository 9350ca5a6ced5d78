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
