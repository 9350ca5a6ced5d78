"""Wire format of evaluation keys and ciphertexts (ks_wire_* of the C ABI).

A blob is a 64-byte header (magic, version, object, Galois element, ring and
basis sizes, FNV-1a digests of the parameters and of the header + payload) followed by
the uint64 words in the in-memory layout: a full key [digits][2][L+alpha][N]
or a ciphertext [polys][level_limbs][N].  Unpacking rejects another parameter
set, a wrong size, a bad Galois element, a digest mismatch (any changed byte)
or a non-canonical residue.  The
reference has no serialised form: its key distribution
(src/multi_gpu/distributed_context.cu:112-134) regenerates keys per GPU.
Host functions only; no device is needed."""
from __future__ import annotations

import ctypes as C
from typing import Sequence, Tuple

import numpy as np

from . import _capi
from ._capi import (KS_WIRE_CIPHERTEXT, KS_WIRE_GALOIS_KEY, KS_WIRE_RELIN_KEY, KsError,
                    ks_params)

__all__ = ["pack_key", "pack_ciphertext", "unpack", "save", "load", "KS_WIRE_RELIN_KEY",
           "KS_WIRE_GALOIS_KEY", "KS_WIRE_CIPHERTEXT"]


class _Params:
    def __init__(self, log_n: int, q: Sequence[int], p: Sequence[int]):
        self.q = np.ascontiguousarray(q, dtype=np.uint64)
        self.p = np.ascontiguousarray(p, dtype=np.uint64)
        self.s = ks_params(int(log_n), len(self.q), self.q.ctypes.data_as(C.POINTER(C.c_uint64)),
                           len(self.p), self.p.ctypes.data_as(C.POINTER(C.c_uint64)), 0, 1)
        self.log_n = int(log_n)


def _pack(prm: _Params, obj: int, elt: int, level: int, polys: int, words: np.ndarray) -> bytes:
    lib = _capi.load()
    n = lib.ks_wire_size(C.byref(prm.s), obj, level, polys)
    w = np.ascontiguousarray(words, dtype=np.uint64).reshape(-1)
    if n == 0 or w.size * 8 + 64 != n:
        raise KsError(_capi.KS_ERR_INVALID, "words do not match the object's shape")
    buf = C.create_string_buffer(n)
    rc = lib.ks_wire_pack(C.byref(prm.s), obj, int(elt), level, polys,
                          w.ctypes.data_as(C.POINTER(C.c_uint64)), buf, n)
    if rc != 0:
        raise KsError(rc, "pack failed")
    return buf.raw


def pack_key(log_n: int, q, p, key: np.ndarray, galois_elt: int | None = None) -> bytes:
    """Full key [digits][2][L+alpha][N]; galois_elt None = relinearisation key."""
    prm = _Params(log_n, q, p)
    obj = KS_WIRE_RELIN_KEY if galois_elt is None else KS_WIRE_GALOIS_KEY
    return _pack(prm, obj, galois_elt or 0, 0, 0, key)


def pack_ciphertext(log_n: int, q, p, ct: np.ndarray) -> bytes:
    """Ciphertext [polys][level_limbs][N] (canonical residues)."""
    prm = _Params(log_n, q, p)
    ct = np.asarray(ct)
    return _pack(prm, KS_WIRE_CIPHERTEXT, 0, ct.shape[1], ct.shape[0], ct)


def unpack(log_n: int, q, p, blob: bytes) -> Tuple[int, int, np.ndarray]:
    """-> (object, galois_elt, words reshaped to the object's layout)."""
    prm = _Params(log_n, q, p)
    lib = _capi.load()
    obj, elt, level, polys = C.c_int(), C.c_uint32(), C.c_int(), C.c_int()
    raw = C.create_string_buffer(bytes(blob), len(blob))
    rc = lib.ks_wire_unpack(C.byref(prm.s), raw, len(blob), C.byref(obj), C.byref(elt),
                            C.byref(level), C.byref(polys), None, 0)
    if rc != 0:
        raise KsError(rc, "not a valid blob for these parameters")
    N = 1 << prm.log_n
    if obj.value == KS_WIRE_CIPHERTEXT:
        shape = (polys.value, level.value, N)
    else:
        L, a = len(prm.q), len(prm.p)
        shape = ((L + a - 1) // a, 2, L + a, N)
    out = np.empty(shape, dtype=np.uint64)
    rc = lib.ks_wire_unpack(C.byref(prm.s), raw, len(blob), None, None, None, None,
                            out.ctypes.data_as(C.POINTER(C.c_uint64)), out.size)
    if rc != 0:
        raise KsError(rc, "unpack failed")
    return obj.value, int(elt.value), out


def save(path: str, blob: bytes) -> None:
    with open(path, "wb") as f:
        f.write(blob)


def load(path: str) -> bytes:
    with open(path, "rb") as f:
        return f.read()
