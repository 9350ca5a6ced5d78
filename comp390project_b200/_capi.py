"""ctypes binding of libks_b200.so (the C ABI in include/ks_capi.h).

There is no fallback: if the library is missing or does not load, importing
this module raises.  Build it with ``python -m comp390project_b200.build``
(or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

KS_OK = 0
KS_ERR_INVALID = -1
KS_ERR_CUDA = -2
KS_ERR_NCCL = -3
KS_ERR_NO_KEY = -4
KS_ERR_UNSUPPORTED = -5
KS_ERR_ALLOC = -6
KS_ERR_TIMEOUT = -7

KS_KEY_RELIN = 0
KS_KEY_GALOIS = 1
KS_MODE_INPUT_BROADCAST = 0
KS_MODE_OUTPUT_AGGREGATION = 1
KS_WIRE_RELIN_KEY = 1
KS_WIRE_GALOIS_KEY = 2
KS_WIRE_CIPHERTEXT = 3
KS_NCCL_ID_BYTES = 128

_ERR_NAMES = {
    KS_ERR_INVALID: "KS_ERR_INVALID", KS_ERR_CUDA: "KS_ERR_CUDA", KS_ERR_NCCL: "KS_ERR_NCCL",
    KS_ERR_NO_KEY: "KS_ERR_NO_KEY", KS_ERR_UNSUPPORTED: "KS_ERR_UNSUPPORTED",
    KS_ERR_ALLOC: "KS_ERR_ALLOC", KS_ERR_TIMEOUT: "KS_ERR_TIMEOUT",
}


class KsError(RuntimeError):
    """A negative status from the C ABI, with the library's message."""

    def __init__(self, code: int, msg: str):
        super().__init__("%s (%d): %s" % (_ERR_NAMES.get(code, "KS_ERR"), code, msg))
        self.code = code


class ks_params(C.Structure):
    _fields_ = [
        ("log_n", C.c_uint32),
        ("n_q", C.c_int),
        ("q", C.POINTER(C.c_uint64)),
        ("n_p", C.c_int),
        ("p", C.POINTER(C.c_uint64)),
        ("mode", C.c_int),
        ("max_batch", C.c_int),
        ("group", C.c_int),
    ]


_P = C.c_void_p
_I = C.c_int
_U32 = C.c_uint32
_U64 = C.c_uint64
_SZ = C.c_size_t
_u64p = C.POINTER(C.c_uint64)

SIGNATURES = {
    "ks_gen_primes": (_I, [_U32, C.POINTER(C.c_int), _I, _u64p]),
    "ks_secret_generate": (_I, [_U32, _U64, _I, C.POINTER(C.c_int8)]),
    "ks_nccl_unique_id": (_I, [_P, _SZ]),
    "ks_ctx_create": (_I, [C.POINTER(ks_params), _I, _I, _I, _P, C.POINTER(_P)]),
    "ks_ctx_create_all": (_I, [C.POINTER(ks_params), C.POINTER(C.c_int), _I, C.POINTER(_P)]),
    "ks_ctx_destroy": (_I, [_P]),
    "ks_last_error": (_I, [_P, C.c_char_p, _SZ]),
    "ks_set_timeout_ms": (_I, [_P, _I]),
    "ks_n_local_limbs": (_I, [_P, _I]),
    "ks_owner_of_limb": (_I, [_P, _I]),
    "ks_num_digits": (_I, [_P, _I]),
    "ks_galois_elt": (_I, [_P, _I, C.POINTER(C.c_uint32)]),
    "ks_key_words": (_SZ, [_P]),
    "ks_wire_size": (_SZ, [C.POINTER(ks_params), _I, _I, _I]),
    "ks_wire_pack": (_I, [C.POINTER(ks_params), _I, _U32, _I, _I, _u64p, _P, _SZ]),
    "ks_wire_unpack": (_I, [C.POINTER(ks_params), _P, _SZ, C.POINTER(C.c_int),
                            C.POINTER(C.c_uint32), C.POINTER(C.c_int), C.POINTER(C.c_int),
                            _u64p, _SZ]),
    "ks_key_upload_wire": (_I, [_P, _P, _SZ]),
    "ks_key_distribute": (_I, [_P, _I, _U32, _P, _I, _P]),
    "ks_key_upload": (_I, [_P, _I, _U32, _P, _SZ]),
    "ks_key_upload_device": (_I, [_P, _I, _U32, _P, _SZ, _P]),
    "ks_key_generate": (_I, [_P, _I, _U32, _P, _U64, _P]),
    "ks_key_download": (_I, [_P, _I, _U32, _P, _SZ]),
    "ks_key_drop": (_I, [_P, _I, _U32]),
    "ks_relinearize": (_I, [_P, _P, _I, _P]),
    "ks_keyswitch_add": (_I, [_P, _P, _P, _I, _I, _U32, _P]),
    "ks_apply_galois": (_I, [_P, _P, _I, _U32, _P]),
    "ks_apply_galois_noalloc": (_I, [_P, _P, _I, _U32, _P]),
    "ks_rotate": (_I, [_P, _P, _I, _I, _P]),
    "ks_rotate_batch": (_I, [_P, C.POINTER(_P), C.POINTER(C.c_int), _I, _I, _P]),
    "ks_rotate_hoisted": (_I, [_P, _P, _I, C.POINTER(C.c_int), _I, C.POINTER(_P), _P]),
    "ks_rotate_batch_host": (_I, [_P, C.POINTER(_P), C.POINTER(C.c_int), _I, _I, _P]),
    "ks_rescale": (_I, [_P, _P, _I, _P, _P]),
    "ks_linear_transform_hoisted": (_I, [_P, _P, _I, C.POINTER(C.c_int), _I, C.POINTER(_P),
                                         _P, _P]),
    "ks_bsgs_workspace_words": (_SZ, [_P, _I, _I, _I]),
    "ks_bsgs_matmul": (_I, [_P, C.POINTER(_P), C.POINTER(_P), _I, _I, _I, _I, _I, _I, _I,
                            C.POINTER(_P), C.POINTER(_P), _I, _P, _P]),
    "ks_reduce_limbs": (_I, [_P, _P, _I, _I, _P]),
    "ks_ntt_forward": (_I, [_P, _P, _I, _I, _I, _P]),
    "ks_ntt_inverse": (_I, [_P, _P, _I, _I, _I, _P]),
    "ks_scatter_limbs": (_I, [_P, _P, _P, _I, _I, _P]),
    "ks_gather_limbs": (_I, [_P, _P, _P, _I, _I, _P]),
    "ks_allgather_limbs": (_I, [_P, _P, _P, _I, _P]),
    "ks_scatter_ciphertext_to_gpu": (_I, [_P, _P, _SZ, _SZ, _SZ, _I, _I, _P]),
    "ks_gather_ciphertext_from_gpu": (_I, [_P, _P, _SZ, _SZ, _SZ, _I, _I, _P]),
    "ks_last_launch_count": (_I, [_P]),
    "ks_total_launch_count": (C.c_longlong, [_P]),
    "ks_graph_capture_begin": (_I, [_P, _P]),
    "ks_graph_capture_end": (_I, [_P, _P, C.POINTER(_P)]),
    "ks_graph_launch": (_I, [_P, _P]),
    "ks_graph_destroy": (_I, [_P]),
    "ks_profile_enable": (_I, [_P, _I]),
    "ks_profile_stage_count": (_I, []),
    "ks_profile_stage_name": (C.c_char_p, [_I]),
    "ks_profile_read": (_I, [_P, C.POINTER(C.c_double), C.POINTER(C.c_int), _I]),
}

_lib = None


def lib_path() -> str:
    return _build.LIB


def load(build_if_needed: bool = True):
    """Loads the library (building it first when sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    if build_if_needed and _build.needs_build():
        _build.build()
    if not os.path.exists(_build.LIB):
        raise ImportError("libks_b200.so is not built (%s); run __graft_entry__.build()" % _build.LIB)
    L = C.CDLL(_build.LIB)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error(ctx=None) -> str:
    buf = C.create_string_buffer(1024)
    load().ks_last_error(ctx, buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, ctx=None) -> int:
    if rc < 0:
        raise KsError(rc, last_error(ctx))
    return rc
