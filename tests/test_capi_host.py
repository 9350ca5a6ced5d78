"""The C-ABI library without a GPU: it loads, exports every declared symbol,
and its host-side functions and argument checks behave (no kernel launches)."""
import ctypes as C
import json
import os
import re

import numpy as np
import pytest

from comp390project_b200 import _capi, gen_primes, secret_generate
from comp390project_b200._capi import KS_ERR_INVALID, KS_OK, ks_params
from oracle.oracle import Oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "ks_capi.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ks_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _capi.load()
    names = declared_functions()
    assert len(names) >= 30
    for n in names:
        assert hasattr(lib, n), n
    # and the ctypes table covers all of them
    assert set(names) <= set(_capi.SIGNATURES)


def test_gen_primes_matches_reference_kat():
    with open(os.path.join(ROOT, "tests", "golden", "prime_kat.json")) as f:
        kat = json.load(f)
    for rec in kat:
        assert [int(x) for x in gen_primes(rec["log_n"], rec["bits"])] == rec["primes"]


def test_secret_generator_matches_oracle():
    from tests.ksparams import oracle_for
    o = oracle_for("small")
    for seed, h in [(0, 0), (7, 0), (3, 40), (9, o.N)]:
        assert np.array_equal(secret_generate(o.log_n, seed, h), o.secret(seed, h))


def _params(log_n=13, q=None, p=None):
    q = q if q is not None else gen_primes(13, [60, 40, 40])
    p = p if p is not None else gen_primes(13, [61])
    qb = (C.c_uint64 * len(q))(*[int(x) for x in q])
    pb = (C.c_uint64 * max(1, len(p)))(*([int(x) for x in p] or [0]))
    return ks_params(log_n, len(q), qb, len(p), pb, 0, 1), (qb, pb)


def test_create_rejects_bad_parameters_before_touching_a_device():
    lib = _capi.load()
    h = C.c_void_p()
    assert lib.ks_ctx_create(None, 0, 0, 1, None, C.byref(h)) == KS_ERR_INVALID
    assert "null" in _capi.last_error().lower()
    prm, keep = _params(log_n=11)
    assert lib.ks_ctx_create(C.byref(prm), 0, 0, 1, None, C.byref(h)) == KS_ERR_INVALID
    assert "log_n" in _capi.last_error()
    bad_q = np.array([97, 193], dtype=np.uint64)  # not 1 mod 2N for N = 2^13
    prm, keep = _params(q=bad_q)
    assert lib.ks_ctx_create(C.byref(prm), 0, 0, 1, None, C.byref(h)) == KS_ERR_INVALID
    assert "mod 2N" in _capi.last_error()
    prm, keep = _params()
    assert lib.ks_ctx_create(C.byref(prm), 0, 1, 1, None, C.byref(h)) == KS_ERR_INVALID
    assert lib.ks_ctx_create(C.byref(prm), 0, 0, 2, None, C.byref(h)) != KS_OK
    assert not h.value


def test_null_context_calls_fail_cleanly():
    lib = _capi.load()
    assert lib.ks_relinearize(None, None, 3, None) == KS_ERR_INVALID
    assert lib.ks_rotate(None, None, 3, 1, None) == KS_ERR_INVALID
    assert lib.ks_ntt_forward(None, None, 1, 0, 1, None) == KS_ERR_INVALID
    assert lib.ks_ctx_destroy(None) == KS_ERR_INVALID
    assert lib.ks_key_words(None) == 0
    assert lib.ks_bsgs_workspace_words(None, 3, 1, 4) == 0
    assert lib.ks_bsgs_matmul(None, None, None, 1, 3, 1, 2, 2, 0, 2, None, None, 1, None,
                              None) == KS_ERR_INVALID
    assert lib.ks_reduce_limbs(None, None, 2, 3, None) == KS_ERR_INVALID
    assert lib.ks_rescale(None, None, 3, None, None) == KS_ERR_INVALID
    assert lib.ks_total_launch_count(None) == KS_ERR_INVALID
    assert lib.ks_last_launch_count(None) == KS_ERR_INVALID
    buf = C.create_string_buffer(8)
    assert lib.ks_last_error(None, buf, 0) == KS_ERR_INVALID


def test_nccl_unique_id_needs_no_device():
    from comp390project_b200 import nccl_unique_id
    try:
        a = nccl_unique_id()
    except _capi.KsError as e:  # NCCL bootstrap may be unavailable in a sandbox
        pytest.skip("NCCL bootstrap unavailable here: %s" % e)
    assert len(a) == _capi.KS_NCCL_ID_BYTES


def test_partition_copy_argument_checks_without_a_gpu():
    """The context-free partition copies reject a rank outside [0, n_gpus)
    and return without any CUDA call for a rank that owns no limb."""
    lib = _capi.load()
    assert lib.ks_scatter_ciphertext_to_gpu(None, None, 1, 4, 8, 4, 4, None) == KS_ERR_INVALID
    assert lib.ks_gather_ciphertext_from_gpu(None, None, 1, 4, 8, -1, 4, None) == KS_ERR_INVALID
    assert lib.ks_scatter_ciphertext_to_gpu(None, None, 1, 4, 0, 0, 4, None) == KS_ERR_INVALID
    # rank 3 of 8 owns no limb of a 3-limb ciphertext: nothing to copy
    assert lib.ks_scatter_ciphertext_to_gpu(None, None, 2, 3, 8, 3, 8, None) == KS_OK
    assert lib.ks_gather_ciphertext_from_gpu(None, None, 2, 3, 8, 3, 8, None) == KS_OK
