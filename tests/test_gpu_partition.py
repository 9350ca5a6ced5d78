"""The cyclic-partition copies on the GPU against the reference's own kernels.

ks_scatter_ciphertext_to_gpu / ks_gather_ciphertext_from_gpu (and the
context-bound ks_scatter_limbs / ks_gather_limbs) must move exactly the words
that the reference's kernel_scatter_limbs / kernel_gather_limbs move
(src/multi_gpu/partition/rns_partition.cu:26-80, compiled from the reference
tree into oracle/_ref by `make -C oracle ref`), for every rank g of G = 1..8
at config-3 shapes (2 polys x 35 limbs x 2^16), and on ragged cases (odd
degree, ranks that own no limb, 40 limbs).  Where oracle/_ref was not built
the expectation is the index formula of rns_partition.cuh:29-107 evaluated
on the host."""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_partition.so")


def _ref():
    if not os.path.exists(REF_SO):
        return None
    lib = C.CDLL(REF_SO)
    sz, p = C.c_size_t, C.c_void_p
    for name in ("ref_scatter", "ref_gather"):
        f = getattr(lib, name)
        f.restype = C.c_int
        f.argtypes = [p, p, sz, sz, sz, C.c_int, C.c_int]
    return lib


def _expected_local(glob, g, G):
    """rns_partition.cuh: limb loc*G + g of every poly at local slot loc."""
    return glob[:, g::G]


CASES = [(2, 35, 1 << 16, G) for G in range(1, 9)] + [
    (2, 40, 1 << 16, 8),   # extended basis at G = 8: 5 limbs per rank
    (3, 7, 4097, 8),       # odd degree (scalar path), rank 7 owns no limb
    (1, 1, 1000, 3),       # one limb: ranks 1 and 2 own nothing
]


@pytest.mark.parametrize("n_polys,total,degree,G", CASES)
def test_scatter_gather_match_reference_kernels(n_polys, total, degree, G, cuda_device):
    from comp390project_b200 import _capi
    lib = _capi.load()
    ref = _ref()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(total * 131 + G)
    glob = torch.randint(-2 ** 62, 2 ** 62, (n_polys, total, degree), generator=gen,
                         device="cuda", dtype=torch.int64)
    for g in range(G):
        nl = len(range(g, total, G))
        # scatter
        loc = torch.full((n_polys, max(nl, 1), degree), -1, dtype=torch.int64, device="cuda")
        rc = lib.ks_scatter_ciphertext_to_gpu(C.c_void_p(glob.data_ptr()),
                                              C.c_void_p(loc.data_ptr()), n_polys, total,
                                              degree, g, G, None)
        assert rc == 0, _capi.last_error(None)
        torch.cuda.synchronize()
        if nl:
            assert torch.equal(loc[:, :nl], _expected_local(glob, g, G)), (g, G)
        if ref is not None and nl:
            loc_r = torch.full_like(loc, -1)
            assert ref.ref_scatter(glob.data_ptr(), loc_r.data_ptr(), n_polys, total, degree,
                                   g, G) == 0
            assert torch.equal(loc, loc_r), ("scatter differs from the reference", g, G)
        # gather back into a buffer of sentinels: only rank g's limbs change
        src = torch.randint(-2 ** 62, 2 ** 62, loc.shape, generator=gen, device="cuda",
                            dtype=torch.int64)
        out = torch.full_like(glob, 7)
        rc = lib.ks_gather_ciphertext_from_gpu(C.c_void_p(src.data_ptr()),
                                               C.c_void_p(out.data_ptr()), n_polys, total,
                                               degree, g, G, None)
        assert rc == 0, _capi.last_error(None)
        torch.cuda.synchronize()
        want = torch.full_like(glob, 7)
        if nl:
            want[:, g::G] = src[:, :nl]
        assert torch.equal(out, want), (g, G)
        if ref is not None and nl:
            out_r = torch.full_like(glob, 7)
            assert ref.ref_gather(src.data_ptr(), out_r.data_ptr(), n_polys, total, degree,
                                  g, G) == 0
            assert torch.equal(out, out_r), ("gather differs from the reference", g, G)


def test_context_scatter_gather_round_trip(cuda_device):
    """ks_scatter_limbs / ks_gather_limbs of a one-GPU context (rank 0 of 1)
    are the identity copy of the whole ciphertext."""
    from comp390project_b200 import KsContext
    from tests.ksparams import SMALL, split
    log_n, q, p = split(SMALL)
    ctx = KsContext(log_n, q, p, device=0)
    N, L = 1 << log_n, len(q)
    glob = torch.randint(0, 2 ** 40, (2, L, N), device="cuda", dtype=torch.int64)
    loc = torch.zeros_like(glob)
    ctx.scatter_limbs(glob, loc, 2, L)
    back = torch.zeros_like(glob)
    ctx.gather_limbs(loc, back, 2, L)
    torch.cuda.synchronize()
    assert torch.equal(loc, glob) and torch.equal(back, glob)
    ctx.close()


def test_partition_copy_rejects_bad_rank(cuda_device):
    from comp390project_b200 import _capi
    lib = _capi.load()
    a = torch.zeros(16, dtype=torch.int64, device="cuda")
    rc = lib.ks_scatter_ciphertext_to_gpu(C.c_void_p(a.data_ptr()), C.c_void_p(a.data_ptr()),
                                          1, 2, 8, 2, 2, None)
    assert rc == _capi.KS_ERR_INVALID
