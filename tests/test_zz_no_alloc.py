"""The allocation-free rotation, ks_apply_galois_noalloc, through the C ABI.

It exists for callers that may not allocate device memory at call time (a
fixed memory budget, or HBM reserved up front by the host application); its
scratch is the library's fixed device array instead of the context's arena.
Its output must equal ks_apply_galois word for word (the tests' tolerance for
this integer path is exact equality), on two calls in a row, since every call
reuses the same array.  This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from tests.ksparams import CFG1, CFG3, SMALL, oracle_for, split

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _ctx(cfg):
    from comp390project_b200 import KsContext
    log_n, q, p = split(cfg)
    return KsContext(log_n, q, p, device=0)


@pytest.mark.parametrize("name,cfg,Ql", [("cfg1", CFG1, 3), ("small", SMALL, 7), ("small", SMALL, 5)])
def test_noalloc_rotation_matches_apply_galois_twice(name, cfg, Ql, cuda_device):
    from comp390project_b200 import _capi
    o = oracle_for(name)
    ctx = _ctx(cfg)
    s = o.secret(21)
    lib = _capi.load()
    for call, step in enumerate((1, 3)):
        elt = o.galois_elt(step)
        ctx.key_upload(1, elt, o.keygen_galois(s, elt, 900 + step))
        rng = np.random.default_rng(100 + call)
        ct = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                                 for j in range(Ql)]) for _ in range(2)])
        a = torch.from_numpy(ct.view(np.int64).copy()).cuda()
        b = a.clone()
        stream = torch.cuda.current_stream().cuda_stream
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        rc = lib.ks_apply_galois_noalloc(ctx.h, C.c_void_p(a.data_ptr()), Ql, elt,
                                         C.c_void_p(stream))
        assert rc == 0, _capi.last_error(ctx.h)
        torch.cuda.synchronize()
        if call > 0:  # after the first call has set up the device address
            assert torch.cuda.mem_get_info()[0] == free0, "the call allocated device memory"
        rc = lib.ks_apply_galois(ctx.h, C.c_void_p(b.data_ptr()), Ql, elt, C.c_void_p(stream))
        assert rc == 0, _capi.last_error(ctx.h)
        torch.cuda.synchronize()
        assert torch.equal(a, b), "call %d differs from ks_apply_galois" % call
    ctx.close()


def test_noalloc_rejects_parameter_sets_beyond_the_array(cuda_device):
    from comp390project_b200 import _capi
    o = oracle_for("cfg3")
    ctx = _ctx(CFG3)
    ct = torch.zeros((2, 35, o.N), dtype=torch.int64, device="cuda")
    rc = _capi.load().ks_apply_galois_noalloc(ctx.h, C.c_void_p(ct.data_ptr()), 35,
                                              o.galois_elt(1), None)
    assert rc == _capi.KS_ERR_UNSUPPORTED
    assert "scratch" in _capi.last_error(ctx.h)
    ctx.close()
