"""Failure detection on the GPU path: a rank that never joins a collective.

Two processes on two GPUs (NVLS off, plain peer transport).  Both complete a
rotation; then rank 1 leaves between steps (no kernel or collective of its
in flight) and never joins the next one.  Rank 0's next rotation enqueues an
all-gather that cannot complete: the context's collective deadline
(ks_set_timeout_ms) must abort its communicators so the stream drains, and
every later call must fail with KS_ERR_TIMEOUT instead of hanging.  Skipped
when fewer than two GPUs are visible."""
import os
import sys
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, q, left):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from comp390project_b200 import KS_KEY_GALOIS, KsContext, KsError
        from comp390project_b200._capi import KS_ERR_TIMEOUT
        from tests.ksparams import SMALL, oracle_for, split
        o = oracle_for("small")
        log_n, qs, ps = split(SMALL)
        ctx = KsContext.from_process_group(log_n, qs, ps, device=rank)
        ctx.set_timeout_ms(1500)
        s = o.secret(3, 64)
        e = o.galois_elt(1)
        ctx.key_upload(KS_KEY_GALOIS, e, o.keygen_galois(s, e, 9))
        Ql = o.L
        rng = np.random.default_rng(4)
        ct = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                                 for j in range(Ql)]) for _ in range(2)])
        mine = list(range(rank, Ql, world))
        d = torch.from_numpy(np.ascontiguousarray(ct[:, mine]).view(np.int64)).cuda()
        ctx.rotate(d, Ql, 1)  # a step both ranks complete
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 1:  # leaves between steps and never joins the next collective
            left.wait(timeout=120)
            ctx.close()
            q.put((rank, True))
            return
        t0 = time.time()
        ctx.rotate(d, Ql, 1)  # its all-gather waits for rank 1
        torch.cuda.synchronize()  # drains once the deadline aborts the communicators
        waited = time.time() - t0
        code = None
        try:
            ctx.rotate(d, Ql, 1)
        except KsError as err:
            code = err.code
        left.set()
        ctx.close()
        q.put((rank, (waited < 60.0 and code == KS_ERR_TIMEOUT, waited, code)))
    except Exception:
        import traceback
        left.set()
        q.put((rank, traceback.format_exc()))


def test_rank_that_never_joins_times_out(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from tests.procs import run_ranks
    res = run_ranks(_worker, 2, extra_objs=lambda ctx: [ctx.Event()])
    assert res.get(1) is True, res
    assert isinstance(res.get(0), tuple) and res[0][0], res
