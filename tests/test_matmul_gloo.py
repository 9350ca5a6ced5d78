"""World-size-2 and 3 process test (gloo, CPU) of the multi-GPU BSGS matmul
plan, ``matmul.matmul_giant_parallel``: the baby-step rotations are split
over the ranks and all-gathered, each rank computes the partial product of
its giant-step range, and the partial products are summed by an int64
all-reduce and reduced mod q.  A stand-in context does the arithmetic with
the CPU oracle and checks that the baby-step rotations it is handed after the
all-gather are the right ones in the right order; every rank's result must
equal the single-process oracle product word for word."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _np(t):
    return t.numpy().view(np.uint64)


class OracleCtx:
    """CPU stand-in for a one-GPU KsContext (the calls matmul_giant_parallel
    makes), computing with the oracle."""
    world = 1

    def __init__(self, c):
        self.c, self.o = c, c["o"]
        self.q = np.ascontiguousarray(self.o.moduli[:self.o.L], dtype=np.uint64)

    def _rot(self, x, Ql, steps):
        o, keys = self.o, self.c["keys"]
        return o.rotate_hoisted(_np(x), Ql, [o.galois_elt(s) for s in steps],
                                [keys[s] for s in steps])

    def rotate_hoisted(self, ct, Ql, steps, outs, stream=None):
        for t, w in zip(outs, self._rot(ct, Ql, steps)):
            t.copy_(torch.from_numpy(w.view(np.int64)))

    def bsgs_workspace_words(self, Ql, n_in, n_baby):
        return 2

    def bsgs_matmul(self, xs, Ql, unit, B, G, pts, ys, work, g_range=None, baby=None,
                    stream=None):
        assert baby is not None and len(baby) == len(xs) * (B - 1)
        for i, x in enumerate(xs):
            want = self._rot(x, Ql, [b * unit for b in range(1, B)])
            for b in range(1, B):
                assert np.array_equal(_np(baby[i * (B - 1) + b - 1]), want[b - 1]), \
                    "gathered baby step (%d, %d) differs" % (i, b)
        y = self.o.bsgs_matmul([_np(x) for x in xs], Ql, unit, B, G, [_np(p) for p in pts],
                               self.c["keys"], g_range=g_range)
        for t, w in zip(ys, y):
            t.copy_(torch.from_numpy(w.view(np.int64)))

    def reduce_limbs(self, x, n_polys, Ql):
        a = _np(x).reshape(n_polys, Ql, -1) % self.q[None, :Ql, None]
        x.copy_(torch.from_numpy(a.view(np.int64)).reshape(x.shape))


def _worker(rank, world, port, n_baby, result_q):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from comp390project_b200 import matmul
        from tests.matmul_case import case, split_reference
        c = case(n_baby)
        lay, Ql, o = c["lay"], c["Ql"], c["o"]
        xs = [torch.from_numpy(x.view(np.int64).copy()) for x in c["xs"]]
        pts = [torch.from_numpy(p.view(np.int64).copy()) for p in c["pts"]]
        ys = torch.zeros((lay.n_out, 2, Ql, o.N), dtype=torch.int64)
        matmul.matmul_giant_parallel(OracleCtx(c), xs, Ql, lay, pts, ys)
        # the oracle over the same giant-step ranges (one ModDown per range), summed
        want = split_reference(c, world)
        result_q.put((rank, bool(np.array_equal(_np(ys), want))))
    except Exception:
        import traceback
        result_q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_baby", [(2, None), (3, None), (2, 64)])
def test_giant_parallel_plan_gloo(world, n_baby):
    """(2, 64): G = 1, so rank 1 has no giant step and contributes zeros."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_baby, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(v is True for v in res.values()), res
