"""The child-process helper of the multi-GPU tests (no GPU): results come
back per rank, and a rank that never reports is killed, not left running."""
import os
import sys
import time

from tests.procs import run_ranks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _echo(rank, world, port, q, tag):
    q.put((rank, (tag, world, port > 0)))


def _stuck(rank, world, port, q, pidq):
    pidq.put(os.getpid())
    if rank == 0:
        q.put((rank, True))
        return
    time.sleep(600)  # never reports


def test_run_ranks_collects_every_rank():
    res = run_ranks(_echo, 3, extra_args=("x",))
    assert res == {r: ("x", 3, True) for r in range(3)}


def test_run_ranks_kills_a_rank_that_never_reports():
    sys.path.insert(0, ROOT)
    holder = {}

    def objs(ctx):
        holder["q"] = ctx.Queue()
        return [holder["q"]]

    t0 = time.time()
    res = run_ranks(_stuck, 2, timeout=5, grace=1, extra_objs=objs)
    assert res == {0: True}
    assert time.time() - t0 < 60
    pids = [holder["q"].get(timeout=10) for _ in range(2)]
    for pid in pids:  # both children are gone (the stuck one was killed)
        try:
            os.kill(pid, 0)
            alive = True
        except ProcessLookupError:
            alive = False
        assert not alive, pid
