"""One child process per rank for the multi-GPU tests: results come back on
a queue; whatever the outcome, every child this helper started is joined,
and killed (by its own handle) if it is still alive after the grace period,
so a stuck rank cannot keep the test run or its GPU."""
import queue as _queue
import socket


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def run_ranks(target, world, extra_args=(), timeout=300, grace=60, extra_objs=None):
    """Runs target(rank, world, port, q, *extra) in `world` spawned processes
    and returns {rank: result} for the ranks that reported within `timeout`
    seconds (in total).  extra_objs(ctx) may build shared objects (events)
    passed after q."""
    import time

    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    objs = tuple(extra_objs(ctx)) if extra_objs else ()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + objs + tuple(extra_args))
             for r in range(world)]
    res = {}
    try:
        for p in procs:
            p.start()
        deadline = time.time() + timeout
        while len(res) < world:
            left = deadline - time.time()
            if left <= 0:
                break
            try:
                r, v = q.get(timeout=left)
            except _queue.Empty:
                break
            res[r] = v
    finally:
        for p in procs:
            p.join(timeout=grace)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    return res
