"""World-size-2 (and 3) process tests of the sharded key-switch host logic on
CPU with the gloo backend.

Each rank keeps its cyclic share of the limbs (rank g owns limb j iff
j % G == g), exactly as libks_b200.so lays a rank out, and the ranks exchange
data with real torch.distributed collectives:
  input broadcast:     all-gather of the coefficient-form input limbs (padded
                       to ceil(Ql/G) slots, rank-grouped), limb-local ModUp and
                       inner product, all-gather of the special-prime limbs,
                       limb-local ModDown;
  output aggregation:  every rank holds the whole input and the digits
                       d % G == g; it converts and extends only its digits'
                       limbs, forms the partial inner product over all
                       extended limbs, and a uint64 all-reduce + mod reduce
                       gives every rank the whole cx; ModDown on every rank
                       (the library's plan, after the reference's
                       keyswitching_output_aggregation).
The result (gathered, for input broadcast) must equal the single-process
oracle key switch bit for bit.  The arithmetic is the CPU oracle's; what is under test is the
partition, padding, slot order and collective plan."""
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


def _allgather_np(arr):
    t = torch.from_numpy(np.ascontiguousarray(arr).view(np.int64))
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [o.numpy().view(np.uint64) for o in out]


def _worker(rank, world, port, mode, result_q):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from comp390project_b200 import partition as P
        from tests.ksparams import oracle_for
        o = oracle_for("small")
        N, L, a = o.N, o.L, o.alpha
        Ql = 7
        QlP = Ql + a
        s = o.secret(5)
        elt = o.galois_elt(3)
        key = o.keygen_galois(s, elt, 77)
        rng = np.random.default_rng(123)  # same input on every rank
        c = np.stack([rng.integers(0, int(o.moduli[j]), size=N, dtype=np.uint64)
                      for j in range(Ql)])
        ref = o.keyswitch(c, Ql, key)
        idx = list(range(Ql)) + [L + i for i in range(a)]  # key-basis index of QlP limb j
        G, g = world, rank
        digits = P.digits(Ql, a)
        beta = len(digits)
        if mode == "oa":
            # 1. the limbs of this rank's digits to coefficient form (whole input here)
            mine_d = list(range(g, beta, G))
            dl = [j for d in mine_d for j in digits[d]]
            coef = np.zeros((Ql, N), dtype=np.uint64)
            if dl:
                coef[dl] = o.ntt(c[dl], dl, inverse=True)
            t = np.zeros((beta, QlP, N), dtype=np.uint64)
            for d in mine_d:
                D = digits[d]
                for j in range(QlP):
                    if j in D:
                        t[d, j] = c[j]
                    else:
                        t[d, j] = o.ntt(o.bconv(coef[D], D, [idx[j]]), [idx[j]])[0]
            part = o.inner_product(t, Ql, key)  # [2][QlP][N], partial over my digits
            # 2. uint64 all-reduce (G q < 2^64: the integer sum is exact) + mod q
            tt = torch.from_numpy(np.ascontiguousarray(part).view(np.int64))
            dist.all_reduce(tt, op=dist.ReduceOp.SUM)
            q_of = np.array([int(o.moduli[idx[j]]) for j in range(QlP)],
                            dtype=np.uint64)[None, :, None]
            cx = tt.numpy().view(np.uint64) % q_of
            # 3. ModDown of both polys on every rank: the whole result everywhere
            full = np.stack([o.moddown(cx[p], Ql) for p in range(2)])
            result_q.put((rank, bool(np.array_equal(full, ref))))
            return
        my_q = P.limbs_for_gpu(g, G, Ql)
        # 1. own limbs to coefficient form, padded rank-grouped all-gather
        ml = P.max_local(Ql, G)
        send = np.zeros((ml, N), dtype=np.uint64)
        if my_q:
            send[:len(my_q)] = o.ntt(c[my_q], my_q, inverse=True)
        gathered = _allgather_np(send)
        coef = np.stack([gathered[P.owner_of_limb(j, G)][P.local_index_of_limb(j, G)]
                         for j in range(Ql)])
        assert np.array_equal(coef, o.ntt(c, list(range(Ql)), inverse=True))

        def extend(d, j):
            """t[d][j] in NTT form from the all-gathered coefficients."""
            D = digits[d]
            if j in D:
                return c[j]
            y = o.bconv(coef[D], D, [idx[j]])
            return o.ntt(y, [idx[j]])[0]

        outs = P.owned_output_limbs(g, G, Ql, L, a)
        t = np.zeros((beta, QlP, N), dtype=np.uint64)
        for d in range(beta):
            for j in outs:
                t[d, j] = extend(d, j)
        cx_full = o.inner_product(t, Ql, key)  # limb-wise: only owned rows are used
        mine = {j: cx_full[:, j] for j in outs}
        # 2. special-prime limbs of cx to every rank
        own_p = [j for j in mine if j >= Ql]
        maxp = max(len([i for i in range(a) if (L + i) % G == r]) for r in range(G))
        sendp = np.zeros((max(1, maxp), 2, N), dtype=np.uint64)
        for k, j in enumerate(own_p):
            sendp[k] = mine[j]
        gp = _allgather_np(sendp)
        # 3. ModDown of my Q limbs
        out = {}
        for p in range(2):
            cx_poly = np.zeros((QlP, N), dtype=np.uint64)
            for j in mine:
                cx_poly[j] = mine[j][p]
            for i in range(a):
                owner = (L + i) % G
                k = sum(1 for i2 in range(i) if (L + i2) % G == owner)
                cx_poly[Ql + i] = gp[owner][k][p]
            md = o.moddown(cx_poly, Ql)
            for j in my_q:
                out.setdefault(j, [None, None])[p] = md[j]
        # 4. collect on every rank and compare with the single-process result
        sendo = np.zeros((ml, 2, N), dtype=np.uint64)
        for k, j in enumerate(my_q):
            sendo[k, 0], sendo[k, 1] = out[j]
        go = _allgather_np(sendo)
        full = np.zeros((2, Ql, N), dtype=np.uint64)
        for j in range(Ql):
            full[:, j] = go[P.owner_of_limb(j, G)][P.local_index_of_limb(j, G)]
        ok = bool(np.array_equal(full, ref))
        result_q.put((rank, ok))
    except Exception as e:  # report instead of hanging the parent
        result_q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,mode", [(2, "ib"), (3, "ib"), (2, "oa"), (3, "oa")])
def test_sharded_keyswitch_plan_matches_single_process(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, ok = q.get(timeout=240)
        results[r] = ok
    for p in procs:
        p.join(timeout=60)
    assert all(v is True for v in results.values()), results


def _id_worker(rank, world, port, result_q):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from comp390project_b200 import nccl_unique_id
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        blobs = [None] * world
        dist.all_gather_object(blobs, obj[0])
        result_q.put((rank, all(b == blobs[0] for b in blobs) and len(blobs[0]) == 128))
    except Exception as e:
        result_q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_nccl_id_reaches_every_rank():
    """The rank-0 NCCL id travels to every rank over the process group, as
    KsContext.from_process_group does before ks_ctx_create."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_id_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
    if any(isinstance(v, str) and "KS_ERR_NCCL" in v for v in res.values()):
        pytest.skip("NCCL bootstrap unavailable here: %s" % res)
    assert all(v is True for v in res.values()), res
