"""Multi-GPU key switching through the C ABI: one process per GPU, NCCL
communicators created by the library from an id broadcast over a gloo
process group.  Input broadcast: every rank holds its cyclic share of the
limbs and the gathered result must equal the single-process CPU oracle bit
for bit.  Output aggregation: every rank holds the whole ciphertext and its
digits of the key, and every rank's result must equal the oracle.  Rank 0
evaluates the oracle references and every rank compares a digest of its
result with rank 0's, so the CPU oracle runs once per check, not once per
rank.  Skipped when fewer than two GPUs are visible."""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, q, name, mode):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # the ranks share the host's cores for the oracle's OpenMP loops
    os.environ["OMP_NUM_THREADS"] = str(max(1, (os.cpu_count() or 1) // world))
    import hashlib

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from comp390project_b200 import (KS_KEY_GALOIS, KS_KEY_RELIN, KsContext,
                                         KS_MODE_OUTPUT_AGGREGATION)
        from tests.ksparams import oracle_for, split, CFG3, SMALL
        cfg = {"small": SMALL, "cfg3": CFG3}[name]
        o = oracle_for(name)
        log_n, qs, ps = split(cfg)
        N, L = o.N, o.L
        Ql = L
        oa = mode == "oa"
        ctx = KsContext.from_process_group(log_n, qs, ps, device=rank, max_batch=2, batch_group=2,
                                           mode=KS_MODE_OUTPUT_AGGREGATION if oa else 0)
        ctx.set_timeout_ms(60000)
        s = o.secret(11, 64 if name == "small" else 192)
        steps = [1, 3]
        keys = {}
        for st in steps:
            e = o.galois_elt(st)
            keys[st] = o.keygen_galois(s, e, 500 + st)
        ctx.key_upload(KS_KEY_GALOIS, o.galois_elt(1), keys[1])  # host upload of the shard
        ctx.key_generate(KS_KEY_GALOIS, o.galois_elt(3), s, 503)  # device generation of the shard
        rk = o.keygen_relin(s, 600)
        ctx.key_upload(KS_KEY_RELIN, 0, rk)
        rng = np.random.default_rng(77)
        cts = [np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=N, dtype=np.uint64)
                                   for j in range(Ql)]) for _ in range(2)]) for _ in steps + [1]]
        c3 = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=N, dtype=np.uint64)
                                 for j in range(Ql)]) for _ in range(3)])
        mine = list(range(rank, Ql, world)) if not oa else list(range(Ql))

        def local(ct):
            return torch.from_numpy(np.ascontiguousarray(ct[:, mine]).view(np.int64)).cuda()

        def gather(t, n_polys):
            if oa:  # every rank holds the whole result
                return t.cpu()[:n_polys].numpy().view(np.uint64)
            h = torch.zeros((n_polys, (Ql + world - 1) // world, N), dtype=torch.int64)
            h[:, :len(mine)] = t.cpu()[:n_polys]
            out = [torch.zeros_like(h) for _ in range(world)]
            dist.all_gather(out, h)
            full = np.zeros((n_polys, Ql, N), dtype=np.uint64)
            for j in range(Ql):
                full[:, j] = out[j % world][:, j // world].numpy().view(np.uint64)
            return full

        def check(full, ref):
            """Every rank's full result must equal rank 0's (a digest over
            gloo), and rank 0 alone evaluates the oracle reference `ref()`."""
            h = int.from_bytes(hashlib.sha256(np.ascontiguousarray(full).tobytes()).digest()[:8],
                               "little", signed=True)
            t = torch.tensor([h], dtype=torch.int64)
            dist.broadcast(t, 0)
            same = int(t.item()) == h
            return same and (rank != 0 or np.array_equal(full, ref()))

        ok = True
        # single rotation
        d = local(cts[0])
        ctx.rotate(d, Ql, steps[0])
        torch.cuda.synchronize()
        ok &= check(gather(d, 2), lambda: o.apply_galois(cts[0], Ql, o.galois_elt(1), keys[1]))
        # batch of three: a group of two on lane 0 (grouped all-gathers /
        # all-reduce) and a group of one on lane 1 (its own split communicator)
        bsteps = steps + [1]
        ds = [local(c) for c in cts]
        ctx.rotate_batch(ds, bsteps, Ql)
        torch.cuda.synchronize()
        for c, dd, st in zip(cts, ds, bsteps):
            ok &= check(gather(dd, 2),
                        lambda c=c, st=st: o.apply_galois(c, Ql, o.galois_elt(st), keys[st]))
        # relinearisation
        d3 = local(c3)
        ctx.relinearize(d3, Ql)
        torch.cuda.synchronize()
        ok &= check(gather(d3, 2), lambda: o.relinearize(c3, Ql, rk))
        # a lower level (short last digit)
        Ql2 = Ql - 3
        c2 = cts[0][:, :Ql2]
        mine2 = list(range(rank, Ql2, world)) if not oa else list(range(Ql2))
        d2 = torch.from_numpy(np.ascontiguousarray(c2[:, mine2]).view(np.int64)).cuda()
        ctx.rotate(d2, Ql2, 1)
        torch.cuda.synchronize()
        if oa:
            full2 = d2.cpu().numpy().view(np.uint64)
        else:
            h = torch.zeros((2, (Ql2 + world - 1) // world, N), dtype=torch.int64)
            h[:, :len(mine2)] = d2.cpu()
            outs = [torch.zeros_like(h) for _ in range(world)]
            dist.all_gather(outs, h)
            full2 = np.zeros((2, Ql2, N), dtype=np.uint64)
            for j in range(Ql2):
                full2[:, j] = outs[j % world][:, j // world].numpy().view(np.uint64)
        ok &= check(full2, lambda: o.apply_galois(c2, Ql2, o.galois_elt(1), keys[1]))
        # key distribution: rank 0 holds the full key on its device, every
        # rank receives its shard over NCCL point-to-point
        ctx.key_drop(KS_KEY_GALOIS, o.galois_elt(1))
        full = torch.from_numpy(keys[1].view(np.int64).copy()).cuda() if rank == 0 else None
        ctx.key_distribute(KS_KEY_GALOIS, o.galois_elt(1), full, root=0)
        dk = local(cts[0])
        ctx.rotate(dk, Ql, 1)
        torch.cuda.synchronize()
        ok &= check(gather(dk, 2), lambda: o.apply_galois(cts[0], Ql, o.galois_elt(1), keys[1]))
        # rescale: the owner of the last limb broadcasts it (input broadcast)
        mine3 = list(range(rank, Ql - 1, world)) if not oa else list(range(Ql - 1))
        dr = local(cts[1])
        out3 = torch.zeros((2, len(mine3), N), dtype=torch.int64, device="cuda")
        ctx.rescale(dr, Ql, out3)
        torch.cuda.synchronize()
        want3 = o.rescale(cts[1], Ql)[:, mine3]
        ok &= np.array_equal(out3.cpu().numpy().view(np.uint64), want3)
        # ks_allgather_limbs: every rank ends with the limbs in sequential
        # order, as allgather_c2_limbs + reorder_gathered_to_sequential give
        # (input_broadcast.cu:45-111); a rank without limbs still joins
        seq = cts[0][1]
        mine_ag = list(range(rank, Ql, world))
        loc = (torch.from_numpy(np.ascontiguousarray(seq[mine_ag]).view(np.int64)).cuda()
               if mine_ag else torch.zeros(2, dtype=torch.int64, device="cuda"))
        full_ag = torch.zeros((Ql, N), dtype=torch.int64, device="cuda")
        ctx.allgather_limbs(loc, full_ag, Ql)
        torch.cuda.synchronize()
        ok &= np.array_equal(full_ag.cpu().numpy().view(np.uint64), seq)
        ctx.close()
        q.put((rank, bool(ok)))
    except Exception as e:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 8])
@pytest.mark.parametrize("mode", ["ib", "oa"])
@pytest.mark.parametrize("name", ["small", "cfg3"])
def test_multi_gpu_keyswitch_bitexact(name, mode, world, cuda_device):
    """world 8 at config 3 output aggregation: 7 digits over 8 ranks, rank 7
    contributes a zero partial sum."""
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    from tests.procs import run_ranks
    # every worker sets a 60 s collective deadline, so a failed rank ends the
    # others' collectives with an error instead of a hang
    res = run_ranks(_worker, world, extra_args=(name, mode))
    assert len(res) == world and all(v is True for v in res.values()), res
