"""BSGS ciphertext x plaintext matmul through the C ABI (ks_bsgs_matmul):
baby-step rotations hoisted per input, plaintext products of up to four giant
steps per pass, giant-step key switches accumulated in the extended basis
with one ModDown per output.  Every output word must equal the CPU oracle's
composition (ork_bsgs_matmul) exactly, for the whole product, for a
giant-step sub-range with caller-supplied baby steps, and for the giant-step
split over two GPUs (all-gather of the baby steps, integer all-reduce of the
partial products; the oracle summed over the same ranges, since each range
rounds in its own ModDown); the product decodes to X W."""
import functools
import os
import sys

import numpy as np
import pytest

from tests.matmul_case import case, decode_outputs, split_reference

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _dev(a, device=0):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64).copy()).to(f"cuda:{device}")


def _host(t):
    return t.cpu().numpy().view(np.uint64)


@functools.lru_cache(maxsize=None)
def _want(g_range=None, n_baby=None):
    c = case(n_baby)
    lay = c["lay"]
    return c["o"].bsgs_matmul(c["xs"], c["Ql"], lay.unit, lay.n_baby, lay.n_giant, c["pts"],
                              c["keys"], g_range=g_range)


def _setup(device=0, keys=True, n_baby=None):
    from comp390project_b200 import KS_KEY_GALOIS, KsContext
    from tests.ksparams import SMALL, split
    c = case(n_baby)
    log_n, q, p = split(SMALL)
    ctx = KsContext(log_n, q, p, device=device, max_batch=2)
    if keys:
        for st, k in c["keys"].items():
            ctx.key_upload(KS_KEY_GALOIS, ctx.galois_elt(st), k)
    xs = [_dev(x, device) for x in c["xs"]]
    pts = [_dev(pt, device) for pt in c["pts"]]
    lay = c["lay"]
    ys = torch.zeros((lay.n_out, 2, c["Ql"], 1 << log_n), dtype=torch.int64,
                     device=f"cuda:{device}")
    return c, ctx, xs, pts, ys


@pytest.mark.parametrize("n_baby", [None, 64])
def test_bsgs_matmul_matches_oracle(n_baby, cuda_device):
    c, ctx, xs, pts, ys = _setup(n_baby=n_baby)
    lay, Ql = c["lay"], c["Ql"]
    work = torch.empty(ctx.bsgs_workspace_words(Ql, lay.n_in, lay.n_baby), dtype=torch.int64,
                       device="cuda")
    ctx.bsgs_matmul(xs, Ql, lay.unit, lay.n_baby, lay.n_giant, pts, [ys[o] for o in range(lay.n_out)],
                    work)
    torch.cuda.synchronize()
    got = _host(ys)
    assert np.array_equal(got, _want(None, n_baby)), "BSGS product differs from the oracle"
    for x, h in zip(xs, c["xs"]):
        assert np.array_equal(_host(x), h), "input modified"
    Y = decode_outputs(c, got)
    assert np.abs(Y - c["X"] @ c["W"]).max() < 1e-4
    ctx.close()


def test_bsgs_matmul_subrange_with_supplied_baby_steps(cuda_device):
    c, ctx, xs, pts, ys = _setup()
    lay, Ql = c["lay"], c["Ql"]
    baby = []
    for x in xs:
        outs = [torch.zeros_like(x) for _ in lay.baby_steps()]
        ctx.rotate_hoisted(x, Ql, lay.baby_steps(), outs)
        baby += outs
    work = torch.empty(ctx.bsgs_workspace_words(Ql, lay.n_in, 1), dtype=torch.int64,
                       device="cuda")
    ctx.bsgs_matmul(xs, Ql, lay.unit, lay.n_baby, lay.n_giant, pts, [ys[o] for o in range(lay.n_out)],
                    work, g_range=(2, 7), baby=baby)
    torch.cuda.synchronize()
    assert np.array_equal(_host(ys), _want((2, 7)))
    ctx.close()


def test_giant_parallel_single_rank(cuda_device):
    from comp390project_b200 import matmul
    c, ctx, xs, pts, ys = _setup()
    matmul.matmul_giant_parallel(ctx, xs, c["Ql"], c["lay"], pts, ys)
    torch.cuda.synchronize()
    assert np.array_equal(_host(ys), _want())
    ctx.close()


def test_reduce_limbs(cuda_device):
    c, ctx, xs, pts, ys = _setup(keys=False)
    o, Ql = c["o"], c["Ql"]
    rng = np.random.default_rng(9)
    x = rng.integers(0, 1 << 63, size=(3, Ql, o.N), dtype=np.uint64) * np.uint64(2) + \
        rng.integers(0, 2, size=(3, Ql, o.N), dtype=np.uint64)
    d = _dev(x)
    ctx.reduce_limbs(d, 3, Ql)
    torch.cuda.synchronize()
    q = np.array([int(o.moduli[j]) for j in range(Ql)], dtype=np.uint64)[None, :, None]
    assert np.array_equal(_host(d), x % q)
    ctx.close()


def test_bsgs_matmul_rejects_missing_key_and_alias(cuda_device):
    from comp390project_b200 import KsError
    c, ctx, xs, pts, ys = _setup(keys=False)
    lay, Ql = c["lay"], c["Ql"]
    work = torch.empty(ctx.bsgs_workspace_words(Ql, lay.n_in, lay.n_baby), dtype=torch.int64,
                       device="cuda")
    with pytest.raises(KsError):
        ctx.bsgs_matmul(xs, Ql, lay.unit, lay.n_baby, lay.n_giant, pts,
                        [ys[o] for o in range(lay.n_out)], work)
    with pytest.raises(KsError):
        ctx.bsgs_matmul(xs, Ql, lay.unit, lay.n_baby, lay.n_giant, pts, [xs[0], ys[1]], work)
    with pytest.raises(KsError):
        ctx.bsgs_matmul(xs, Ql, lay.unit, lay.n_baby, lay.n_giant, pts,
                        [ys[o] for o in range(lay.n_out)], work, g_range=(3, 3))
    ctx.close()


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from comp390project_b200 import matmul
        c, ctx, xs, pts, ys = _setup(device=rank)
        matmul.matmul_giant_parallel(ctx, xs, c["Ql"], c["lay"], pts, ys)
        torch.cuda.synchronize()
        ok = bool(np.array_equal(_host(ys), split_reference(c, world)))
        ctx.close()
        q.put((rank, ok))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_giant_parallel_two_gpus(cuda_device):
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    from tests.procs import run_ranks
    res = run_ranks(_worker, world)
    assert len(res) == world and all(v is True for v in res.values()), res


def test_bsgs_matmul_config3_ring_reduced_layer(cuda_device):
    """The BSGS product on config 5's own ring (config 3: N = 2^16, Ql = 35,
    alpha = 5, dnum = 7) with a reduced layer: 8192 tokens give F = 4
    features per ciphertext, so d_in = d_out = 4 is one input and one output
    ciphertext with B = G = 2 (one hoisted baby step, one giant step, four
    diagonals).  Ciphertexts and diagonals are uniform residues; every output
    word must equal the oracle's ork_bsgs_matmul."""
    from comp390project_b200 import KS_KEY_GALOIS, KsContext, matmul
    from tests.ksparams import CFG3, oracle_for, split
    o = oracle_for("cfg3")
    log_n, q, p = split(CFG3)
    Ql, N = 35, o.N
    lay = matmul.layout(N // 2, 8192, 4, 4, n_baby=2)
    assert (lay.n_in, lay.n_out, lay.n_baby, lay.n_giant) == (1, 1, 2, 2)
    s = o.secret(4, 192)
    steps = lay.baby_steps() + lay.giant_steps()
    keys = {st: o.keygen_galois(s, o.galois_elt(st), 700 + k) for k, st in enumerate(steps)}
    rng = np.random.default_rng(44)
    x = np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=N, dtype=np.uint64)
                            for j in range(Ql)]) for _ in range(2)])
    pts = [np.stack([rng.integers(0, int(o.moduli[j]), size=N, dtype=np.uint64)
                     for j in range(Ql)]) for _ in range(lay.n_diagonals)]
    want = o.bsgs_matmul([x], Ql, lay.unit, lay.n_baby, lay.n_giant, pts, keys)
    ctx = KsContext(log_n, q, p, device=0, max_batch=2)
    for st, k in keys.items():
        ctx.key_upload(KS_KEY_GALOIS, ctx.galois_elt(st), k)
    xd = _dev(x)
    pd = [_dev(pt) for pt in pts]
    ys = torch.zeros((1, 2, Ql, N), dtype=torch.int64, device="cuda")
    work = torch.empty(ctx.bsgs_workspace_words(Ql, 1, lay.n_baby), dtype=torch.int64,
                       device="cuda")
    ctx.bsgs_matmul([xd], Ql, lay.unit, lay.n_baby, lay.n_giant, pd, [ys[0]], work)
    torch.cuda.synchronize()
    assert np.array_equal(_host(ys), want), "config-3 ring BSGS product differs from the oracle"
    ctx.close()
