"""CUDA graph capture and replay of hot-path calls through the C ABI
(ks_graph_*): a captured batch of rotations replays to the same words as the
eager calls and as the CPU oracle; capture itself runs nothing; a call that
fails during capture closes the capture."""
import numpy as np
import pytest

from tests.ksparams import SMALL, oracle_for, split

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _setup():
    from comp390project_b200 import KS_KEY_GALOIS, KsContext
    o = oracle_for("small")
    log_n, q, p = split(SMALL)
    ctx = KsContext(log_n, q, p, device=0, max_batch=2)
    s = o.secret(5, 64)
    keys = {}
    for st in (1, 2):
        e = o.galois_elt(st)
        keys[st] = o.keygen_galois(s, e, 40 + st)
        ctx.key_upload(KS_KEY_GALOIS, e, keys[st])
    rng = np.random.default_rng(9)
    Ql = o.L
    cts = [np.stack([np.stack([rng.integers(0, int(o.moduli[j]), size=o.N, dtype=np.uint64)
                               for j in range(Ql)]) for _ in range(2)]) for _ in range(2)]
    return o, ctx, keys, cts, Ql


def _dev(a):
    return torch.from_numpy(a.view(np.int64).copy()).cuda()


def test_graph_replay_matches_eager_and_oracle(cuda_device):
    o, ctx, keys, cts, Ql = _setup()
    steps = [1, 2]
    eager = [_dev(c) for c in cts]
    ctx.rotate_batch(eager, steps, Ql)  # also the first (uncaptured) call of this kind
    torch.cuda.synchronize()
    want1 = [o.apply_galois(c, Ql, o.galois_elt(st), keys[st]) for c, st in zip(cts, steps)]
    for e, w in zip(eager, want1):
        assert np.array_equal(e.cpu().numpy().view(np.uint64), w)

    bufs = [_dev(c) for c in cts]
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    ctx.graph_capture_begin(stream)
    ctx.rotate_batch(bufs, steps, Ql, stream=stream)
    g = ctx.graph_capture_end(stream)
    stream.synchronize()
    for b, c in zip(bufs, cts):  # capture ran nothing
        assert np.array_equal(b.cpu().numpy().view(np.uint64), c)
    g.launch(stream)
    stream.synchronize()
    for b, w in zip(bufs, want1):
        assert np.array_equal(b.cpu().numpy().view(np.uint64), w)
    g.launch(stream)  # a second replay rotates again
    stream.synchronize()
    want2 = [o.apply_galois(w, Ql, o.galois_elt(st), keys[st]) for w, st in zip(want1, steps)]
    for b, w in zip(bufs, want2):
        assert np.array_equal(b.cpu().numpy().view(np.uint64), w)
    g.close()
    ctx.close()


def test_failed_call_closes_the_capture(cuda_device):
    from comp390project_b200 import KsError
    o, ctx, keys, cts, Ql = _setup()
    buf = _dev(cts[0])
    ctx.rotate(buf, Ql, 1)
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    ctx.graph_capture_begin(stream)
    with pytest.raises(KsError):
        ctx.rotate(buf, Ql, 5, stream=stream)  # no key for step 5
    # the capture is closed: a new one can start and the stream runs work again
    ctx.graph_capture_begin(stream)
    ctx.rotate(buf, Ql, 1, stream=stream)
    g = ctx.graph_capture_end(stream)
    g.launch(stream)
    stream.synchronize()
    want = o.apply_galois(o.apply_galois(cts[0], Ql, o.galois_elt(1), keys[1]), Ql,
                          o.galois_elt(1), keys[1])
    assert np.array_equal(buf.cpu().numpy().view(np.uint64), want)
    g.close()
    ctx.close()
