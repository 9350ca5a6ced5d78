"""Python host side over the C ABI: one ``KsContext`` per GPU / rank.

Device buffers are torch tensors (dtype int64 holding uint64 words, the
PhantomCiphertext layout [poly][limb][N]); torch supplies memory and streams
only, every computation runs in libks_b200.so.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import numpy as np

from . import _capi
from ._capi import (KS_KEY_GALOIS, KS_KEY_RELIN, KS_MODE_INPUT_BROADCAST,
                    KS_MODE_OUTPUT_AGGREGATION, KS_NCCL_ID_BYTES,
                    check, ks_params)


def _torch():
    import torch
    return torch


def _stream_ptr(stream, device) -> Optional[int]:
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream(device)
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def gen_primes(log_n: int, bit_sizes: Sequence[int]) -> np.ndarray:
    """Phantom/SEAL CoeffModulus::Create rule (through the C ABI, host only)."""
    bits = (C.c_int * len(bit_sizes))(*[int(b) for b in bit_sizes])
    out = np.zeros(len(bit_sizes), dtype=np.uint64)
    check(_capi.load().ks_gen_primes(int(log_n), bits, len(bit_sizes),
                                     out.ctypes.data_as(C.POINTER(C.c_uint64))))
    return out


def secret_generate(log_n: int, seed: int, hamming_weight: int = 0) -> np.ndarray:
    out = np.zeros(1 << log_n, dtype=np.int8)
    check(_capi.load().ks_secret_generate(int(log_n), int(seed), int(hamming_weight),
                                          out.ctypes.data_as(C.POINTER(C.c_int8))))
    return out


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(KS_NCCL_ID_BYTES)
    check(_capi.load().ks_nccl_unique_id(buf, KS_NCCL_ID_BYTES))
    return buf.raw


class KsGraph:
    """A captured sequence of hot-path calls (ks_graph_*)."""

    def __init__(self, lib, handle):
        self.lib, self.h = lib, handle

    def launch(self, stream=None, device: int = 0):
        check(self.lib.ks_graph_launch(self.h, _stream_ptr(stream, device)), None)

    def close(self):
        if self.h:
            self.lib.ks_graph_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KsContext:
    """Key-switching context of one device (rank ``rank`` of ``world``)."""

    def __init__(self, log_n: int, q: Sequence[int], p: Sequence[int], device: int = 0,
                 rank: int = 0, world: int = 1, nccl_id: Optional[bytes] = None,
                 mode: int = KS_MODE_INPUT_BROADCAST, max_batch: int = 1,
                 batch_group: int = 1, _handle=None):
        self.lib = _capi.load()
        self.log_n = int(log_n)
        self.N = 1 << self.log_n
        self.q = np.ascontiguousarray(q, dtype=np.uint64)
        self.p = np.ascontiguousarray(p, dtype=np.uint64)
        self.L, self.alpha = len(self.q), len(self.p)
        self.device, self.rank, self.world, self.mode = int(device), int(rank), int(world), mode
        self.h = None
        if _handle is not None:
            self.h = _handle
            return
        prm = self._params(max_batch, batch_group)
        h = C.c_void_p()
        idb = None
        if world > 1:
            if nccl_id is None or len(nccl_id) < KS_NCCL_ID_BYTES:
                raise ValueError("world > 1 needs the NCCL unique id bytes")
            idb = C.create_string_buffer(bytes(nccl_id), KS_NCCL_ID_BYTES)
        check(self.lib.ks_ctx_create(C.byref(prm), self.device, self.rank, self.world, idb,
                                     C.byref(h)))
        self.h = h

    def _params(self, max_batch=1, batch_group=1):
        self._qbuf = (C.c_uint64 * self.L)(*[int(x) for x in self.q])
        self._pbuf = (C.c_uint64 * max(1, self.alpha))(*[int(x) for x in self.p] or [0])
        return ks_params(self.log_n, self.L, self._qbuf, self.alpha, self._pbuf, int(self.mode),
                         int(max_batch), int(batch_group))

    @classmethod
    def create_all(cls, log_n, q, p, devices: Sequence[int], mode=KS_MODE_INPUT_BROADCAST):
        """Single-process multi-GPU (ncclCommInitAll), one context per device."""
        lib = _capi.load()
        proto = cls.__new__(cls)
        proto.q = np.ascontiguousarray(q, dtype=np.uint64)
        proto.p = np.ascontiguousarray(p, dtype=np.uint64)
        proto.L, proto.alpha, proto.log_n, proto.mode = len(proto.q), len(proto.p), int(log_n), mode
        prm = proto._params()
        n = len(devices)
        devs = (C.c_int * n)(*devices)
        hs = (C.c_void_p * n)()
        check(lib.ks_ctx_create_all(C.byref(prm), devs, n, hs))
        return [cls(log_n, q, p, device=devices[i], rank=i, world=n, mode=mode,
                    _handle=C.c_void_p(hs[i])) for i in range(n)]

    @classmethod
    def from_process_group(cls, log_n, q, p, device: Optional[int] = None, group=None,
                           mode=KS_MODE_INPUT_BROADCAST, max_batch=1, batch_group=1):
        """One context per torch.distributed rank; rank 0's NCCL id is broadcast."""
        import torch.distributed as dist
        torch = _torch()
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        if device is None:
            device = torch.cuda.current_device()
        obj = [nccl_unique_id() if rank == 0 else None]
        if world > 1:
            dist.broadcast_object_list(obj, src=0, group=group)
        return cls(log_n, q, p, device=device, rank=rank, world=world,
                   nccl_id=obj[0] if world > 1 else None, mode=mode, max_batch=max_batch,
                   batch_group=batch_group)

    # -- lifecycle -----------------------------------------------------------
    def close(self):
        if self.h is not None:
            self.lib.ks_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        return check(rc, self.h)

    # -- queries -------------------------------------------------------------
    def n_local_limbs(self, total: int) -> int:
        return self._check(self.lib.ks_n_local_limbs(self.h, int(total)))

    def num_digits(self, level_limbs: int) -> int:
        return self._check(self.lib.ks_num_digits(self.h, int(level_limbs)))

    def galois_elt(self, step: int) -> int:
        e = C.c_uint32()
        self._check(self.lib.ks_galois_elt(self.h, int(step), C.byref(e)))
        return int(e.value)

    def key_words(self) -> int:
        return int(self.lib.ks_key_words(self.h))

    def last_launch_count(self) -> int:
        return int(self.lib.ks_last_launch_count(self.h))

    def total_launch_count(self) -> int:
        """Kernel launches of every call since the context was created."""
        return int(self.lib.ks_total_launch_count(self.h))

    # -- CUDA graphs -----------------------------------------------------------
    def graph_capture_begin(self, stream):
        """Starts recording the hot-path calls made on ``stream`` (a torch
        stream or a raw handle; not the legacy default stream)."""
        self._check(self.lib.ks_graph_capture_begin(self.h, _stream_ptr(stream, self.device)))

    def graph_capture_end(self, stream) -> "KsGraph":
        g = C.c_void_p()
        self._check(self.lib.ks_graph_capture_end(self.h, _stream_ptr(stream, self.device),
                                                  C.byref(g)))
        return KsGraph(self.lib, g.value)

    def profile_enable(self, on: bool = True):
        self._check(self.lib.ks_profile_enable(self.h, 1 if on else 0))

    def profile_read(self) -> dict:
        n = int(self.lib.ks_profile_stage_count())
        ms = (C.c_double * n)()
        calls = (C.c_int * n)()
        self._check(self.lib.ks_profile_read(self.h, ms, calls, n))
        return {self.lib.ks_profile_stage_name(i).decode(): (float(ms[i]), int(calls[i]))
                for i in range(n)}

    def set_timeout_ms(self, ms: int):
        self._check(self.lib.ks_set_timeout_ms(self.h, int(ms)))

    # -- keys ----------------------------------------------------------------
    def key_upload(self, kind: int, elt: int, key: np.ndarray):
        key = np.ascontiguousarray(key, dtype=np.uint64)
        self._check(self.lib.ks_key_upload(self.h, kind, int(elt), key.ctypes.data, key.size))

    def key_distribute(self, kind: int, elt: int, full_key=None, root: int = 0, stream=None):
        """Collective: the root passes the full key as a device tensor
        [digits][2][L+alpha][N], the others None; every rank ends with its
        shard (NCCL point-to-point from the root)."""
        ptr = self._ptr(full_key) if full_key is not None else None
        self._check(self.lib.ks_key_distribute(self.h, kind, int(elt), ptr, int(root),
                                               _stream_ptr(stream, self.device)))

    def key_upload_wire(self, blob: bytes):
        """Uploads a key blob of comp390project_b200.wire (validated against
        this context's parameters; the context keeps its shard)."""
        raw = C.create_string_buffer(bytes(blob), len(blob))
        self._check(self.lib.ks_key_upload_wire(self.h, raw, len(blob)))

    def key_upload_device(self, kind: int, elt: int, key, stream=None):
        self._check(self.lib.ks_key_upload_device(self.h, kind, int(elt), self._ptr(key),
                                                  key.numel(), _stream_ptr(stream, self.device)))

    def key_generate(self, kind: int, elt: int, secret: np.ndarray, seed: int, stream=None):
        s = np.ascontiguousarray(secret, dtype=np.int8)
        self._check(self.lib.ks_key_generate(self.h, kind, int(elt), s.ctypes.data, int(seed),
                                             _stream_ptr(stream, self.device)))

    def key_download(self, kind: int, elt: int) -> np.ndarray:
        """The key shard this context holds: [digits][2][limbs][N].  Input
        broadcast (or one GPU): all digits, the cyclic key-basis limbs j % G ==
        rank; output aggregation: the digits d % G == rank, all limbs."""
        beta = (self.L + self.alpha - 1) // self.alpha
        if self.world > 1 and self.mode == KS_MODE_OUTPUT_AGGREGATION:
            digits, limbs = len(range(self.rank, beta, self.world)), self.L + self.alpha
        else:
            digits, limbs = beta, len(range(self.rank, self.L + self.alpha, self.world))
        out = np.zeros((digits, 2, limbs, self.N), dtype=np.uint64)
        self._check(self.lib.ks_key_download(self.h, kind, int(elt), out.ctypes.data, out.size))
        return out

    def key_drop(self, kind: int, elt: int):
        self._check(self.lib.ks_key_drop(self.h, kind, int(elt)))

    # -- hot path ------------------------------------------------------------
    def _ptr(self, t) -> int:
        torch = _torch()
        if not isinstance(t, torch.Tensor):
            raise TypeError("expected a torch tensor")
        if t.dtype not in (torch.int64, torch.uint64):
            raise TypeError("expected int64/uint64 words")
        if not t.is_cuda or t.device.index != self.device:
            raise ValueError("tensor must live on cuda:%d" % self.device)
        if not t.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return t.data_ptr()

    def relinearize(self, ct, level_limbs: int, stream=None):
        self._check(self.lib.ks_relinearize(self.h, self._ptr(ct), int(level_limbs),
                                            _stream_ptr(stream, self.device)))

    def keyswitch_add(self, c, ct, level_limbs: int, kind: int = KS_KEY_RELIN, elt: int = 0,
                      stream=None):
        """ct[0] += ks0(c), ct[1] += ks1(c) for the key (kind, elt)."""
        self._check(self.lib.ks_keyswitch_add(self.h, self._ptr(c), self._ptr(ct),
                                              int(level_limbs), int(kind), int(elt),
                                              _stream_ptr(stream, self.device)))

    def apply_galois(self, ct, level_limbs: int, elt: int, stream=None):
        self._check(self.lib.ks_apply_galois(self.h, self._ptr(ct), int(level_limbs), int(elt),
                                             _stream_ptr(stream, self.device)))

    def apply_galois_noalloc(self, ct, level_limbs: int, elt: int, stream=None):
        """apply_galois without any device allocation on the call: the scratch
        is the library's fixed 16 MiB device array (small parameter sets only;
        calls that overlap on the GPU race)."""
        self._check(self.lib.ks_apply_galois_noalloc(self.h, self._ptr(ct), int(level_limbs),
                                                     int(elt), _stream_ptr(stream, self.device)))

    def rotate(self, ct, level_limbs: int, step: int, stream=None):
        self._check(self.lib.ks_rotate(self.h, self._ptr(ct), int(level_limbs), int(step),
                                       _stream_ptr(stream, self.device)))

    def rotate_batch(self, cts, steps: Sequence[int], level_limbs: int, stream=None):
        n = len(cts)
        ptrs = (C.c_void_p * n)(*[self._ptr(t) for t in cts])
        st = (C.c_int * n)(*[int(s) for s in steps])
        self._check(self.lib.ks_rotate_batch(self.h, ptrs, st, n, int(level_limbs),
                                             _stream_ptr(stream, self.device)))

    def rescale(self, ct, level_limbs: int, out, stream=None):
        """Divide by the last prime and round: ct [2][n_local(Ql)][N] ->
        out [2][n_local(Ql-1)][N]."""
        self._check(self.lib.ks_rescale(self.h, self._ptr(ct), int(level_limbs), self._ptr(out),
                                        _stream_ptr(stream, self.device)))

    def rotate_batch_host(self, host_cts, steps: Sequence[int], level_limbs: int, stream=None):
        """rotate_batch on host tensors (pinned CPU torch tensors or numpy
        uint64 arrays [2][n_local][N]), rotated in place; asynchronous on the
        stream (synchronise before reading them)."""
        n = len(host_cts)

        def hptr(t):
            return t.ctypes.data if isinstance(t, np.ndarray) else t.data_ptr()
        ptrs = (C.c_void_p * n)(*[hptr(t) for t in host_cts])
        st = (C.c_int * n)(*[int(s) for s in steps])
        self._check(self.lib.ks_rotate_batch_host(self.h, ptrs, st, n, int(level_limbs),
                                                  _stream_ptr(stream, self.device)))

    def rotate_hoisted(self, ct, level_limbs: int, steps: Sequence[int], outs, stream=None):
        n = len(steps)
        ptrs = (C.c_void_p * n)(*[self._ptr(t) for t in outs])
        st = (C.c_int * n)(*[int(s) for s in steps])
        self._check(self.lib.ks_rotate_hoisted(self.h, self._ptr(ct), int(level_limbs), st, n,
                                               ptrs, _stream_ptr(stream, self.device)))

    def linear_transform_hoisted(self, ct, level_limbs: int, steps: Sequence[int], diags, out,
                                 stream=None):
        """out = sum_i diags[i] * rotate(ct, steps[i]) with one shared ModUp and
        one ModDown.  diags[i]: NTT-form plaintext in the extended basis, one
        word row per output limb of this rank: [Ql + alpha][N] (Q limbs, then
        P limbs) on one GPU or in output aggregation, the owned Q limbs then the
        owned P limbs in input broadcast."""
        n = len(steps)
        dp = (C.c_void_p * n)(*[self._ptr(t) for t in diags])
        st = (C.c_int * n)(*[int(s) for s in steps])
        self._check(self.lib.ks_linear_transform_hoisted(self.h, self._ptr(ct), int(level_limbs),
                                                         st, n, dp, self._ptr(out),
                                                         _stream_ptr(stream, self.device)))

    def bsgs_workspace_words(self, level_limbs: int, n_in: int, n_baby: int) -> int:
        return int(self.lib.ks_bsgs_workspace_words(self.h, int(level_limbs), int(n_in),
                                                    int(n_baby)))

    def bsgs_matmul(self, xs, level_limbs: int, unit: int, n_baby: int, n_giant: int, pts, ys,
                    workspace, g_range=None, baby=None, stream=None):
        """Block BSGS ciphertext x plaintext product (ks_bsgs_matmul):
        ys[o] = sum_{g in g_range} rot_{g B unit}(sum_i sum_b pts[((o n_in + i) G + g) B + b]
        * rot_{b unit}(xs[i])).  xs, ys: [2][n_local][N]; pts: [n_local][N] NTT-form
        diagonals; baby: optional precomputed rotations, baby[i (B-1) + b - 1] =
        rot_{b unit}(xs[i]); workspace: bsgs_workspace_words(level, n_in, 1 if baby
        else n_baby) words."""
        n_in, n_out = len(xs), len(ys)
        g_lo, g_hi = g_range if g_range is not None else (0, n_giant)
        if len(pts) != n_out * n_in * n_giant * n_baby:
            raise ValueError("pts must hold n_out * n_in * n_giant * n_baby diagonals")
        xp = (C.c_void_p * n_in)(*[self._ptr(t) for t in xs])
        yp = (C.c_void_p * n_out)(*[self._ptr(t) for t in ys])
        pp = (C.c_void_p * len(pts))(*[self._ptr(t) for t in pts])
        bp = None
        if baby is not None:
            if len(baby) != n_in * (n_baby - 1):
                raise ValueError("baby must hold n_in * (n_baby - 1) ciphertexts")
            bp = (C.c_void_p * max(len(baby), 1))(*[self._ptr(t) for t in baby])
        self._check(self.lib.ks_bsgs_matmul(
            self.h, xp, bp, n_in, int(level_limbs), int(unit), int(n_baby), int(n_giant),
            int(g_lo), int(g_hi), pp, yp, n_out, self._ptr(workspace),
            _stream_ptr(stream, self.device)))

    def reduce_limbs(self, x, n_polys: int, level_limbs: int, stream=None):
        """x [n_polys][n_local][N] in place: every word reduced mod its limb's prime."""
        self._check(self.lib.ks_reduce_limbs(self.h, self._ptr(x), int(n_polys),
                                             int(level_limbs), _stream_ptr(stream, self.device)))

    def ntt_forward(self, data, n_limbs: int, first_prime: int = 0, batch: int = 1, stream=None):
        self._check(self.lib.ks_ntt_forward(self.h, self._ptr(data), int(n_limbs),
                                            int(first_prime), int(batch),
                                            _stream_ptr(stream, self.device)))

    def ntt_inverse(self, data, n_limbs: int, first_prime: int = 0, batch: int = 1, stream=None):
        self._check(self.lib.ks_ntt_inverse(self.h, self._ptr(data), int(n_limbs),
                                            int(first_prime), int(batch),
                                            _stream_ptr(stream, self.device)))

    def scatter_limbs(self, global_buf, local_buf, n_polys: int, total_limbs: int, stream=None):
        self._check(self.lib.ks_scatter_limbs(self.h, self._ptr(global_buf), self._ptr(local_buf),
                                              int(n_polys), int(total_limbs),
                                              _stream_ptr(stream, self.device)))

    def gather_limbs(self, local_buf, global_buf, n_polys: int, total_limbs: int, stream=None):
        self._check(self.lib.ks_gather_limbs(self.h, self._ptr(local_buf), self._ptr(global_buf),
                                             int(n_polys), int(total_limbs),
                                             _stream_ptr(stream, self.device)))

    def allgather_limbs(self, local_buf, full_buf, total_limbs: int, stream=None):
        self._check(self.lib.ks_allgather_limbs(self.h, self._ptr(local_buf), self._ptr(full_buf),
                                                int(total_limbs),
                                                _stream_ptr(stream, self.device)))


__all__ = ["KsContext", "gen_primes", "secret_generate", "nccl_unique_id", "KS_KEY_RELIN",
           "KS_KEY_GALOIS"]
