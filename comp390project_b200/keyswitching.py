"""The reference's key-switching interface, over libks_b200.so.

Same names, argument meaning and error behaviour as hkanpak21/Comp390Project
``namespace nexus_multi_gpu`` (src/multi_gpu/keyswitching/*.cuh,
src/multi_gpu/comm/nccl_comm.cuh), with torch device tensors in place of
PhantomCiphertext buffers:

* a ciphertext is a ``Ciphertext`` (int64 words, layout [poly][limb][N],
  limbs of this rank only when n_gpus > 1, cyclic partition);
* calls return after the work is queued and, like the reference, synchronise
  the context's stream before returning (``sync=False`` keeps them async);
* failures raise ``KsError`` (the reference throws std::runtime_error).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

from ._capi import KS_KEY_GALOIS, KS_KEY_RELIN, KS_MODE_INPUT_BROADCAST
from .context import KsContext


@dataclass
class Ciphertext:
    """PhantomCiphertext-style view (paper/code_study.tex:351-364)."""
    data: "object"              # torch.Tensor int64 [size][n_local][N] on the rank's device
    coeff_modulus_size: int      # Ql, Q limbs of the level (all ranks together)
    poly_modulus_degree: int
    scale: float = 1.0
    is_ntt_form: bool = True

    @property
    def size(self) -> int:
        return int(self.data.shape[0])

    def chain_index(self, L: int) -> int:
        """Phantom chain index (1 at the top level): Ql = L - chain_index + 1."""
        return L - self.coeff_modulus_size + 1


class MultiGpuContext:
    """One KsContext per GPU (reference MultiGpuContext, nccl_comm.cuh:42-54).

    ``create(dev_ids, ...)`` is the single-process form (ncclCommInitAll);
    ``from_process_group(...)`` makes the one-rank-per-process form."""

    def __init__(self, contexts: List[KsContext]):
        self.ctxs = contexts
        self.n_gpus = contexts[0].world if contexts else 0
        self.device_ids = [c.device for c in contexts]

    @classmethod
    def create(cls, dev_ids: Sequence[int], log_n, q, p, mode=KS_MODE_INPUT_BROADCAST):
        if len(dev_ids) == 1:
            return cls([KsContext(log_n, q, p, device=dev_ids[0], mode=mode)])
        return cls(KsContext.create_all(log_n, q, p, list(dev_ids), mode=mode))

    @classmethod
    def from_process_group(cls, log_n, q, p, device=None, mode=KS_MODE_INPUT_BROADCAST,
                           max_batch=1):
        return cls([KsContext.from_process_group(log_n, q, p, device=device, mode=mode,
                                                 max_batch=max_batch)])

    def ctx(self, gpu_id: int) -> KsContext:
        if len(self.ctxs) == 1:
            return self.ctxs[0]
        return self.ctxs[gpu_id]

    def destroy(self):
        for c in self.ctxs:
            c.close()
        self.ctxs = []


def _sync(ctx: KsContext, sync: bool):
    if sync:
        import torch
        torch.cuda.current_stream(ctx.device).synchronize()


def keyswitching_input_broadcast(ctx: MultiGpuContext, gpu_id: int, encrypted: Ciphertext,
                                 local_c2, relin_keys=None, total_limbs: Optional[int] = None,
                                 degree: Optional[int] = None, n_gpus: Optional[int] = None,
                                 sync: bool = True):
    """Relinearise: encrypted.data[0:2] += KS(local_c2) with the relinearisation
    key (input_broadcast.cuh:68-78).  ``relin_keys`` may be a host array in the
    full key layout (uploaded once) or None when the context already holds it."""
    k = ctx.ctx(gpu_id)
    if relin_keys is not None:
        k.key_upload(KS_KEY_RELIN, 0, relin_keys)
    Ql = total_limbs if total_limbs is not None else encrypted.coeff_modulus_size
    k.keyswitch_add(local_c2, encrypted.data, Ql, KS_KEY_RELIN, 0)
    _sync(k, sync)


def rotation_input_broadcast(ctx: MultiGpuContext, gpu_id: int, encrypted: Ciphertext,
                             galois_keys=None, galois_elt: int = 3,
                             total_limbs: Optional[int] = None, degree: Optional[int] = None,
                             n_gpus: Optional[int] = None, sync: bool = True):
    """apply_galois on this rank's limbs of ``encrypted`` (input_broadcast.cuh:86-97)."""
    k = ctx.ctx(gpu_id)
    if galois_keys is not None:
        k.key_upload(KS_KEY_GALOIS, galois_elt, galois_keys)
    Ql = total_limbs if total_limbs is not None else encrypted.coeff_modulus_size
    k.apply_galois(encrypted.data, Ql, galois_elt)
    _sync(k, sync)


def keyswitching_output_aggregation(ctx: MultiGpuContext, gpu_id: int, encrypted: Ciphertext,
                                    c2, relin_keys=None, n_gpus: Optional[int] = None,
                                    sync: bool = True):
    """Output-aggregation relinearisation (output_aggregation.cuh:69-77); the
    context decides the collective plan it was created with."""
    keyswitching_input_broadcast(ctx, gpu_id, encrypted, c2, relin_keys, sync=sync)


def dist_rescale_to_next(ctx: MultiGpuContext, gpu_id: int, encrypted: Ciphertext, out,
                         sync: bool = True):
    """Rescale by the last prime (distributed_eval.cu:265-273, there a gather to
    GPU 0): ``out`` [2][n_local(Ql-1)][N] receives this rank's limbs of
    round(encrypted / q_last)."""
    k = ctx.ctx(gpu_id)
    k.rescale(encrypted.data, encrypted.coeff_modulus_size, out)
    _sync(k, sync)


def allgather_c2_limbs(ctx: MultiGpuContext, gpu_id: int, local_c2, full_c2, local_limbs: int,
                       total_limbs: int, degree: Optional[int] = None, sync: bool = True):
    """All limbs of c2 on every rank in sequential order (input_broadcast.cu:75-111
    plus the reorder of :45-69)."""
    k = ctx.ctx(gpu_id)
    k.allgather_limbs(local_c2, full_c2, total_limbs)
    _sync(k, sync)


def scatter_ciphertext_to_gpu(ctx: MultiGpuContext, gpu_id: int, global_buf, local_buf,
                              n_polys: int, total_limbs: int, sync: bool = True):
    """rns_partition.cuh:165-174."""
    k = ctx.ctx(gpu_id)
    k.scatter_limbs(global_buf, local_buf, n_polys, total_limbs)
    _sync(k, sync)


def gather_ciphertext_from_gpu(ctx: MultiGpuContext, gpu_id: int, local_buf, global_buf,
                               n_polys: int, total_limbs: int, sync: bool = True):
    """rns_partition.cuh:182-191."""
    k = ctx.ctx(gpu_id)
    k.gather_limbs(local_buf, global_buf, n_polys, total_limbs)
    _sync(k, sync)


class Evaluator:
    """Phantom-evaluator names on top of one context (rotate_vector /
    relinearize / apply_galois, all in place)."""

    def __init__(self, ctx: KsContext):
        self.ctx = ctx

    def rotate_vector_inplace(self, ct: Ciphertext, step: int):
        self.ctx.rotate(ct.data, ct.coeff_modulus_size, step)

    def relinearize_inplace(self, ct: Ciphertext):
        if ct.size != 3:
            raise ValueError("relinearize expects a size-3 ciphertext")
        self.ctx.relinearize(ct.data, ct.coeff_modulus_size)
        ct.data = ct.data[:2]

    def apply_galois_inplace(self, ct: Ciphertext, galois_elt: int):
        self.ctx.apply_galois(ct.data, ct.coeff_modulus_size, galois_elt)

    def rescale_to_next(self, ct: Ciphertext) -> Ciphertext:
        """Phantom rescale_to_next (the reference's dist_rescale_to_next_inplace,
        distributed_eval.cu:265-273): a new ciphertext one level down, scale
        divided by the dropped prime."""
        import torch
        Ql = ct.coeff_modulus_size
        n_out = self.ctx.n_local_limbs(Ql - 1) if self.ctx.world > 1 and \
            self.ctx.mode == KS_MODE_INPUT_BROADCAST else Ql - 1
        out = torch.empty((2, n_out, ct.poly_modulus_degree), dtype=torch.int64,
                          device=ct.data.device)
        self.ctx.rescale(ct.data[:2].contiguous(), Ql, out)
        q_last = float(self.ctx.q[Ql - 1])
        return Ciphertext(out, Ql - 1, ct.poly_modulus_degree, ct.scale / q_last)

    def rotate_hoisted(self, ct: Ciphertext, steps: Sequence[int]) -> List[Ciphertext]:
        """Rotations of one ciphertext by every step with one shared ModUp."""
        import torch
        outs = [torch.empty_like(ct.data[:2]) for _ in steps]
        self.ctx.rotate_hoisted(ct.data[:2].contiguous(), ct.coeff_modulus_size, steps, outs)
        return [Ciphertext(o, ct.coeff_modulus_size, ct.poly_modulus_degree, ct.scale)
                for o in outs]

    def rotate_batch_inplace(self, cts: Sequence[Ciphertext], steps: Sequence[int]):
        if not cts:
            return
        Ql = cts[0].coeff_modulus_size
        if any(c.coeff_modulus_size != Ql for c in cts):
            raise ValueError("batched rotations need ciphertexts of one level")
        self.ctx.rotate_batch([c.data for c in cts], steps, Ql)
