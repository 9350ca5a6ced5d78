"""Cyclic RNS-limb partition and the per-rank key-switch layout (host logic).

Mirrors the reference's src/multi_gpu/partition/rns_partition.cuh:29-107
(same names, same meaning): limb j lives on rank j % G at local slot j // G,
buffers are [poly][limb][coeff].  The functions after the reference set
describe which key-basis limbs a rank owns in libks_b200.so (Q limbs and
special P limbs continue one cyclic sequence over the key basis) and the
rank-grouped order of an all-gather, exactly as the C++ context lays them out.
"""
from __future__ import annotations

from typing import List


def owner_of_limb(limb_j: int, n_gpus: int) -> int:
    """rns_partition.cuh:29-31."""
    return limb_j % n_gpus


def local_index_of_limb(limb_j: int, n_gpus: int) -> int:
    """rns_partition.cuh:38-40."""
    return limb_j // n_gpus


def global_limb_index(gpu_id: int, local_idx: int, n_gpus: int) -> int:
    """rns_partition.cuh:46-48."""
    return local_idx * n_gpus + gpu_id


def n_local_limbs(gpu_id: int, n_gpus: int, total_limbs: int) -> int:
    """rns_partition.cuh:55-60."""
    if gpu_id >= total_limbs:
        return 0
    return (total_limbs - gpu_id - 1) // n_gpus + 1


def limbs_for_gpu(gpu_id: int, n_gpus: int, total_limbs: int) -> List[int]:
    """rns_partition.cuh:67-73."""
    return list(range(gpu_id, total_limbs, n_gpus))


def local_buf_offset(poly_i: int, local_limb_loc: int, local_n_limbs: int, degree: int) -> int:
    """rns_partition.cuh:90-95 (word offset)."""
    return (poly_i * local_n_limbs + local_limb_loc) * degree


def global_buf_offset(poly_i: int, limb_j: int, total_limbs: int, degree: int) -> int:
    """rns_partition.cuh:102-107 (word offset)."""
    return (poly_i * total_limbs + limb_j) * degree


# ---------------------------------------------------------------------------
# Key-switch layout of libks_b200.so
# ---------------------------------------------------------------------------
def max_local(total_limbs: int, n_gpus: int) -> int:
    """Slots per rank of a padded all-gather (input_broadcast.cu:85)."""
    return (total_limbs + n_gpus - 1) // n_gpus


def gathered_slot(limb_j: int, n_gpus: int, total_limbs: int) -> int:
    """Slot of limb j in the rank-grouped all-gather buffer [G][max_local][N]
    (the order reorder_gathered_to_sequential undoes, input_broadcast.cu:45-69)."""
    return (limb_j % n_gpus) * max_local(total_limbs, n_gpus) + limb_j // n_gpus


def owned_key_limbs(rank: int, world: int, L: int, alpha: int) -> List[int]:
    """Key-basis limbs (Q primes 0..L-1, then P primes L..L+alpha-1) a rank keeps."""
    return list(range(rank, L + alpha, world))


def owned_output_limbs(rank: int, world: int, Ql: int, L: int, alpha: int) -> List[int]:
    """Indices into the extended basis (Q limbs of the level, then P limbs) of
    the key-switch outputs a rank computes: its Q limbs, then the P limbs whose
    key-basis index L + i it owns."""
    q = list(range(rank, Ql, world))
    p = [Ql + i for i in range(alpha) if (L + i) % world == rank]
    return q + p


def digits(Ql: int, alpha: int) -> List[List[int]]:
    """The Q limbs of each decomposition digit at a level with Ql limbs."""
    return [list(range(d * alpha, min((d + 1) * alpha, Ql))) for d in range((Ql + alpha - 1) // alpha)]
