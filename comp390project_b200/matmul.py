"""Encrypted activations times a plaintext weight matrix by BSGS diagonals.

This is the BERT-layer matmul that NEXUS runs: activations X [T][d_in]
(encrypted), weights W [d_in][d_out] (plaintext), Y = X W.  The reference
describes it only as multiply_plain + add_many + rescale per output column
(src/benchmarks/bert_matmul_pipeline.cu:7-15), and NEXUS's packing code is
absent from it, so this module defines the packing:

* Column-major blocks.  With S slots per ciphertext and T tokens, a
  ciphertext holds F = S / T features.  Activation block i (features
  [iF, (i+1)F)) is ciphertext i, slot f*T + t = X[t][iF + f].  The output
  blocks of Y use the same packing.
* A rotation by u = T slots moves every token's feature index by one,
  cyclically within the block.  So
      Y_o = sum_i sum_{k < F} d_{o,i,k} (.) rot_{k u}(X_i),
      d_{o,i,k}[f*T + t] = W[iF + (f + k) mod F][oF + f].
* Baby and giant steps: k = g B + b with F = B G, and
      Y_o = sum_g rot_{g B u}( sum_i sum_b rot_{-g B u}(d_{o,i,gB+b}) (.) rot_{b u}(X_i) ).
  This needs n_in (B - 1) baby-step rotations, shared by all outputs and
  hoisted per input, and n_out (G - 1) giant-step rotations.
  ``KsContext.bsgs_matmul`` (ks_bsgs_matmul) evaluates the formula.
  ``diagonals`` produces the pre-rotated diagonals in the order it reads them:
  pts[((o n_in + i) G + g) B + b].

The plaintext encoder (slot vectors -> NTT-form plaintexts at scale Delta) is
the caller's, as in the reference, where Phantom's CKKSEncoder does it.

Multi-GPU split (``matmul_giant_parallel``).  Every rank holds whole
ciphertexts and a one-GPU context.  The n_in (B - 1) baby-step rotations are
split evenly over the ranks and all-gathered over NCCL.  Each rank takes a
contiguous range of giant steps for every output block (``giant_ranges``) and
computes a partial product.  The partial products are summed by an integer
all-reduce and then reduced mod q (``ks_reduce_limbs``).  The weight matrix's
output columns are the attention heads (64 features each); in this packing
an output block carries F / 64 heads.  A literal split by head would repeat
every baby step on every rank, so the split is by giant step instead: the
heads' diagonals are divided over the GPUs, and each rank's rotations,
plaintext products and weight traffic fall by the world size.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence, Tuple

import numpy as np


@dataclass(frozen=True)
class MatmulLayout:
    """Shapes of one packed matmul: T tokens, F features per ciphertext, n_in /
    n_out ciphertexts of activations / outputs, rotation unit u = T, and the
    baby / giant split F = B G."""
    slots: int
    tokens: int
    feats: int
    n_in: int
    n_out: int
    unit: int
    n_baby: int
    n_giant: int

    @property
    def n_diagonals(self) -> int:
        return self.n_out * self.n_in * self.n_giant * self.n_baby

    def baby_steps(self) -> List[int]:
        return [b * self.unit for b in range(1, self.n_baby)]

    def giant_steps(self) -> List[int]:
        return [g * self.n_baby * self.unit for g in range(1, self.n_giant)]


def layout(slots: int, tokens: int, d_in: int, d_out: int, n_baby: int | None = None
           ) -> MatmulLayout:
    """Packing of a [tokens][d_in] x [d_in][d_out] product into ciphertexts of
    `slots` slots.  Each dimension must be a multiple of F = slots / tokens,
    which must be a power of two.  The default B = 2^ceil(log2(F) / 2)
    balances baby and giant steps."""
    if slots % tokens:
        raise ValueError("tokens must divide the slot count")
    F = slots // tokens
    if F & (F - 1):
        raise ValueError("features per ciphertext must be a power of two")
    if d_in % F or d_out % F:
        raise ValueError("d_in and d_out must be multiples of %d" % F)
    if n_baby is None:
        n_baby = 1 << ((F.bit_length() - 1 + 1) // 2)
    if F % n_baby:
        raise ValueError("n_baby must divide the features per ciphertext")
    return MatmulLayout(slots, tokens, F, d_in // F, d_out // F, tokens, n_baby, F // n_baby)


def pack(X: np.ndarray, lay: MatmulLayout) -> np.ndarray:
    """X [T][n_in F] -> slot vectors [n_in][slots], slot f T + t = X[t][iF + f]."""
    X = np.asarray(X)
    if X.shape != (lay.tokens, lay.n_in * lay.feats):
        raise ValueError("X must be [%d][%d]" % (lay.tokens, lay.n_in * lay.feats))
    blk = X.reshape(lay.tokens, lay.n_in, lay.feats)      # [t][i][f]
    return np.ascontiguousarray(blk.transpose(1, 2, 0)).reshape(lay.n_in, lay.slots)


def unpack(vecs: np.ndarray, lay: MatmulLayout) -> np.ndarray:
    """Slot vectors [n_out][slots] -> Y [T][n_out F] (inverse of pack)."""
    v = np.asarray(vecs).reshape(lay.n_out, lay.feats, lay.tokens)   # [o][f][t]
    return np.ascontiguousarray(v.transpose(2, 0, 1)).reshape(lay.tokens, lay.n_out * lay.feats)


def diagonals(W: np.ndarray, lay: MatmulLayout) -> np.ndarray:
    """W [n_in F][n_out F] -> the pre-rotated diagonals [n_diagonals][slots] in
    the order pts[((o n_in + i) G + g) B + b] = rot_{-g B u}(d_{o,i,gB+b})."""
    W = np.asarray(W)
    F, T, B, G = lay.feats, lay.tokens, lay.n_baby, lay.n_giant
    if W.shape != (lay.n_in * F, lay.n_out * F):
        raise ValueError("W must be [%d][%d]" % (lay.n_in * F, lay.n_out * F))
    f = np.arange(F)
    out = np.empty((lay.n_out, lay.n_in, G, B, lay.slots), dtype=W.dtype)
    for o in range(lay.n_out):
        for i in range(lay.n_in):
            blk = W[i * F:(i + 1) * F, o * F:(o + 1) * F]
            for g in range(G):
                for b in range(B):
                    k = g * B + b
                    d = np.repeat(blk[(f + k) % F, f], T)          # slot f T + t
                    out[o, i, g, b] = np.roll(d, g * B * lay.unit)  # rot_{-g B u}
    return out.reshape(lay.n_diagonals, lay.slots)


def split(n: int, world: int) -> List[Tuple[int, int]]:
    """[0, n) in `world` contiguous ranges of sizes differing by at most one
    (some empty when world > n)."""
    if n < 0 or world < 1:
        raise ValueError("bad split")
    base, extra = divmod(n, world)
    out, lo = [], 0
    for r in range(world):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def giant_ranges(n_giant: int, world: int) -> List[Tuple[int, int]]:
    """Giant steps of each rank (contiguous, balanced)."""
    return split(n_giant, world)


def baby_chunk(lay: MatmulLayout, world: int) -> int:
    """Baby-step rotations per rank in the all-gather: ceil(n_in (B-1) / world)."""
    total = lay.n_in * (lay.n_baby - 1)
    return (total + world - 1) // world


def baby_assignment(lay: MatmulLayout, world: int, rank: int) -> List[Tuple[int, int]]:
    """The (input i, baby step b >= 1) pairs rank `rank` rotates: global
    rotation index r = i (B - 1) + b - 1 in [rank c, rank c + c), c = baby_chunk."""
    c = baby_chunk(lay, world)
    total = lay.n_in * (lay.n_baby - 1)
    return [(r // (lay.n_baby - 1), r % (lay.n_baby - 1) + 1)
            for r in range(rank * c, min(total, (rank + 1) * c))]


def check_sum_fits(q_max: int, world: int) -> None:
    """The partial products are summed as int64 words: world residues below
    q_max must stay below 2^63."""
    if world * (int(q_max) - 1) >= 1 << 63:
        raise ValueError("sum of %d residues mod a %d-bit prime overflows int64"
                         % (world, int(q_max).bit_length()))


def matmul_giant_parallel(ctx, xs: Sequence, level_limbs: int, lay: MatmulLayout, pts: Sequence,
                          ys, group=None, stream=None) -> None:
    """Y = X W over the ranks of `group`: every rank passes the whole input
    ciphertexts xs [n_in] ([2][Ql][N] torch tensors), its one-GPU context
    (keys for the baby steps it rotates and the giant steps of its range),
    the diagonals pts of its giant-step range (others may be any tensor of
    the right shape, they are not read), and ys, a [n_out][2][Ql][N] tensor,
    which every rank receives whole.  The baby-step rotations are split over
    the ranks and all-gathered, the giant steps are split by
    ``giant_ranges``, and the partial products are all-reduced (int64 sum)
    and reduced mod q."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group) if group is not None or dist.is_initialized() else 1
    rank = dist.get_rank(group) if world > 1 else 0
    if ctx.world != 1:
        raise ValueError("matmul_giant_parallel needs a one-GPU context on every rank")
    check_sum_fits(int(max(ctx.q[:level_limbs])), world)
    B = lay.n_baby
    x0 = xs[0]
    total = lay.n_in * (B - 1)
    baby = None
    if total > 0:
        c = baby_chunk(lay, world)
        buf = torch.empty((world * c,) + tuple(x0.shape), dtype=x0.dtype, device=x0.device)
        mine = baby_assignment(lay, world, rank)
        for i in sorted({i for i, _ in mine}):
            bs = [b for ii, b in mine if ii == i]
            outs = [buf[i * (B - 1) + b - 1] for b in bs]
            ctx.rotate_hoisted(xs[i], level_limbs, [b * lay.unit for b in bs], outs, stream=stream)
        if world > 1:
            if stream is not None:
                torch.cuda.current_stream(x0.device).wait_stream(stream)
            gathered = torch.empty_like(buf)
            dist.all_gather_into_tensor(gathered, buf[rank * c:(rank + 1) * c], group=group)
            buf = gathered
        baby = [buf[r] for r in range(total)]
    g_lo, g_hi = giant_ranges(lay.n_giant, world)[rank]
    work = torch.empty(max(ctx.bsgs_workspace_words(level_limbs, lay.n_in, 1), 2),
                       dtype=torch.int64, device=x0.device)
    if g_hi > g_lo:
        ctx.bsgs_matmul(list(xs), level_limbs, lay.unit, B, lay.n_giant, pts,
                        [ys[o] for o in range(lay.n_out)], work, g_range=(g_lo, g_hi),
                        baby=baby, stream=stream)
    else:
        ys.zero_()
    if world > 1:
        if stream is not None:
            torch.cuda.current_stream(x0.device).wait_stream(stream)
        dist.all_reduce(ys, op=dist.ReduceOp.SUM, group=group)
        ctx.reduce_limbs(ys, 2 * lay.n_out, level_limbs)
        if stream is not None:
            stream.wait_stream(torch.cuda.current_stream(x0.device))


__all__ = ["MatmulLayout", "layout", "pack", "unpack", "diagonals", "split", "giant_ranges",
           "baby_chunk", "baby_assignment", "check_sum_fits", "matmul_giant_parallel"]
