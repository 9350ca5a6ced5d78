// ks_ntt.cuh -- batched negacyclic NTT / INTT over RNS limbs (sm_100a).
//
// Convention (the same as the CPU oracle): forward = Cooley-Tukey with the
// table psi^brev(i), natural order in, bit-reversed order out; inverse =
// Gentleman-Sande with psi^-brev(i), bit-reversed in, natural out, N^-1
// folded into the last stage.  Replaces Phantom's nwt_2d_radix8_forward /
// backward_inplace (paper/code_study.tex:493-506 of the reference).
#pragma once
#include <cuda_runtime.h>

#include "ks_arith.cuh"

namespace ksb {

// Where limb i of a batch lives and which prime it uses.  Launches over a
// group of key switches add a third grid dimension: member b of the group
// finds its limbs bstride words further on.
struct LimbMap {
  u64 *base;
  long long stride;          // words between consecutive limbs (normally N)
  const long long *offsets;  // device array; if set, limb i is at base + offsets[i]
  const int *prime_tab;      // device array; if null: first_prime + (i % period)
  int first_prime, period;
  long long bstride;         // words between the limbs of consecutive group members
};

// A group of independent key switches run through each launch together (the
// third grid dimension is the member).  Buffers the caller owns differ per
// member and are passed by value; scratch buffers sit at uniform strides.
constexpr int kMaxGroup = 8;
// Words of one thread's 16 column values in the 42-bit packed form (pack42):
// a packed limb of N words takes kPackWords * N / 16.
constexpr int kPackWords = 11;
struct MemberIn {             // per-member input limbs read through an automorphism
  const u64 *in[kMaxGroup];   // null in[0]: use the LimbMap's own base
  uint32_t elt[kMaxGroup];
};

// The FP64 tables hold w as a double at the same index as the integer
// tables, except inside the row-pass region: for row-pass local bit b < LM-4
// (LM = row length log2 = logN - logN/2) the 2^u twiddles of each row
// (u = LM-1-b) are stored at row_tw_pos(LM, b, k) instead of k.  In the
// second radix-16 round of a row pass thread t needs k = (t << s) | m
// (s = LM-5-b, m < 2^s); the position puts t in the low bits, so the lanes
// of a warp read consecutive words (no shared-memory bank conflicts, one
// 128-byte line per row from global memory).
__host__ __device__ constexpr int row_tw_pos(int lm, int b, int k) {
  return b >= lm - 4 ? k
                     : (k & ~((1 << (lm - 5 - b + lm - 4)) - 1)) |
                           ((k & ((1 << (lm - 5 - b + lm - 4)) - 1)) >> (lm - 5 - b)) |
                           ((k & ((1 << (lm - 5 - b)) - 1)) << (lm - 4));
}

struct NttTables {
  const ulonglong2 *fwd;  // [n_primes][N] {w, w_shoup}, w = psi^brev(i)
  const ulonglong2 *inv;  // [n_primes][N] {w, w_shoup}, w = psi^-brev(i)
  const PrimeDev *primes; // [n_primes]
  int log_n;
  const double *fwd_fp;   // [n_primes][N] w as a double (primes below kFpBound),
  const double *inv_fp;   // row-pass region permuted by row_tw_pos
  // [n_primes][2^(logN/2)] {w, fl(w/q)} of the column-pass indices (FP64 primes)
  const double2 *fwd_col, *inv_col;
};

// Transforms n_limbs limbs in place; outputs are canonical in [0, q).
// Inputs must be < q (canonical).  Limbs whose prime index is negative are
// skipped.  Supported ring degrees: 2^12 .. 2^16.
cudaError_t ntt_forward(const LimbMap &m, int n_limbs, const NttTables &T, cudaStream_t s);
cudaError_t ntt_inverse(const LimbMap &m, int n_limbs, const NttTables &T, cudaStream_t s);
bool ntt_supported_log_n(int log_n);
// Only the second pass of a forward transform (the first pass of an inverse
// one), for callers that run a fused first/second pass of their own.
cudaError_t ntt_forward_rows_only(const LimbMap &m, int n_limbs, const NttTables &T,
                                  cudaStream_t s);
// out: optional separate destination (same limb order and primes as m).
// elt != 1: the input is read through X -> X^elt (needs a separate out).
// mi (with group > 1 or a per-member input): member b reads its limbs at
// mi->in[b] + (the limb's offset from m.base) through mi->elt[b]; the output
// of member b is out->base + b * out->bstride.
cudaError_t ntt_inverse_rows_only(const LimbMap &m, int n_limbs, const NttTables &T,
                                  cudaStream_t s, const LimbMap *out = nullptr,
                                  uint32_t elt = 1, const MemberIn *mi = nullptr,
                                  int group = 1);

}  // namespace ksb
