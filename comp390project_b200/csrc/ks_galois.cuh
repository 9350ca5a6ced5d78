// ks_galois.cuh -- the automorphism X -> X^elt in the bit-reversed NTT order.
//
// Slot i of an NTT-form limb holds the evaluation at psi^(2 brev(i) + 1), so
// under X -> X^elt output slot i reads input slot
//   galois_src(i) = brev(((2 brev(i) + 1) elt mod 2N - 1) / 2).
// The low b bits of i are the top b bits of brev(i), which only reach the
// top b bits of the exponent product: an aligned block of 2^b output slots
// reads an aligned block of 2^b input slots (permuted inside), for every b.
// Kernels use this to gather whole tiles (b = 12) and warp segments (b = 5)
// coalesced; for the adjacent pair (2m, 2m + 1) the sources are
// galois_src(2m) and galois_src(2m) ^ 1.
#pragma once
#include <cstdint>

namespace ksb {

__device__ __forceinline__ uint32_t brev_n(uint32_t x, int log_n) {
  return __brev(x) >> (32 - log_n);
}

__device__ __forceinline__ uint32_t galois_src(uint32_t i, uint32_t elt, int log_n) {
  const uint32_t mask2n = (2u << log_n) - 1u;
  const uint32_t e = 2u * brev_n(i, log_n) + 1u;
  const uint32_t ge = (e * elt) & mask2n;
  return brev_n((ge - 1u) >> 1, log_n);
}

}  // namespace ksb
