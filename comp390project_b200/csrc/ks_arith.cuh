// ks_arith.cuh -- 64-bit modular arithmetic on the integer pipes of sm_100a.
//
// Shoup multiplication (V. Shoup, NTL; D. Harvey, "Faster arithmetic for
// number-theoretic transforms", 2014) for products by a known constant, and
// Barrett reduction (P. Barrett, 1986) of 128-bit accumulators with the
// two-word ratio floor(2^128/q).  Every routine is derived from those
// published methods; lazy ranges are stated per function.
#pragma once
#include <cstdint>

namespace ksb {

typedef uint64_t u64;

struct __align__(16) PrimeDev {
  u64 q, two_q;
  u64 br_hi, br_lo;      // floor(2^128 / q)
  u64 ninv, ninv_sh;     // N^-1 and its Shoup companion
  u64 w1ninv, w1ninv_sh; // psi^-brev(1) * N^-1 (last inverse stage, N^-1 folded in)
  u64 mu, pad_;          // floor(2^64 / q)
};

// Forward butterflies skip every conditional subtraction when q < 2^58:
// each Cooley-Tukey stage grows the bound by 2q, so 16 stages from inputs
// < q end below 33q < 2^64.  Inverse butterflies skip them when q < 2^46:
// each Gentleman-Sande stage at most doubles the bound, 2^16 * q < 2^62.
constexpr u64 kFwdLazyBound = 1ull << 58;
constexpr u64 kInvLazyBound = 1ull << 46;

constexpr int KS_MAX_PRIMES = 96;

// x * w mod q for a constant w with wp = floor(w 2^64 / q): result in [0, 2q)
// for any x < 2^64 and q < 2^63.
__device__ __forceinline__ u64 mul_shoup_lazy(u64 x, u64 w, u64 wp, u64 q) {
  u64 hi = __umul64hi(x, wp);
  return x * w - hi * q;
}
__device__ __forceinline__ u64 csub(u64 x, u64 m) { return x >= m ? x - m : x; }
__device__ __forceinline__ u64 mul_shoup(u64 x, u64 w, u64 wp, u64 q) {
  return csub(mul_shoup_lazy(x, w, wp, q), q);
}
__device__ __forceinline__ u64 add_mod(u64 a, u64 b, u64 q) { return csub(a + b, q); }
__device__ __forceinline__ u64 sub_mod(u64 a, u64 b, u64 q) { return a >= b ? a - b : a + q - b; }

// 128-bit accumulator.
struct u128v {
  u64 lo, hi;
};
__device__ __forceinline__ void mac(u128v &acc, u64 a, u64 b) {
  u64 lo = a * b, hi = __umul64hi(a, b);
  acc.lo += lo;
  acc.hi += hi + (acc.lo < lo ? 1ull : 0ull);
}

// Barrett: x mod q for x < 2^128 with (rh, rl) = floor(2^128 / q), q < 2^62.
// qhat = floor(x * ratio / 2^128) satisfies floor(x/q) - 2 < qhat <= floor(x/q),
// so r = x - qhat q lies in [0, 2q) and one conditional subtraction finishes.
__device__ __forceinline__ u64 barrett128(u128v x, u64 q, u64 rh, u64 rl) {
  u64 c0 = __umul64hi(x.lo, rl);
  u64 b_lo = x.lo * rh, b_hi = __umul64hi(x.lo, rh);
  u64 c_lo = x.hi * rl, c_hi = __umul64hi(x.hi, rl);
  u64 s = c0 + b_lo;
  u64 carry = s < c0 ? 1ull : 0ull;
  u64 s2 = s + c_lo;
  carry += s2 < s ? 1ull : 0ull;
  u64 qhat = x.hi * rh + b_hi + c_hi + carry;
  u64 r = x.lo - qhat * q;
  return csub(r, q);
}

// Harvey's forward (Cooley-Tukey) butterfly: X, Y in [0, 4q) -> [0, 4q).
__device__ __forceinline__ void ct_bfly(u64 &X, u64 &Y, u64 w, u64 wp, u64 q, u64 two_q) {
  u64 x = csub(X, two_q);
  u64 t = mul_shoup_lazy(Y, w, wp, q);
  X = x + t;
  Y = x - t + two_q;
}

// Harvey's inverse (Gentleman-Sande) butterfly: X, Y in [0, 2q) -> [0, 2q).
__device__ __forceinline__ void gs_bfly(u64 &X, u64 &Y, u64 w, u64 wp, u64 q, u64 two_q) {
  u64 s = csub(X + Y, two_q);
  u64 d = X - Y + two_q;
  X = s;
  Y = mul_shoup_lazy(d, w, wp, q);
}

// Last inverse stage with N^-1 folded in; outputs in [0, 2q).
__device__ __forceinline__ void gs_bfly_last(u64 &X, u64 &Y, const PrimeDev &P) {
  u64 s = X + Y;  // < 4q
  u64 d = X - Y + P.two_q;
  X = mul_shoup_lazy(s, P.ninv, P.ninv_sh, P.q);
  Y = mul_shoup_lazy(d, P.w1ninv, P.w1ninv_sh, P.q);
}

// [0, 4q) -> [0, q)
__device__ __forceinline__ u64 reduce4(u64 x, u64 q, u64 two_q) { return csub(csub(x, two_q), q); }

// Any x < 2^64 -> [0, q): qhat = floor(x * mu / 2^64) >= floor(x/q) - 1.
__device__ __forceinline__ u64 reduce_full(u64 x, u64 q, u64 mu) {
  return csub(x - __umul64hi(x, mu) * q, q);
}

// Forward butterfly without reductions (q < kFwdLazyBound): bound grows by 2q.
__device__ __forceinline__ void ct_bfly_lazy(u64 &X, u64 &Y, u64 w, u64 wp, u64 q, u64 two_q) {
  const u64 t = mul_shoup_lazy(Y, w, wp, q);
  const u64 x = X;
  X = x + t;
  Y = x - t + two_q;
}

// Inverse butterfly without reductions (q < kInvLazyBound).  K is a multiple
// of q no smaller than the bound on Y, so X + K - Y never wraps.
__device__ __forceinline__ void gs_bfly_lazy(u64 &X, u64 &Y, u64 w, u64 wp, u64 q, u64 K) {
  const u64 s = X + Y;
  const u64 d = X + K - Y;
  X = s;
  Y = mul_shoup_lazy(d, w, wp, q);
}
__device__ __forceinline__ void gs_bfly_last_lazy(u64 &X, u64 &Y, const PrimeDev &P, u64 K) {
  const u64 s = X + Y;
  const u64 d = X + K - Y;
  X = mul_shoup_lazy(s, P.ninv, P.ninv_sh, P.q);
  Y = mul_shoup_lazy(d, P.w1ninv, P.w1ninv_sh, P.q);
}

}  // namespace ksb
