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
  // FP64 representation (primes below kFpBound): q, 1/q, and the last
  // inverse-stage scales as {s, s/q} pairs.
  double qd, qinv;
  double ninv_d, ninv_q, w1ninv_d, w1ninv_q;
};

// Primes below 2^43 run their NTT butterflies on the FP64 pipe: values are
// exact signed integers in doubles, products split exactly with an FMA
// (Dekker/Ogita two-product), the quotient estimate round(y*w/q) comes from
// the precomputed w/q, and every intermediate stays below 2^53.
constexpr u64 kFpBound = 1ull << 43;

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

// (acc + x * k) mod q for acc < q, x, k < 2^62 (x * k + acc < 2^125).
__device__ __forceinline__ u64 mac_reduce(u64 acc, u64 x, u64 k, u64 q, u64 rh, u64 rl) {
  u128v m;
  m.lo = x * k;
  m.hi = __umul64hi(x, k);
  m.lo += acc;
  m.hi += m.lo < acc ? 1ull : 0ull;
  return barrett128(m, q, rh, rl);
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
// ---------------------------------------------------------------------------
// FP64 modular arithmetic for q < kFpBound.  Operands are integers held in
// doubles, |y| <= 2^50.  fp_mulmod returns r = y*w - qt*q exactly with
// qt = rint(y * fl(w/q)):  h + l = y*w exactly (FMA two-product);
// |y*fl(w/q) - y*w/q| <= 2^50 * 2^-54, so |y*w/q - qt| < 0.57 and |r| < 0.57q;
// h - qt*q and the final sum are integers below 2^53, hence exact.
// ---------------------------------------------------------------------------
constexpr double kRound = 6755399441055744.0;  // 1.5 * 2^52: x + kRound - kRound = rint(x)
constexpr double kTwo52 = 4503599627370496.0;

__device__ __forceinline__ double fp_mulmod(double y, double w, double wq, double q) {
  const double h = __dmul_rn(y, w);
  const double l = __fma_rn(y, w, -h);
  const double qt = __dsub_rn(__fma_rn(y, wq, kRound), kRound);
  return __dadd_rn(__fma_rn(-qt, q, h), l);
}
// Cooley-Tukey: |X|,|Y| < B -> < B + 0.57q.
__device__ __forceinline__ void fp_ct_bfly(double &X, double &Y, double w, double wq, double q) {
  const double r = fp_mulmod(Y, w, wq, q);
  const double x = X;
  X = __dadd_rn(x, r);
  Y = __dsub_rn(x, r);
}
// Gentleman-Sande: |X|,|Y| < B -> |X| < 2B, |Y| < 0.57q.
__device__ __forceinline__ void fp_gs_bfly(double &X, double &Y, double w, double wq, double q) {
  const double s = __dadd_rn(X, Y);
  const double d = __dsub_rn(X, Y);
  X = s;
  Y = fp_mulmod(d, w, wq, q);
}
// (With |y| <= 2^50 the estimate error is below 2^-4, so |r| < 0.57q.)
// x - round(x/q) q, |result| <= 0.5q (+1), for |x| < 2^51.
__device__ __forceinline__ double fp_reduce_sym(double x, double q, double qinv) {
  const double t = __dsub_rn(__fma_rn(x, qinv, kRound), kRound);
  return __fma_rn(-t, q, x);
}
// Canonical [0, q) as a uint64, for |x| < 64q: floor(x/q) = rint(x/q - 1/2)
// because x/q - 1/2 is never within 1/(2q) of an integer.
__device__ __forceinline__ u64 fp_to_canon(double x, double q, double qinv) {
  const double u = __fma_rn(x, qinv, -0.5);
  const double t = __dsub_rn(__dadd_rn(u, kRound), kRound);
  const double r = __fma_rn(-t, q, x);
  return (u64)__double_as_longlong(__dadd_rn(r, kTwo52)) & 0xFFFFFFFFFFFFFull;
}
// Exact uint64 -> double for x < 2^52.
__device__ __forceinline__ double u64_to_fp(u64 x) {
  return __dsub_rn(__longlong_as_double((long long)(x | 0x4330000000000000ull)), kTwo52);
}

__device__ __forceinline__ void gs_bfly_last_lazy(u64 &X, u64 &Y, const PrimeDev &P, u64 K) {
  const u64 s = X + Y;
  const u64 d = X + K - Y;
  X = mul_shoup_lazy(s, P.ninv, P.ninv_sh, P.q);
  Y = mul_shoup_lazy(d, P.w1ninv, P.w1ninv_sh, P.q);
}

}  // namespace ksb
