// ks_fused.cu -- fused key-switch kernels (sm_100a).
//
// ModUp base extension fused into the first NTT pass: the inputs of a column
// tile are produced from the alpha scaled coefficient limbs of their digit,
//   y = sum_i v_i * [Q_d/q_i]_{m_j}  mod m_j,
// one source limb at a time (16 independent coalesced loads per thread per
// source, Shoup products against the per-(digit, limb) constants accumulated
// in 64 bits), and fed straight into the butterflies, so the extended limbs
// in coefficient form never touch HBM.  The scaled inputs
// v_i = [x_i (Q_d/q_i)^-1]_{q_i} come out of the input INTT, whose last stage
// multiplies by N^-1 (Q_d/q_i)^-1 instead of N^-1.
//
// ModDown: the P -> Q conversion is fused the same way into the first pass,
// and the second pass ends with (cx - z) P^-1 mod q_j and the add to the
// ciphertext, staged through shared memory so every global access of the
// epilogue is coalesced.
#include "ks_fused.cuh"
#include "ks_galois.cuh"
#include "ks_launch.cuh"
#include "ks_tmem.cuh"
#include "ks_ntt_impl.cuh"

namespace ksb {
namespace {

using namespace ntt;

template <int LOG_M>
__global__ void __launch_bounds__(kThreads) k_inv_cols_scaled(LimbMap m, NttTables T,
                                                             const ulonglong2 *scale) {
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int li = blockIdx.y;
  u64 *a = m.base + (m.offsets ? m.offsets[li] : (long long)li * m.stride);
  const int prime = m.prime_tab ? m.prime_tab[li] : m.first_prime + (li % m.period);
  if (prime < 0) return;
  const PrimeDev P = T.primes[prime];
  const int log_n = T.log_n, N = 1 << log_n, M2 = N >> LOG_M;
  const ulonglong2 *tw = T.inv + (long long)prime * N;
  const int c = threadIdx.x % G::C, t = threadIdx.x / G::C;
  const int col = blockIdx.x * G::C + c;
  const ulonglong2 s0 = scale[2 * li], s1 = scale[2 * li + 1];
  auto load = [&](int r, int cl) { return a[(long long)r * M2 + cl]; };
  auto store = [&](int r, int cl, u64 v) { a[(long long)r * M2 + cl] = v; };
  if (P.q < kFpBound) {
    // scale entries of FP64 primes hold the bits of {s, fl(s/q)}; the output
    // (the ModUp source limbs) stays a double: canonical, as its bits
    inv_cols_fp<LOG_M, true>(sm, col, t, c, log_n, T.inv_col + ((long long)prime << LOG_M), P,
                       make_double2(as_fp(s0.x), as_fp(s0.y)),
                       make_double2(as_fp(s1.x), as_fp(s1.y)), load, store);
  } else if (P.q < kInvLazyBound) {
    inv_cols<LOG_M, true>(sm, col, t, c, log_n, tw, P, s0, s1, load, store);
  } else {
    inv_cols<LOG_M, false>(sm, col, t, c, log_n, tw, P, s0, s1, load, store);
  }
}

// Source limbs of the base conversions: scaled coefficient limbs from
// ntt_inverse_scaled, canonical, stored as the bits of a double for primes
// below kFpBound and as uint64 otherwise.
__device__ __forceinline__ u64 src_u64(u64 bits, bool fp_src) {
  return fp_src ? (u64)__double2ull_rn(as_fp(bits)) : bits;
}

// Fills the 16 column inputs of this thread with
//   y = sum_{i < n_src} [v_i * w_i]_{q}  (each term canonical, sum < 8q),
// reduced to [0, q).  src(i) points at source limb i, fp_src(i) tells its
// storage (src_u64).
template <int LOG_M, class Src, class SrcFp>
__device__ __forceinline__ void bconv_fill(u64 (&x)[kEpt], int t, int col, int M2, int n_src,
                                           Src &&src, SrcFp &&fp_src, const u64 *w,
                                           const u64 *wsh, const PrimeDev &P) {
  using G = ColGeom<LOG_M>;
  u64 acc[kEpt];
#pragma unroll
  for (int e = 0; e < kEpt; ++e) acc[e] = 0;
#pragma unroll 1
  for (int i = 0; i < n_src; ++i) {
    const u64 *s = src(i);
    const u64 wi = __ldg(&w[i]), wp = __ldg(&wsh[i]);
    const bool fs = fp_src(i);
    u64 v[kEpt];
#pragma unroll
    for (int e = 0; e < kEpt; ++e)
      v[e] = __ldg(s + (long long)lidx<LOG_M, G::HI, 4>(t, e) * M2 + col);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) acc[e] += mul_shoup(src_u64(v[e], fs), wi, wp, P.q);
  }
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = reduce_full(acc[e], P.q, P.mu);
}

// FP64 variant for targets q < kFpBound: x = sum_i fp_mulmod(v_i, w_i, w_i/q),
// |x| < 0.57 q n_src < 4.6q.  Sources below kFpBound are read as doubles as
// stored; a source limb whose prime is not below 2^50 (the 58-bit q_0) is
// first reduced mod q with the integer Barrett-style reduce_full so that
// every product input stays below 2^50.
template <int LOG_M, class Src, class SrcQ>
__device__ __forceinline__ void bconv_fill_fp(double (&x)[kEpt], int t, int col, int M2,
                                              int n_src, Src &&src, SrcQ &&src_q,
                                              const u64 *w, const double *wq,
                                              const PrimeDev &P) {
  using G = ColGeom<LOG_M>;
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = 0.0;
#pragma unroll 1
  for (int i = 0; i < n_src; ++i) {
    const u64 *s = src(i);
    const double wd = (double)__ldg(&w[i]), wqd = __ldg(&wq[i]);
    const u64 qs = src_q(i);
    u64 v[kEpt];
#pragma unroll
    for (int e = 0; e < kEpt; ++e)
      v[e] = __ldg(s + (long long)lidx<LOG_M, G::HI, 4>(t, e) * M2 + col);
    if (qs < kFpBound) {
#pragma unroll
      for (int e = 0; e < kEpt; ++e) x[e] = __dadd_rn(x[e], fp_mulmod(as_fp(v[e]), wd, wqd, P.qd));
    } else {
      if (qs >= (1ull << 50)) {
#pragma unroll
        for (int e = 0; e < kEpt; ++e) v[e] = reduce_full(v[e], P.q, P.mu);
      }
#pragma unroll
      for (int e = 0; e < kEpt; ++e)
        x[e] = __dadd_rn(x[e], fp_mulmod(u64_to_fp(v[e]), wd, wqd, P.qd));
    }
  }
}

// ---------------------------------------------------------------------------
// ModUp: base conversion + forward column pass
// ---------------------------------------------------------------------------
// The arithmetic path is chosen per CTA from the target prime (FP64 below
// kFpBound, integer above); jobs are ordered FP64 first.
template <int LOG_M>
__global__ void __launch_bounds__(kThreads, 3)
    k_modup_cols(const u64 *__restrict__ v_all, const int *__restrict__ src_slot, u64 *t,
                 ModUpDev mu, KsLayout lay, const int *__restrict__ job_d,
                 const int *__restrict__ job_s, int job0, NttTables T) {
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int d = job_d[job0 + blockIdx.y], s = job_s[job0 + blockIdx.y];
  const int j = lay.out_j[s];
  const int prime = mu.prime_of[j];
  const PrimeDev P = T.primes[prime];
  const int log_n = T.log_n, N = 1 << log_n, M2 = N >> LOG_M;
  const int c = threadIdx.x % G::C, tt = threadIdx.x / G::C;
  const int col = blockIdx.x * G::C + c;
  const int n_src = min(mu.alpha, mu.Ql - d * mu.alpha);
  const long long wo = ((long long)d * mu.QlP + j) * mu.alpha;
  auto src = [&](int i) { return v_all + (long long)src_slot[d * mu.alpha + i] * N; };
  u64 *out = t + ((long long)d * lay.n_out + s) * N;
  auto store = [&](int r, int cl, u64 v) { out[(long long)r * M2 + cl] = v; };
  if (P.q < kFpBound) {
    const int *src_prime = mu.prime_of + d * mu.alpha;  // Q limb d*alpha+i has prime index d*alpha+i
    auto filld = [&](double (&x)[kEpt]) {
      bconv_fill_fp<LOG_M>(x, tt, col, M2, n_src, src,
                           [&](int i) { return T.primes[src_prime[i]].q; }, mu.w + wo,
                           mu.wq + wo, P);
    };
    fwd_cols_fpd<LOG_M>(sm, col, tt, c, log_n, T.fwd_col + ((long long)prime << LOG_M), P, filld,
                        store);
  } else {
    const int *src_prime = mu.prime_of + d * mu.alpha;
    auto fp_src = [&](int i) { return T.primes[src_prime[i]].q < kFpBound; };
    auto fill = [&](u64 (&x)[kEpt]) {
      bconv_fill<LOG_M>(x, tt, col, M2, n_src, src, fp_src, mu.w + wo, mu.wsh + wo, P);
    };
    const ulonglong2 *tw = T.fwd + (long long)prime * N;
    if (P.q < kFwdLazyBound) fwd_cols<LOG_M, true>(sm, col, tt, c, log_n, tw, P, fill, store);
    else fwd_cols<LOG_M, false>(sm, col, tt, c, log_n, tw, P, fill, store);
  }
}

// One digit's contribution to an accumulator: acc + y * k mod m_j.  FP:
// y and acc are the bits of doubles, every term |.| < 0.57 m_j, re-centred
// every 32 digits; integer: Barrett reduction of y * k + acc.
template <bool FP>
__device__ __forceinline__ u64 ip_term(u64 acc, u64 y, u64 k, bool first, bool recentre,
                                       const PrimeDev &P) {
  if (FP) {
    const double kd = u64_to_fp(k);
    double a = first ? 0.0 : as_fp(acc);
    a = __dadd_rn(a, fp_mulmod(as_fp(y), kd, __dmul_rn(kd, P.qinv), P.qd));
    if (recentre) a = fp_reduce_sym(a, P.qd, P.qinv);
    return fp_bits(a);
  }
  return mac_reduce(first ? 0ull : acc, y, k, P.q, P.br_hi, P.br_lo);
}

// ---------------------------------------------------------------------------
// ModUp row pass fused with the evaluation-key inner product
// ---------------------------------------------------------------------------
// One CTA: one kBipTile-word tile of one output limb s (prime m_j), all
// digits of the key shard; each warp owns the 512 words [512 w, 512 w + 512)
// of the tile (whole rows) and runs on its own, with no CTA-wide barrier
// after set-up.  Per digit a warp's inputs are three contiguous 4 KB blocks
// -- its slice of t[d][s] (column pass done; for the digit that holds q_j,
// the aligned source slice of the NTT-form input instead) and its slices of
// the two key polys -- which lane 0 moves into the warp's shared-memory
// stage with cp.async.bulk (the bulk-copy engine; completion counted in
// bytes on the warp's mbarrier), and whose next-digit blocks it prefetches
// into L2 with cp.async.bulk.prefetch, so the refill of the stage is an L2
// hit.  The slice gets its row pass (the second pass of the forward NTT) in
// registers with the exchange done in place in the stage, swizzled so that
// both access patterns are free of bank conflicts, and is multiplied into
// the two accumulators:
//   cx[0][s] = sum_d t[d][s] * key[d][0][j],   cx[1][s] = sum_d t[d][s] * key[d][1][j].
// The 32 accumulators of a thread (two polys x 16 words) live in Tensor
// Memory (tcgen05.ld / st), which keeps the kernel at 128 registers and four
// CTAs (16 warps) per SM.
struct RowsIpArgs {
  const u64 *t, *c_ntt, *key;
  u64 *cx;
  int key_limbs;
  uint32_t elt;  // c_ntt is read through X -> X^elt (1: as it is)
  int *status;   // device status word: kDevTimeout when a copy never completed
};

constexpr int kBipWarps = 4;
constexpr int kBipThreads = kBipWarps * 32;
constexpr int kBipTile = kBipWarps * 512;      // words of one CTA tile
constexpr int kBipSlice = 512;                 // words of one warp's slice
constexpr int kBipSliceBytes = kBipSlice * 8;  // one 4 KB block
constexpr int kBipWarpWords = 3 * kBipSlice;   // t, key poly 0, key poly 1
constexpr size_t kBipSmemBytes = (size_t)kBipWarps * kBipWarpWords * 8;  // 48 KB

// Physical position of row-local word i of a row in the exchange: i with its
// 16-word group index XORed into its low four bits.  Thread t's 16 words
// {16e + t} (first round) and {16t + e} (second round) then fall in 16
// different bank groups, and the warp's pair reads cover whole segments.
__device__ __forceinline__ int bip_swz(int i) { return i ^ ((i >> 4) & 15); }

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits for the phase of the given parity, at most limit_ns; false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > limit_ns) return false;
  return true;
}
// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// this GPU's global memory into this CTA's shared memory, counted on bar.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Bulk prefetch of `bytes` (multiple of 16, 16-byte aligned) of this GPU's
// global memory into L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Row pass of the warp's slice in its stage buffer sb (rows of M words,
// row-major as the bulk copy left them), thread (row rw of the slice, t);
// the result stays in sb at the swizzled positions (rw M + bip_swz(i)).
// FP: the bits of doubles, |x| < 12q; integer: canonical.
template <int LOG_M, bool FP, bool LAZY>
__device__ __forceinline__ void bip_row_pass(u64 *sb, int t, int rw, long long row,
                                             const NttTables &T, int prime, const PrimeDev &P) {
  using G = RowGeom<LOG_M>;
  u64 *rb = sb + (rw << LOG_M);
  const int log_n = T.log_n, N = 1 << log_n;
  if (FP) {
    const TwRowsGlobal<LOG_M> tw{T.fwd_fp + (long long)prime * N, log_n, P.qinv};
    double x[kEpt];
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = as_fp(rb[lidx<LOG_M, G::HI, 4>(t, e)]);
    fwd_round_fp<LOG_M, G::HI, 4>(x, t, row, tw, P.qd, P.qinv);
    __syncwarp();
#pragma unroll
    for (int e = 0; e < kEpt; ++e) rb[bip_swz(lidx<LOG_M, G::HI, 4>(t, e))] = fp_bits(x[e]);
    __syncwarp();
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = as_fp(rb[bip_swz(lidx<LOG_M, 0, G::NLO>(t, e))]);
    fwd_round_fp<LOG_M, 0, G::NLO>(x, t, row, tw, P.qd, P.qinv);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) rb[bip_swz(lidx<LOG_M, 0, G::NLO>(t, e))] = fp_bits(x[e]);
  } else {
    const ulonglong2 *tw = T.fwd + (long long)prime * N;
    u64 x[kEpt];
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = rb[lidx<LOG_M, G::HI, 4>(t, e)];
    fwd_round<LOG_M, G::HI, 4, LAZY>(x, t, row, 0, log_n, tw, P.q, P.two_q);
    __syncwarp();
#pragma unroll
    for (int e = 0; e < kEpt; ++e) rb[bip_swz(lidx<LOG_M, G::HI, 4>(t, e))] = x[e];
    __syncwarp();
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = rb[bip_swz(lidx<LOG_M, 0, G::NLO>(t, e))];
    fwd_round<LOG_M, 0, G::NLO, LAZY>(x, t, row, 0, log_n, tw, P.q, P.two_q);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) {
      const u64 v = LAZY ? reduce_full(x[e], P.q, P.mu) : reduce4(x[e], P.q, P.two_q);
      rb[bip_swz(lidx<LOG_M, 0, G::NLO>(t, e))] = v;
    }
  }
  __syncwarp();
}

// FP: prime below kFpBound (FP64 butterflies); else LAZY selects the
// integer butterflies without reductions.  Returns false when a copy did not
// complete within the bound (the caller records it).
template <int LOG_M, bool FP, bool LAZY>
__device__ __forceinline__ bool rows_ip_body(const RowsIpArgs &A, const ModUpDev &mu,
                                             const KsLayout &lay, const NttTables &T, int s,
                                             int prime, u64 *sb, uint64_t *bar, uint32_t tacc) {
  using G = RowGeom<LOG_M>;
  constexpr int M = 1 << LOG_M;
  const PrimeDev P = T.primes[prime];
  const int log_n = T.log_n, N = 1 << log_n;
  const int j = lay.out_j[s];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tt = lane % G::TT, rw = lane / G::TT;  // thread of a row, row of the slice
  const long long slice0 = (long long)blockIdx.x * kBipTile + warp * kBipSlice;
  const long long row = (slice0 >> LOG_M) + rw;
  const int dj = j < mu.Ql ? j / mu.alpha : -1;
  const long long kstride = (long long)A.key_limbs * N;
  const u64 *kbase = A.key + (long long)lay.key_slot[s] * N + slice0;
  const u64 *tbase = A.t + (long long)s * N + slice0;
  const long long tstride = (long long)lay.n_out * N;
  // own-digit limb, read through the automorphism: the slice gathers from
  // one aligned source slice of the same size
  const u64 *cown = dj >= 0 ? A.c_ntt + (long long)lay.c_slot[s] * N +
                                  (galois_src((uint32_t)slice0, A.elt, log_n) &
                                   ~(uint32_t)(kBipSlice - 1))
                            : nullptr;
  const int n_dig = lay.n_digits;
  auto src_t = [&](int di) {
    const int d = __ldg(&lay.digits[di]);
    return d == dj ? cown : tbase + d * tstride;
  };
  auto issue = [&](int di) {  // lane 0: digit di's three blocks -> the stage
    const u64 *kb = kbase + (long long)(2 * di) * kstride;
    mbar_expect_tx(bar, 3 * kBipSliceBytes);
    bulk_g2s(sb, src_t(di), kBipSliceBytes, bar);
    bulk_g2s(sb + kBipSlice, kb, kBipSliceBytes, bar);
    bulk_g2s(sb + 2 * kBipSlice, kb + kstride, kBipSliceBytes, bar);
  };
  auto prefetch = [&](int di) {  // lane 0: digit di's three blocks -> L2
    const u64 *kb = kbase + (long long)(2 * di) * kstride;
    bulk_prefetch_l2(src_t(di), kBipSliceBytes);
    bulk_prefetch_l2(kb, kBipSliceBytes);
    bulk_prefetch_l2(kb + kstride, kBipSliceBytes);
  };
  if (lane == 0) {
    issue(0);
    if (n_dig > 1) prefetch(1);
  }
#pragma unroll 1
  for (int di = 0; di < n_dig; ++di) {
    const bool ok = mbar_wait_bounded(bar, di & 1, 1000000000ull);
    if (__any_sync(0xffffffffu, !ok)) {
      // a copy never completed: wait (bounded) for it before the CTA exits
      if (lane == 0) mbar_wait_bounded(bar, di & 1, 1000000000ull);
      __syncwarp();
      return false;
    }
    if (lane == 0 && di + 2 < n_dig) prefetch(di + 2);
    const int d = __ldg(&lay.digits[di]);
    const bool own = d == dj;
    if (!own) bip_row_pass<LOG_M, FP, LAZY>(sb, tt, rw, row, T, prime, P);
    const u64 *k0b = sb + kBipSlice, *k1b = sb + 2 * kBipSlice;
    const bool first = di == 0, recentre = (di & 31) == 31;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      u64 y[4], kb0[4], kb1[4];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int w = 2 * lane + 64 * (2 * h + q);  // even slice word
        u64 y0, y1;
        if (own) {
          const uint32_t src =
              galois_src((uint32_t)(slice0 + w), A.elt, log_n) & (uint32_t)(kBipSlice - 1);
          const ulonglong2 v = *reinterpret_cast<const ulonglong2 *>(sb + (src & ~1u));
          y0 = (src & 1u) ? v.y : v.x;
          y1 = (src & 1u) ? v.x : v.y;
          if (FP) {
            y0 = fp_bits(u64_to_fp(y0));
            y1 = fp_bits(u64_to_fp(y1));
          }
        } else {
          const int c = w & (M - 1), x = (c >> 4) & 15;
          const ulonglong2 v =
              *reinterpret_cast<const ulonglong2 *>(sb + (w - c) + ((c ^ x) & ~1));
          y0 = (x & 1) ? v.y : v.x;
          y1 = (x & 1) ? v.x : v.y;
        }
        const ulonglong2 b = *reinterpret_cast<const ulonglong2 *>(k0b + w);
        const ulonglong2 a = *reinterpret_cast<const ulonglong2 *>(k1b + w);
        y[2 * q] = y0;
        y[2 * q + 1] = y1;
        kb0[2 * q] = b.x;
        kb0[2 * q + 1] = b.y;
        kb1[2 * q] = a.x;
        kb1[2 * q + 1] = a.y;
      }
      uint32_t r0[8], r1[8];
      if (!first) {
        tmem::ld8(tacc + 8 * h, r0);
        tmem::ld8(tacc + 32 + 8 * h, r1);
        tmem::wait_ld(r0, r1);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const u64 v0 = ip_term<FP>(tmem::pack(r0[2 * u], r0[2 * u + 1]), y[u], kb0[u], first,
                                   recentre, P);
        const u64 v1 = ip_term<FP>(tmem::pack(r1[2 * u], r1[2 * u + 1]), y[u], kb1[u], first,
                                   recentre, P);
        r0[2 * u] = (uint32_t)v0;
        r0[2 * u + 1] = (uint32_t)(v0 >> 32);
        r1[2 * u] = (uint32_t)v1;
        r1[2 * u + 1] = (uint32_t)(v1 >> 32);
      }
      tmem::st8(tacc + 8 * h, r0);
      tmem::st8(tacc + 32 + 8 * h, r1);
    }
    tmem::wait_st();
    // the warp's generic accesses to the stage precede the next bulk copy
    // into it (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0 && di + 1 < n_dig) issue(di + 1);
  }
  u64 *o0 = A.cx + (long long)s * N + slice0 + 2 * lane;
  u64 *o1 = o0 + (long long)lay.n_out * N;
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    uint32_t r0[8], r1[8];
    tmem::ld8(tacc + 8 * h, r0);
    tmem::ld8(tacc + 32 + 8 * h, r1);
    tmem::wait_ld(r0, r1);
    u64 v0[4], v1[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v0[u] = tmem::pack(r0[2 * u], r0[2 * u + 1]);
      v1[u] = tmem::pack(r1[2 * u], r1[2 * u + 1]);
      if (FP) {
        v0[u] = fp_to_canon(as_fp(v0[u]), P.qd, P.qinv);
        v1[u] = fp_to_canon(as_fp(v1[u]), P.qd, P.qinv);
      }
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int i = 2 * h + q;
      *reinterpret_cast<ulonglong2 *>(o0 + 64 * i) = make_ulonglong2(v0[2 * q], v0[2 * q + 1]);
      *reinterpret_cast<ulonglong2 *>(o1 + 64 * i) = make_ulonglong2(v1[2 * q], v1[2 * q + 1]);
    }
  }
  return true;
}

// The integer bodies (q_0 and the special primes) stay out of line: inlined
// they would push the FP64 body, which most output limbs run, into spills.
template <int LOG_M, bool LAZY>
__device__ __noinline__ bool rows_ip_body_int(const RowsIpArgs &A, const ModUpDev &mu,
                                              const KsLayout &lay, const NttTables &T, int s,
                                              int prime, u64 *sb, uint64_t *bar, uint32_t tacc) {
  return rows_ip_body<LOG_M, false, LAZY>(A, mu, lay, T, s, prime, sb, bar, tacc);
}

template <int LOG_M>
__global__ void __launch_bounds__(kBipThreads, 4)
    k_modup_rows_ip(RowsIpArgs A, ModUpDev mu, KsLayout lay, NttTables T) {
  // TMEM: warp w uses lane quarter w (32x32b shape) and 64 columns (two polys
  // x 16 words x 2 columns per word).  Shared memory (48 KB per CTA) caps
  // residency at four CTAs per SM, 256 columns of the 512, so the
  // allocation never waits.
  constexpr uint32_t kCols = 64;
  static_assert(kBipWarps == 4, "one TMEM lane quarter per warp");
  static_assert(kBipSmemBytes > 232448 / (512 / kCols + 1),
                "TMEM columns could be oversubscribed");
  extern __shared__ __align__(128) u64 dsm[];
  __shared__ __align__(8) uint64_t bars[kBipWarps];
  __shared__ uint32_t tmem_slot;
  const int s = blockIdx.y;
  const int prime = mu.prime_of[lay.out_j[s]];
  const u64 q = T.primes[prime].q;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) tmem::alloc(&tmem_slot, kCols);
  if (lane == 0) {
    mbar_init(&bars[warp], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tmem::fence_before_sync();
  __syncthreads();
  tmem::fence_after_sync();
  const uint32_t tacc = tmem_slot + ((uint32_t)(32 * warp) << 16);
  u64 *sb = dsm + warp * kBipWarpWords;
  bool ok;
  if (q < kFpBound) ok = rows_ip_body<LOG_M, true, false>(A, mu, lay, T, s, prime, sb, &bars[warp], tacc);
  else if (q < kFwdLazyBound) ok = rows_ip_body_int<LOG_M, true>(A, mu, lay, T, s, prime, sb, &bars[warp], tacc);
  else ok = rows_ip_body_int<LOG_M, false>(A, mu, lay, T, s, prime, sb, &bars[warp], tacc);
  if (!ok && lane == 0) atomicExch(A.status, kDevTimeout);
  tmem::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tmem::fence_after_sync();
    tmem::dealloc(tmem_slot, kCols);
  }
}

// ---------------------------------------------------------------------------
// ModDown: base conversion P -> q_j + forward column pass
// ---------------------------------------------------------------------------
template <int LOG_M>
__global__ void __launch_bounds__(kThreads, 2)
    k_moddown_cols(const u64 *__restrict__ y_base, const long long *__restrict__ y_off, u64 *z,
                   int n_q, const int *__restrict__ q_index, ModDownDev md, NttTables T,
                   const int *__restrict__ job_ps, int job0) {
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int ps = job_ps[job0 + blockIdx.y];
  const int p = ps / n_q, s = ps % n_q;
  const int j = q_index[s];
  const PrimeDev P = T.primes[j];
  const int log_n = T.log_n, N = 1 << log_n, M2 = N >> LOG_M;
  const int c = threadIdx.x % G::C, tt = threadIdx.x / G::C;
  const int col = blockIdx.x * G::C + c;
  const long long wo = (long long)j * md.alpha;
  auto src = [&](int i) { return y_base + y_off[p * md.alpha + i]; };
  auto fp_src = [&](int i) { return T.primes[md.first_p + i].q < kFpBound; };
  auto fill = [&](u64 (&x)[kEpt]) {
    bconv_fill<LOG_M>(x, tt, col, M2, md.alpha, src, fp_src, md.w + wo, md.wsh + wo, P);
  };
  u64 *out = z + ((long long)p * n_q + s) * N;
  auto store = [&](int r, int cl, u64 v) { out[(long long)r * M2 + cl] = v; };
  if (P.q < kFpBound) {
    // FP64 conversion (sources reduced mod q_j first when they do not fit):
    // spreads the work over the FP64 and integer pipes
    auto filld = [&](double (&x)[kEpt]) {
      bconv_fill_fp<LOG_M>(x, tt, col, M2, md.alpha, src,
                           [&](int i) { return T.primes[md.first_p + i].q; }, md.w + wo,
                           md.wq + wo, P);
    };
    fwd_cols_fpd<LOG_M>(sm, col, tt, c, log_n, T.fwd_col + ((long long)j << LOG_M), P, filld,
                        store);
  } else {
    const ulonglong2 *tw = T.fwd + (long long)j * N;
    if (P.q < kFwdLazyBound) fwd_cols<LOG_M, true>(sm, col, tt, c, log_n, tw, P, fill, store);
    else fwd_cols<LOG_M, false>(sm, col, tt, c, log_n, tw, P, fill, store);
  }
}

// Row pass of z with the ModDown finish fused into the epilogue.
template <int LOG_M>
__global__ void __launch_bounds__(kThreads)
    k_moddown_rows(const u64 *__restrict__ z, int n_q, const int *__restrict__ q_index,
                   const int *__restrict__ cx_slot, const u64 *__restrict__ cx,
                   long long cx_stride_poly, u64 *ct0, u64 *ct1, const u64 *g0, int rotate,
                   const u64 *__restrict__ diag, ModDownDev md, NttTables T) {
  using G = RowGeom<LOG_M>;
  extern __shared__ __align__(16) u64 dsm[];
  u64 *sm = dsm;
  double *smtw = reinterpret_cast<double *>(dsm + G::SMEM);
  const int p = blockIdx.y / n_q, s = blockIdx.y % n_q;
  const int j = q_index[s];
  const PrimeDev P = T.primes[j];
  const int log_n = T.log_n, N = 1 << log_n;
  const int t = threadIdx.x % G::TT, rr = threadIdx.x / G::TT;
  const long long tile0 = (long long)blockIdx.x * kTile;
  const u64 *tile = z + ((long long)p * n_q + s) * N + tile0;
  const long long row0 = (long long)blockIdx.x * G::R, row = row0 + rr;
  const u64 *cxp = cx + p * cx_stride_poly + (long long)cx_slot[s] * N + tile0;
  u64 *dst = (p == 0 ? ct0 : ct1) + (long long)s * N + tile0;
  // rotate with g0 == null: ct0 = o (no c0 term; the hoisted linear transform)
  const u64 *g0t = g0 ? g0 + (long long)s * N + tile0 : nullptr;
  const u64 *base = (p == 0) ? (rotate ? g0t : dst) : (rotate ? nullptr : dst);
  const bool fp = P.q < kFpBound;
  if (fp) stage_row_twiddles<LOG_M, G::R>(smtw, T.fwd_fp + (long long)j * N, log_n, row0);
  // Pull the epilogue operands into L2 while the butterflies run: one
  // prefetch per 128-byte line of the tile (4096 words = 256 lines).
  {
    const int line = threadIdx.x * 16;  // words; kThreads * 16 == kTile
    asm volatile("prefetch.global.L2 [%0];" ::"l"(cxp + line));
    if (base) asm volatile("prefetch.global.L2 [%0];" ::"l"(base + line));
  }
  u64 x[kEpt];
  if (fp) {
    cp_async_wait_all();
    __syncthreads();
    fwd_rows_regs_fp<LOG_M>(x, sm, smtw, tile, t, rr, row, row0, P);
  } else {
    const ulonglong2 *tw = T.fwd + (long long)j * N;
    if (P.q < kFwdLazyBound) fwd_rows_regs<LOG_M, true>(x, sm, tile, t, rr, row, log_n, tw, P);
    else fwd_rows_regs<LOG_M, false>(x, sm, tile, t, rr, row, log_n, tw, P);
  }
#pragma unroll
  for (int e = 0; e < kEpt; ++e) sm[padx<LOG_M>(rr, lidx<LOG_M, 0, G::NLO>(t, e))] = x[e];
  __syncthreads();
  const ulonglong2 pinv = md.pinv[j];
  const u64 *dg = diag ? diag + (long long)s * N + tile0 : nullptr;
#pragma unroll 4
  for (int i = 0; i < kEpt; ++i) {
    const int lin = threadIdx.x + i * kThreads;
    const u64 zv = sm[padx<LOG_M>(lin >> LOG_M, lin & (G::M - 1))];
    const u64 o = mul_shoup(cxp[lin] + P.q - zv, pinv.x, pinv.y, P.q);
    const u64 v = base ? add_mod(base[lin], o, P.q) : o;
    dst[lin] = dg ? mac_reduce(dst[lin], v, dg[lin], P.q, P.br_hi, P.br_lo) : v;
  }
}

// ---------------------------------------------------------------------------
// Rescale: the last limb (coefficient form, both polys) to the Q limbs + the
// forward column pass; the row pass is k_moddown_rows with q_last^-1
// ---------------------------------------------------------------------------
// Job (p, s), j = q_index[s]: y = ([c_p + h]_{q_last} mod q_j) - [h]_{q_j},
// h = floor(q_last / 2), c_p the last limb of poly p (last[p * N + k];
// stored as the bits of a double when q_last < kFpBound).
template <int LOG_M>
__global__ void __launch_bounds__(kThreads, 3)
    k_rescale_cols(const u64 *__restrict__ last, u64 q_last, int last_fp, u64 *z, int n_q,
                   const int *__restrict__ q_index, NttTables T) {
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int p = blockIdx.y / n_q, s = blockIdx.y % n_q;
  const int j = q_index[s];
  const PrimeDev P = T.primes[j];
  const int log_n = T.log_n, N = 1 << log_n, M2 = N >> LOG_M;
  const int c = threadIdx.x % G::C, tt = threadIdx.x / G::C;
  const int col = blockIdx.x * G::C + c;
  const u64 h = q_last >> 1, hj = reduce_full(h, P.q, P.mu);
  const u64 *src = last + (long long)p * N;
  auto fill = [&](u64 (&x)[kEpt]) {
#pragma unroll
    for (int e = 0; e < kEpt; ++e) {
      const u64 v = src_u64(__ldg(src + (long long)lidx<LOG_M, G::HI, 4>(tt, e) * M2 + col),
                            last_fp != 0);
      x[e] = sub_mod(reduce_full(csub(v + h, q_last), P.q, P.mu), hj, P.q);
    }
  };
  u64 *out = z + ((long long)p * n_q + s) * N;
  auto store = [&](int r, int cl, u64 v) { out[(long long)r * M2 + cl] = v; };
  if (P.q < kFpBound) {
    fwd_cols_fp<LOG_M>(sm, col, tt, c, log_n, T.fwd_col + ((long long)j << LOG_M), P, fill, store);
  } else {
    const ulonglong2 *tw = T.fwd + (long long)j * N;
    if (P.q < kFwdLazyBound) fwd_cols<LOG_M, true>(sm, col, tt, c, log_n, tw, P, fill, store);
    else fwd_cols<LOG_M, false>(sm, col, tt, c, log_n, tw, P, fill, store);
  }
}

template <int LOG_M>
cudaError_t launch_moddown_rows(dim3 grid, cudaStream_t s, const u64 *z, int n_q,
                               const int *q_index, const int *cx_slot, const u64 *cx,
                               long long cx_stride_poly, u64 *ct0, u64 *ct1, const u64 *g0,
                               int rot, const u64 *diag, const ModDownDev &md,
                               const NttTables &T) {
  constexpr size_t smem = row_smem_bytes<LOG_M>();
  static std::atomic<unsigned> attr_done{0};
  cudaError_t e = ensure_dynamic_smem(k_moddown_rows<LOG_M>, smem, attr_done);
  if (e != cudaSuccess) return e;
  k_moddown_rows<LOG_M><<<grid, kThreads, smem, s>>>(z, n_q, q_index, cx_slot, cx, cx_stride_poly,
                                                     ct0, ct1, g0, rot, diag, md, T);
  return cudaGetLastError();
}

template <int LOG_M>
cudaError_t launch_modup_rows_ip(cudaStream_t s, const u64 *t, const u64 *c_ntt, const u64 *key,
                                 int key_limbs, u64 *cx, const ModUpDev &mu, const KsLayout &lay,
                                 const NttTables &T, uint32_t elt, int *status) {
  static std::atomic<unsigned> attr_done{0};
  cudaError_t e = ensure_dynamic_smem(k_modup_rows_ip<LOG_M>, kBipSmemBytes, attr_done);
  if (e != cudaSuccess) return e;
  const dim3 grid((1 << T.log_n) / kBipTile, lay.n_out);
  const RowsIpArgs A{t, c_ntt, key, cx, key_limbs, elt, status};
  k_modup_rows_ip<LOG_M><<<grid, kBipThreads, kBipSmemBytes, s>>>(A, mu, lay, T);
  return cudaGetLastError();
}

inline int col_tiles(int log_n, int log_m) {
  const int M2 = (1 << log_n) >> log_m;
  return M2 / (kThreads / ((1 << log_m) / 16));
}

}  // namespace

cudaError_t ntt_inverse_scaled(const LimbMap &src, const LimbMap &dst, int n_limbs,
                               const ulonglong2 *scale, const NttTables &T, cudaStream_t s,
                               uint32_t elt) {
  if (!ntt_supported_log_n(T.log_n) || n_limbs < 0 || n_limbs > 65535) return cudaErrorInvalidValue;
  if (n_limbs == 0) return cudaSuccess;
  // first pass: the ordinary inverse row pass, src (through elt) -> dst
  cudaError_t e = ntt_inverse_rows_only(src, n_limbs, T, s, &dst, elt);
  if (e != cudaSuccess) return e;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), n_limbs);
  switch (s1) {
    case 6: k_inv_cols_scaled<6><<<grid, kThreads, 0, s>>>(dst, T, scale); break;
    case 7: k_inv_cols_scaled<7><<<grid, kThreads, 0, s>>>(dst, T, scale); break;
    case 8: k_inv_cols_scaled<8><<<grid, kThreads, 0, s>>>(dst, T, scale); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t modup_fused_cols(const u64 *v_all, const int *src_slot, u64 *t, const ModUpDev &mu,
                             const KsLayout &lay, const int *job_d, const int *job_s, int n_jobs,
                             int n_fp, const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_jobs < 0 || n_jobs > 65535) return cudaErrorInvalidValue;
  if (mu.alpha > KS_MAX_ALPHA || n_fp < 0 || n_fp > n_jobs) return cudaErrorInvalidValue;
  if (n_jobs == 0) return cudaSuccess;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), n_jobs);
  switch (s1) {
    case 6: k_modup_cols<6><<<grid, kThreads, 0, s>>>(v_all, src_slot, t, mu, lay, job_d, job_s, 0, T); break;
    case 7: k_modup_cols<7><<<grid, kThreads, 0, s>>>(v_all, src_slot, t, mu, lay, job_d, job_s, 0, T); break;
    case 8: k_modup_cols<8><<<grid, kThreads, 0, s>>>(v_all, src_slot, t, mu, lay, job_d, job_s, 0, T); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t modup_rows_inner_product(const u64 *t, const u64 *c_ntt, const u64 *key,
                                     int key_limbs, u64 *cx, const ModUpDev &mu,
                                     const KsLayout &lay, const NttTables &T, cudaStream_t s,
                                     uint32_t elt, int *status) {
  if (!(elt & 1u) || elt >= (2u << T.log_n)) return cudaErrorInvalidValue;
  if (!ntt_supported_log_n(T.log_n) || lay.n_out < 0 || lay.n_out > 65535)
    return cudaErrorInvalidValue;
  if (lay.n_out == 0) return cudaSuccess;
  const int s2 = T.log_n - T.log_n / 2;
  switch (s2) {
    case 6: return launch_modup_rows_ip<6>(s, t, c_ntt, key, key_limbs, cx, mu, lay, T, elt, status);
    case 7: return launch_modup_rows_ip<7>(s, t, c_ntt, key, key_limbs, cx, mu, lay, T, elt, status);
    case 8: return launch_modup_rows_ip<8>(s, t, c_ntt, key, key_limbs, cx, mu, lay, T, elt, status);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t moddown_fused_cols(const u64 *y_base, const long long *y_off, u64 *z, int n_q,
                               const int *q_index, const ModDownDev &md, const int *job_ps,
                               int n_fp, const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_q < 0 || 2 * n_q > 65535) return cudaErrorInvalidValue;
  if (md.alpha > KS_MAX_ALPHA || n_fp < 0 || n_fp > 2 * n_q) return cudaErrorInvalidValue;
  if (n_q == 0) return cudaSuccess;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), 2 * n_q);
  switch (s1) {
    case 6: k_moddown_cols<6><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T, job_ps, 0); break;
    case 7: k_moddown_cols<7><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T, job_ps, 0); break;
    case 8: k_moddown_cols<8><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T, job_ps, 0); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t rescale_fused_cols(const u64 *last, u64 q_last, bool last_fp, u64 *z, int n_q,
                               const int *q_index, const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_q < 0 || 2 * n_q > 65535) return cudaErrorInvalidValue;
  if (n_q == 0) return cudaSuccess;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), 2 * n_q);
  const int fp = last_fp ? 1 : 0;
  switch (s1) {
    case 6: k_rescale_cols<6><<<grid, kThreads, 0, s>>>(last, q_last, fp, z, n_q, q_index, T); break;
    case 7: k_rescale_cols<7><<<grid, kThreads, 0, s>>>(last, q_last, fp, z, n_q, q_index, T); break;
    case 8: k_rescale_cols<8><<<grid, kThreads, 0, s>>>(last, q_last, fp, z, n_q, q_index, T); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t moddown_fused_rows(const u64 *z, int n_q, const int *q_index, const int *cx_slot,
                               const u64 *cx, long long cx_stride_poly, u64 *ct0, u64 *ct1,
                               const u64 *g0, bool rotate, const u64 *diag,
                               const ModDownDev &md, const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_q < 0 || 2 * n_q > 65535) return cudaErrorInvalidValue;
  if (n_q == 0) return cudaSuccess;
  const int s2 = T.log_n - T.log_n / 2;
  dim3 grid((1 << T.log_n) / kTile, 2 * n_q);
  const int rot = rotate ? 1 : 0;
  switch (s2) {
    case 6: return launch_moddown_rows<6>(grid, s, z, n_q, q_index, cx_slot, cx, cx_stride_poly, ct0, ct1, g0, rot, diag, md, T);
    case 7: return launch_moddown_rows<7>(grid, s, z, n_q, q_index, cx_slot, cx, cx_stride_poly, ct0, ct1, g0, rot, diag, md, T);
    case 8: return launch_moddown_rows<8>(grid, s, z, n_q, q_index, cx_slot, cx, cx_stride_poly, ct0, ct1, g0, rot, diag, md, T);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ksb
