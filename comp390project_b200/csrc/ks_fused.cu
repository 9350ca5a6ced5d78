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

template <int LOG_N>
__global__ void __launch_bounds__(kThreads, 4) k_inv_cols_scaled(LimbMap m, NttTables T,
                                                             const ulonglong2 *scale) {
  constexpr int LOG_M = LOG_N / 2;  // column pass of 2^LOG_M points, stride M2
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int li = blockIdx.y;
  u64 *a = m.base + (m.offsets ? m.offsets[li] : (long long)li * m.stride) +
           (long long)blockIdx.z * m.bstride;
  const int prime = m.prime_tab ? m.prime_tab[li] : m.first_prime + (li % m.period);
  if (prime < 0) return;
  const PrimeDev P = T.primes[prime];
  constexpr int log_n = LOG_N, N = 1 << LOG_N, M2 = N >> LOG_M;
  const ulonglong2 *tw = T.inv + (long long)prime * N;
  const int c = threadIdx.x % G::C, t = (threadIdx.x / G::C) & (G::TT - 1);  // known range t < TT
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

// k_inv_cols_scaled from src (the row-pass output) into dst, limbs
// li >= pack_from in the 42-bit packed form (pack42; their primes are below
// 2^42 and take the FP64 path), the others in k_inv_cols_scaled's form.
template <int LOG_N>
__global__ void __launch_bounds__(kThreads, 4)
    k_inv_cols_scaled_pack(LimbMap src, LimbMap dst, NttTables T, const ulonglong2 *scale,
                           int pack_from) {
  constexpr int LOG_M = LOG_N / 2;
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int li = blockIdx.y;
  const u64 *a = src.base + (src.offsets ? src.offsets[li] : (long long)li * src.stride) +
                 (long long)blockIdx.z * src.bstride;
  u64 *o = dst.base + (dst.offsets ? dst.offsets[li] : (long long)li * dst.stride) +
           (long long)blockIdx.z * dst.bstride;
  const int prime = src.prime_tab ? src.prime_tab[li] : src.first_prime + (li % src.period);
  if (prime < 0) return;
  const PrimeDev P = T.primes[prime];
  constexpr int log_n = LOG_N, N = 1 << LOG_N, M2 = N >> LOG_M;
  const ulonglong2 *tw = T.inv + (long long)prime * N;
  const int c = threadIdx.x % G::C, t = (threadIdx.x / G::C) & (G::TT - 1);  // known range t < TT
  const int col = blockIdx.x * G::C + c;
  const ulonglong2 s0 = scale[2 * li], s1 = scale[2 * li + 1];
  auto load = [&](int r, int cl) { return a[(long long)r * M2 + cl]; };
  auto store = [&](int r, int cl, u64 v) { o[(long long)r * M2 + cl] = v; };
  if (P.q < kFpBound) {
    const double2 d0 = make_double2(as_fp(s0.x), as_fp(s0.y));
    const double2 d1 = make_double2(as_fp(s1.x), as_fp(s1.y));
    const double2 *twc = T.inv_col + ((long long)prime << LOG_M);
    if (li >= pack_from) {
      u64 v[kEpt], w[kPackWords];
      inv_cols_fp_regs<LOG_M>(sm, col, t, c, log_n, twc, P, d0, d1, load, v);
      pack42(v, w);
#pragma unroll
      for (int k = 0; k < kPackWords; ++k) o[(long long)(t * kPackWords + k) * M2 + col] = w[k];
    } else {
      inv_cols_fp<LOG_M, true>(sm, col, t, c, log_n, twc, P, d0, d1, load, store);
    }
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
// The 16 values of this thread's column in source limb s: canonical uint64
// from the 42-bit packed form (packed) or as stored (the caller converts).
template <int LOG_M>
__device__ __forceinline__ void load_src_col(u64 (&v)[kEpt], const u64 *s, int t, int col,
                                             int M2, bool packed) {
  using G = ColGeom<LOG_M>;
  if (packed) {
    u64 w[kPackWords];
#pragma unroll
    for (int k = 0; k < kPackWords; ++k) w[k] = __ldg(s + (long long)(t * kPackWords + k) * M2 + col);
    unpack42(w, v);
  } else {
#pragma unroll
    for (int e = 0; e < kEpt; ++e)
      v[e] = __ldg(s + (long long)lidx<LOG_M, G::HI, 4>(t, e) * M2 + col);
  }
}

template <int LOG_M, class Src, class SrcFp, class SrcPk>
__device__ __forceinline__ void bconv_fill(u64 (&x)[kEpt], int t, int col, int M2, int n_src,
                                           Src &&src, SrcFp &&fp_src, SrcPk &&pk_src,
                                           const u64 *w, const u64 *wsh, const PrimeDev &P) {
  u64 acc[kEpt];
#pragma unroll
  for (int e = 0; e < kEpt; ++e) acc[e] = 0;
#pragma unroll 1
  for (int i = 0; i < n_src; ++i) {
    const u64 *s = src(i);
    const u64 wi = __ldg(&w[i]), wp = __ldg(&wsh[i]);
    const bool pk = pk_src(i);
    const bool fs = fp_src(i) && !pk;  // packed limbs hold canonical uint64
    u64 v[kEpt];
    load_src_col<LOG_M>(v, s, t, col, M2, pk);
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
template <int LOG_M, class Src, class SrcQ, class SrcPk>
__device__ __forceinline__ void bconv_fill_fp(double (&x)[kEpt], int t, int col, int M2,
                                              int n_src, Src &&src, SrcQ &&src_q, SrcPk &&pk_src,
                                              const u64 *w, const double *wq,
                                              const PrimeDev &P) {
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = 0.0;
#pragma unroll 1
  for (int i = 0; i < n_src; ++i) {
    const u64 *s = src(i);
    const double wd = (double)__ldg(&w[i]), wqd = __ldg(&wq[i]);
    const u64 qs = src_q(i);
    const bool pk = pk_src(i);
    u64 v[kEpt];
    load_src_col<LOG_M>(v, s, t, col, M2, pk);
    if (pk) {  // canonical uint64 below 2^42
#pragma unroll
      for (int e = 0; e < kEpt; ++e)
        x[e] = __dadd_rn(x[e], fp_mulmod(u64_to_fp(v[e]), wd, wqd, P.qd));
    } else if (qs < kFpBound) {
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
template <int LOG_N, bool PACKED>
__global__ void __launch_bounds__(kThreads, 3)
    k_modup_cols(const u64 *__restrict__ v_all, const long long *__restrict__ src_ref, u64 *t,
                 ModUpDev mu, KsLayout lay, const int *__restrict__ job_d,
                 const int *__restrict__ job_s, int job0, NttTables T, long long v_bstride,
                 long long t_bstride) {
  constexpr int LOG_M = LOG_N / 2;  // column pass of 2^LOG_M points, stride M2
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int d = job_d[job0 + blockIdx.y], s = job_s[job0 + blockIdx.y];
  const int j = lay.out_j[s];
  const int prime = mu.prime_of[j];
  const PrimeDev P = T.primes[prime];
  constexpr int log_n = LOG_N, N = 1 << LOG_N, M2 = N >> LOG_M;
  const int c = threadIdx.x % G::C, tt = (threadIdx.x / G::C) & (G::TT - 1);  // tt < TT (known range)
  const int col = blockIdx.x * G::C + c;
  const int n_src = min(mu.alpha, mu.Ql - d * mu.alpha);
  const long long wo = ((long long)d * mu.QlP + j) * mu.alpha;
  v_all += blockIdx.z * v_bstride;  // member of the group
  // source limb i of digit d: word offset src_ref >> 1 in the gathered input,
  // 42-bit packed when bit 0 is set
  auto src = [&](int i) { return v_all + (src_ref[d * mu.alpha + i] >> 1); };
  auto pk_src = [&](int i) { return PACKED && (src_ref[d * mu.alpha + i] & 1) != 0; };
  u64 *out = t + blockIdx.z * t_bstride + ((long long)d * lay.n_out + s) * N;
  auto store = [&](int r, int cl, u64 v) { out[(long long)r * M2 + cl] = v; };
  if (P.q < kFpBound) {
    const int *src_prime = mu.prime_of + d * mu.alpha;  // Q limb d*alpha+i has prime index d*alpha+i
    auto filld = [&](double (&x)[kEpt]) {
      bconv_fill_fp<LOG_M>(x, tt, col, M2, n_src, src,
                           [&](int i) { return T.primes[src_prime[i]].q; }, pk_src, mu.w + wo,
                           mu.wq + wo, P);
    };
    fwd_cols_fpd<LOG_M>(sm, col, tt, c, log_n, T.fwd_col + ((long long)prime << LOG_M), P, filld,
                        store);
  } else {
    const int *src_prime = mu.prime_of + d * mu.alpha;
    auto fp_src = [&](int i) { return T.primes[src_prime[i]].q < kFpBound; };
    auto fill = [&](u64 (&x)[kEpt]) {
      bconv_fill<LOG_M>(x, tt, col, M2, n_src, src, fp_src, pk_src, mu.w + wo, mu.wsh + wo, P);
    };
    const ulonglong2 *tw = T.fwd + (long long)prime * N;
    if (P.q < kFwdLazyBound) fwd_cols<LOG_M, true>(sm, col, tt, c, log_n, tw, P, fill, store);
    else fwd_cols<LOG_M, false>(sm, col, tt, c, log_n, tw, P, fill, store);
  }
}

// One FP64 inner-product term: acc + y k (mod q, unreduced), with acc
// brought back to (-q, q) every 32 digits.
__device__ __forceinline__ u64 ip_term_fp(u64 acc, u64 y, u64 k, bool first, bool recentre,
                                          const PrimeDev &P) {
  const double kd = u64_to_fp(k);
  double a = first ? 0.0 : as_fp(acc);
  a = __dadd_rn(a, fp_mulmod(as_fp(y), kd, __dmul_rn(kd, P.qinv), P.qd));
  if (recentre) a = fp_reduce_sym(a, P.qd, P.qinv);
  return fp_bits(a);
}

// One integer inner-product term on a 128-bit sum held as four 32-bit TMEM
// words r[c..c+4): sum += y k.
__device__ __forceinline__ void ip_acc128(uint32_t (&r)[8], int c, u64 y, u64 k, bool first) {
  u128v acc;
  acc.lo = first ? 0ull : tmem::pack(r[c], r[c + 1]);
  acc.hi = first ? 0ull : tmem::pack(r[c + 2], r[c + 3]);
  mac(acc, y, k);
  r[c] = (uint32_t)acc.lo;
  r[c + 1] = (uint32_t)(acc.lo >> 32);
  r[c + 2] = (uint32_t)acc.hi;
  r[c + 3] = (uint32_t)(acc.hi >> 32);
}
// sum := sum mod q in place (every 32 digits, so that 32 more products fit).
__device__ __forceinline__ void acc128_to_reduced(uint32_t (&r)[8], int c, const PrimeDev &P) {
  u128v acc;
  acc.lo = tmem::pack(r[c], r[c + 1]);
  acc.hi = tmem::pack(r[c + 2], r[c + 3]);
  const u64 v = barrett128(acc, P.q, P.br_hi, P.br_lo);
  r[c] = (uint32_t)v;
  r[c + 1] = (uint32_t)(v >> 32);
  r[c + 2] = 0;
  r[c + 3] = 0;
}
__device__ __forceinline__ u64 acc128_reduce(const uint32_t (&r)[8], int c, const PrimeDev &P) {
  u128v acc;
  acc.lo = tmem::pack(r[c], r[c + 1]);
  acc.hi = tmem::pack(r[c + 2], r[c + 3]);
  return barrett128(acc, P.q, P.br_hi, P.br_lo);
}

// ---------------------------------------------------------------------------
// ModUp row pass fused with the evaluation-key inner product
// ---------------------------------------------------------------------------
// One CTA: one 4096-word tile of one output limb s (prime m_j), all digits.
// For each digit d the tile of t[d][s] gets its row pass in registers (the
// digit that contains q_j instead reads the NTT-form input limb), goes
// through shared memory into a warp-coalesced order (warp w owns tile words
// [512w, 512w + 512), lane l the pairs 2l + 64i, i < 8), and is multiplied
// into the two accumulators against the key limbs of digit d:
//   cx[0][s] = sum_d t[d][s] * key[d][0][j],   cx[1][s] = sum_d t[d][s] * key[d][1][j].
// The key pairs of a lane are copied into shared memory with cp.async when
// the digit starts, so they arrive while the butterflies run; the next
// digit's value tile is prefetched into L2.  The 32 accumulators of a
// thread live in TMEM, not in registers: for FP64 primes 64 columns (poly 0
// in [0, 32), poly 1 in [32, 64), one u64 as two columns), for integer
// primes 128 (a 128-bit sum as four columns, reduced once at the end).  The
// extended limbs never return to HBM.
struct RowsIpArgs {
  const u64 *t;                  // member b: t + b t_bstride
  u64 *cx;                       // member b: cx + b cx_bstride
  long long t_bstride, cx_bstride;
  int key_limbs;
  const u64 *c_ntt[kMaxGroup];   // NTT-form input of member b ...
  uint32_t elt[kMaxGroup];       // ... read through X -> X^elt[b] (1: as it is)
  const u64 *key[kMaxGroup];     // key shard of member b
  u64 *fold;                     // member b: fold + b fold_bstride (lay.fold_off)
  long long fold_bstride;
};

// A CTA is kRipWarps warps; warp w owns the 512 tile words [512w, 512w + 512)
// (32 / TT rows of M words).  Smaller CTAs than the NTT kernels' 8 warps
// shorten the wave tail of this long-running kernel.
constexpr int kRipWarps = 4;
constexpr int kRipThreads = kRipWarps * 32;
constexpr int kRipTile = kRipWarps * 512;

template <int LOG_M>
__host__ __device__ constexpr int rows_ip_rows() {  // rows of M words per CTA
  return kRipTile >> LOG_M;
}
// The FP64 launch stages its CTA's row twiddles in shared memory (true) or
// reads them from the global table through L1 (false, 16 KB less shared
// memory per CTA: 4 CTAs per SM instead of 3).  Staged measured faster at
// config 3 (fused row-pass stage 132 against 139 µs per key switch); the
// integer launch needs no twiddle stage and runs 4 CTAs per SM either way.
constexpr bool kRipStageTw = true;
template <int LOG_M, bool FP_SLOTS>
__host__ __device__ constexpr size_t rows_ip_smem_bytes() {
  // padded exchange rows + per-warp key stage [warps][2 polys][8 pairs][32 lanes] x 16 B
  // + (FP64 launch, staged) the row-pass twiddles of the CTA's rows, the
  // same for every digit
  return (size_t)rows_ip_rows<LOG_M>() * ((1 << LOG_M) + (1 << LOG_M) / 16) * 8 +
         (size_t)kRipWarps * 2 * 8 * 32 * 16 +
         (FP_SLOTS && kRipStageTw ? (size_t)rows_ip_rows<LOG_M>() * ((1 << LOG_M) - 1) * 8 : 0);
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

// FP: prime below kFpBound (FP64 butterflies); else LAZY selects the
// integer butterflies without reductions.
template <int LOG_M, bool FP, bool LAZY>
__device__ __forceinline__ void rows_ip_body(const RowsIpArgs &A, const ModUpDev &mu,
                                             const KsLayout &lay, const NttTables &T, int s,
                                             int prime, u64 *sm, ulonglong2 *kst,
                                             const double *smtw, uint32_t tacc) {
  using G = RowGeom<LOG_M>;
  const PrimeDev P = T.primes[prime];
  const int mb = blockIdx.z;  // member of the group
  const u64 *const a_key = A.key[mb], *const a_t = A.t + mb * A.t_bstride;
  const u64 *const a_c = A.c_ntt[mb];
  u64 *const a_cx = A.cx + mb * A.cx_bstride;
  const uint32_t elt = A.elt[mb];
  const int log_n = T.log_n, N = 1 << log_n;
  const int j = lay.out_j[s];
  const int tt = threadIdx.x % G::TT, rr = threadIdx.x / G::TT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long tile0 = (long long)blockIdx.x * kRipTile;
  const long long row = (long long)blockIdx.x * rows_ip_rows<LOG_M>() + rr;
  const int wofs = warp * 512 + 2 * lane;  // + 64 i: this lane's pairs in the tile
  const int dj = j < mu.Ql ? j / mu.alpha : -1;
  const long long kstride = (long long)A.key_limbs * N;
  const u64 *kbase = a_key + (long long)lay.key_slot[s] * N + tile0 + wofs;
  const u64 *tbase = a_t + (long long)s * N + tile0;
  const long long tstride = (long long)lay.n_out * N;
  // own-digit limb, read through the automorphism: the CTA's tile gathers
  // from the aligned source tile cown, pair (k, k+1) from (src & ~1) (swapped
  // when src is odd)
  const u64 *climb = dj >= 0 ? a_c + (long long)lay.c_slot[s] * N : nullptr;
  const u64 *cown =
      climb ? climb + (galois_src((uint32_t)tile0, elt, log_n) & ~(uint32_t)(kRipTile - 1))
            : nullptr;
  const ulonglong2 *tw = T.fwd + (long long)prime * N;
  // FP64 primes: the CTA's row twiddles, staged once in shared memory or
  // read from the global table
  const auto twf = [&] {
    if constexpr (kRipStageTw)
      return TwRowsSmem<LOG_M, rows_ip_rows<LOG_M>()>{
          smtw, (long long)blockIdx.x * rows_ip_rows<LOG_M>(), P.qinv};
    else
      return TwRowsGlobal<LOG_M>{T.fwd_fp + (long long)prime * N, log_n, P.qinv};
  }();
  kst += warp * (2 * 8 * 32) + lane;  // [p][i] at kst[(p * 8 + i) * 32]
  // L2 prefetch of digit d's value tile: 128-byte lines (16 words), spread
  // over the CTA's threads.
  auto prefetch = [&](int d) {
    const u64 *v = d == dj ? cown : tbase + d * tstride;
#pragma unroll
    for (int line = threadIdx.x * 16; line < kRipTile; line += kRipThreads * 16)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(v + line));
  };
  const int n_dig = lay.n_digits;
  prefetch(__ldg(&lay.digits[0]));
#pragma unroll 1
  for (int di = 0; di < n_dig; ++di) {
    const int d = __ldg(&lay.digits[di]);  // digit di of the key shard
    const bool own = d == dj;
    {
      const u64 *kb = kbase + (long long)(2 * di) * kstride;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        cp_async16(kst + i * 32, kb + 64 * i);
        cp_async16(kst + (8 + i) * 32, kb + kstride + 64 * i);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    if (di + 1 < n_dig) prefetch(__ldg(&lay.digits[di + 1]));
    if (!own) {
      u64 x[kEpt];
      const u64 *tile = tbase + d * tstride;
      if (FP) fwd_rows_regs_fp_tw<LOG_M, false>(x, sm, twf, tile, tt, rr, row, P);
      else fwd_rows_regs<LOG_M, LAZY>(x, sm, tile, tt, rr, row, log_n, tw, P);
#pragma unroll
      for (int e = 0; e < kEpt; ++e) sm[padx<LOG_M>(rr, lidx<LOG_M, 0, G::NLO>(tt, e))] = x[e];
      __syncwarp();
    }
    cp_async_wait_all();  // this lane's own key pairs
    const bool first = di == 0, recentre = (di & 31) == 31;
    // this lane's pair i of the digit's value tile
    auto pair = [&](int i) {
      if (own) {
        const uint32_t src = galois_src((uint32_t)(tile0 + wofs + 64 * i), elt, log_n);
        ulonglong2 v = *reinterpret_cast<const ulonglong2 *>(climb + (src & ~1u));
        if (src & 1u) {
          const u64 tmp = v.x;
          v.x = v.y;
          v.y = tmp;
        }
        return v;
      }
      const int w = wofs + 64 * i;
      const int a = padx<LOG_M>(w >> LOG_M, w & (G::M - 1));  // pair's second word: a + 1
      return make_ulonglong2(sm[a], sm[a + 1]);
    };
    if constexpr (FP) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        u64 y[4];
        ulonglong2 k0[2], k1[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int i = 2 * h + q;
          k0[q] = kst[i * 32];
          k1[q] = kst[(8 + i) * 32];
          const ulonglong2 v = pair(i);
          y[2 * q] = own ? fp_bits(u64_to_fp(v.x)) : v.x;
          y[2 * q + 1] = own ? fp_bits(u64_to_fp(v.y)) : v.y;
        }
        uint32_t r0[8], r1[8];
        if (!first) {
          tmem::ld8(tacc + 8 * h, r0);
          tmem::ld8(tacc + 32 + 8 * h, r1);
          tmem::wait_ld(r0, r1);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const u64 b = (u & 1) ? k0[u >> 1].y : k0[u >> 1].x;
          const u64 a = (u & 1) ? k1[u >> 1].y : k1[u >> 1].x;
          const u64 v0 = ip_term_fp(tmem::pack(r0[2 * u], r0[2 * u + 1]), y[u], b, first, recentre, P);
          const u64 v1 = ip_term_fp(tmem::pack(r1[2 * u], r1[2 * u + 1]), y[u], a, first, recentre, P);
          r0[2 * u] = (uint32_t)v0;
          r0[2 * u + 1] = (uint32_t)(v0 >> 32);
          r1[2 * u] = (uint32_t)v1;
          r1[2 * u + 1] = (uint32_t)(v1 >> 32);
        }
        tmem::st8(tacc + 8 * h, r0);
        tmem::st8(tacc + 32 + 8 * h, r1);
      }
    } else {
      // Integer primes: 128-bit sums of the raw products, reduced only every
      // 32 digits (y < 4q, k < q < 2^60: a product is below 2^122, 32 of
      // them and a reduced remainder below 2^128).  Pair i of poly p sits in
      // columns [64 p + 8 i, 64 p + 8 i + 8): {lo, hi} of word x, then of y.
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const ulonglong2 k0 = kst[i * 32], k1 = kst[(8 + i) * 32];
        const ulonglong2 v = pair(i);
        uint32_t r0[8], r1[8];
        if (!first) {
          tmem::ld8(tacc + 8 * i, r0);
          tmem::ld8(tacc + 64 + 8 * i, r1);
          tmem::wait_ld(r0, r1);
        }
        ip_acc128(r0, 0, v.x, k0.x, first);
        ip_acc128(r0, 4, v.y, k0.y, first);
        ip_acc128(r1, 0, v.x, k1.x, first);
        ip_acc128(r1, 4, v.y, k1.y, first);
        tmem::st8(tacc + 8 * i, r0);
        tmem::st8(tacc + 64 + 8 * i, r1);
      }
      if (recentre) {  // rare (every 32 digits): kept out of the unrolled loop
        tmem::wait_st();
#pragma unroll 1
        for (int i = 0; i < 16; ++i) {
          uint32_t r[8];
          tmem::ld8(tacc + 8 * i, r);
          tmem::wait_ld(r);
          acc128_to_reduced(r, 0, P);
          acc128_to_reduced(r, 4, P);
          tmem::st8(tacc + 8 * i, r);
        }
      }
    }
    tmem::wait_st();
    __syncwarp();  // exchange buffer and key stage are reused by the next digit
  }
  u64 *o0 = a_cx + (long long)s * N + tile0 + wofs;
  u64 *o1 = o0 + (long long)lay.n_out * N;
  if constexpr (FP) {
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      uint32_t r0[8], r1[8];
      tmem::ld8(tacc + 8 * h, r0);
      tmem::ld8(tacc + 32 + 8 * h, r1);
      tmem::wait_ld(r0, r1);
      u64 v0[4], v1[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        v0[u] = fp_to_canon(as_fp(tmem::pack(r0[2 * u], r0[2 * u + 1])), P.qd, P.qinv);
        v1[u] = fp_to_canon(as_fp(tmem::pack(r1[2 * u], r1[2 * u + 1])), P.qd, P.qinv);
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int i = 2 * h + q;
        *reinterpret_cast<ulonglong2 *>(o0 + 64 * i) = make_ulonglong2(v0[2 * q], v0[2 * q + 1]);
        *reinterpret_cast<ulonglong2 *>(o1 + 64 * i) = make_ulonglong2(v1[2 * q], v1[2 * q + 1]);
      }
    }
  } else {
    const long long f0 = lay.fold_off ? lay.fold_off[2 * s] : -1;  // CTA-uniform
    if (f0 < 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t r0[8], r1[8];
        tmem::ld8(tacc + 8 * i, r0);
        tmem::ld8(tacc + 64 + 8 * i, r1);
        tmem::wait_ld(r0, r1);
        *reinterpret_cast<ulonglong2 *>(o0 + 64 * i) =
            make_ulonglong2(acc128_reduce(r0, 0, P), acc128_reduce(r0, 4, P));
        *reinterpret_cast<ulonglong2 *>(o1 + 64 * i) =
            make_ulonglong2(acc128_reduce(r1, 0, P), acc128_reduce(r1, 4, P));
      }
    } else {
      // P slot: the first (row) pass of the inverse transform of both polys
      // runs here on the finished tile, which goes back to the exchange
      // buffer in row order; the row-passed tile is written where the
      // separate inverse row pass would have put it.  Every P prime of a
      // folding level takes the non-lazy integer inverse path.
      const ulonglong2 *twi = T.inv + (long long)prime * N;
      u64 *fb = A.fold + mb * A.fold_bstride + tile0;
#pragma unroll 1
      for (int p = 0; p < 2; ++p) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          uint32_t r0[8], r1[8];
          tmem::ld8(tacc + 64 * p + 8 * i, r0);
          tmem::ld8(tacc + 64 * p + 8 * (i + 1), r1);
          tmem::wait_ld(r0, r1);
          const int w0 = wofs + 64 * i, w1 = w0 + 64;
          const int a0 = padx<LOG_M>(w0 >> LOG_M, w0 & (G::M - 1));
          const int a1 = padx<LOG_M>(w1 >> LOG_M, w1 & (G::M - 1));
          sm[a0] = acc128_reduce(r0, 0, P);
          sm[a0 + 1] = acc128_reduce(r0, 4, P);
          sm[a1] = acc128_reduce(r1, 0, P);
          sm[a1 + 1] = acc128_reduce(r1, 4, P);
        }
        __syncwarp();
        u64 x[kEpt];
        inv_rows_regs<LOG_M, false>(x, sm, tt, rr, row, log_n, twi, P);
        u64 *ot = fb + lay.fold_off[2 * s + p];
#pragma unroll
        for (int e = 0; e < kEpt; ++e) ot[rr * G::M + lidx<LOG_M, G::HI, 4>(tt, e)] = x[e];
        __syncwarp();  // the exchange buffer is refilled for poly 1
      }
    }
  }
}

// FP_SLOTS: the launch over lay.slots_fp (the FP64 body); otherwise the
// launch over lay.slots_int (the integer body).  One arithmetic kind per
// kernel keeps its code small enough for the instruction cache.
template <int LOG_M, bool FP_SLOTS>
__global__ void __launch_bounds__(kRipThreads, 16 / kRipWarps)
    k_modup_rows_ip(const __grid_constant__ RowsIpArgs A, ModUpDev mu, KsLayout lay, NttTables T) {
  // Warp w uses TMEM lane quarter w % 4 and kWg columns at kWg (w / 4): 64
  // for the FP64 sums (one 64-bit word per accumulator), 128 for the integer
  // 128-bit sums.  Shared memory caps how many CTAs share an SM so that their
  // columns never exceed the 512 of an SM, hence tmem::alloc never waits.
  constexpr uint32_t kWg = FP_SLOTS ? 64 : 128;
  constexpr uint32_t kCols = kWg * (kRipWarps / 4);
  static_assert(kRipWarps == 4 || kRipWarps == 8, "CTA of 4 or 8 warps");
  // Any mix of the two launches on one SM: at most 232448 / (smallest CTA)
  // CTAs, each with at most 128 columns.
  static_assert(kCols <= 128 &&
                    (rows_ip_smem_bytes<LOG_M, true>() < rows_ip_smem_bytes<LOG_M, false>()
                         ? rows_ip_smem_bytes<LOG_M, true>()
                         : rows_ip_smem_bytes<LOG_M, false>()) > 232448 / (512 / 128 + 1),
                "TMEM columns could be oversubscribed");
  extern __shared__ __align__(16) u64 dsm[];
  __shared__ uint32_t tmem_slot;
  u64 *sm = dsm;
  ulonglong2 *kst = reinterpret_cast<ulonglong2 *>(
      dsm + (size_t)rows_ip_rows<LOG_M>() * ((1 << LOG_M) + (1 << LOG_M) / 16));
  double *smtw = reinterpret_cast<double *>(kst + kRipWarps * 2 * 8 * 32);
  const int s = FP_SLOTS ? lay.slots_fp[blockIdx.y] : lay.slots_int[blockIdx.y];
  const int prime = mu.prime_of[lay.out_j[s]];
  const int warp = threadIdx.x >> 5;
  if (warp == 0) tmem::alloc(&tmem_slot, kCols);
  tmem::fence_before_sync();
  __syncthreads();
  tmem::fence_after_sync();
  // warp w: TMEM lanes 32 (w % 4) .., columns kWg (w / 4) ..
  const uint32_t tacc = tmem_slot + ((uint32_t)(32 * (warp & 3)) << 16) + kWg * (warp >> 2);
  if constexpr (FP_SLOTS) {
    if constexpr (kRipStageTw) {
      constexpr int R = rows_ip_rows<LOG_M>();
      stage_row_twiddles<LOG_M, R, kRipThreads>(
          smtw, T.fwd_fp + (long long)prime * (1 << T.log_n), T.log_n, (long long)blockIdx.x * R);
      cp_async_wait_all();
      __syncthreads();
    }
    rows_ip_body<LOG_M, true, false>(A, mu, lay, T, s, prime, sm, kst, smtw, tacc);
  } else {
    // Every integer prime (q0 below 2^58 as well as the P primes) takes
    // Harvey's [0, 4q) butterflies (valid for q < 2^62): one forward body
    // per kernel, since two of them overflow the instruction cache.
    rows_ip_body<LOG_M, false, false>(A, mu, lay, T, s, prime, sm, kst, smtw, tacc);
  }
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
template <int LOG_N>
__global__ void __launch_bounds__(kThreads, 3)
    k_moddown_cols(const u64 *__restrict__ y_base, const long long *__restrict__ y_off, u64 *z,
                   int n_q, const int *__restrict__ q_index, ModDownDev md, NttTables T,
                   const int *__restrict__ job_ps, int job0, long long y_bstride,
                   long long z_bstride) {
  constexpr int LOG_M = LOG_N / 2;  // column pass of 2^LOG_M points, stride M2
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int ps = job_ps[job0 + blockIdx.y];
  const int p = ps / n_q, s = ps % n_q;
  const int j = q_index[s];
  const PrimeDev P = T.primes[j];
  constexpr int log_n = LOG_N, N = 1 << LOG_N, M2 = N >> LOG_M;
  const int c = threadIdx.x % G::C, tt = (threadIdx.x / G::C) & (G::TT - 1);  // tt < TT (known range)
  const int col = blockIdx.x * G::C + c;
  const long long wo = (long long)j * md.alpha;
  y_base += blockIdx.z * y_bstride;  // member of the group
  z += blockIdx.z * z_bstride;
  auto src = [&](int i) { return y_base + y_off[p * md.alpha + i]; };
  auto fp_src = [&](int i) { return T.primes[md.first_p + i].q < kFpBound; };
  auto fill = [&](u64 (&x)[kEpt]) {
    bconv_fill<LOG_M>(x, tt, col, M2, md.alpha, src, fp_src, [](int) { return false; },
                      md.w + wo, md.wsh + wo, P);
  };
  u64 *out = z + ((long long)p * n_q + s) * N;
  auto store = [&](int r, int cl, u64 v) { out[(long long)r * M2 + cl] = v; };
  if (P.q < kFpBound) {
    // FP64 conversion (sources reduced mod q_j first when they do not fit):
    // spreads the work over the FP64 and integer pipes
    auto filld = [&](double (&x)[kEpt]) {
      bconv_fill_fp<LOG_M>(x, tt, col, M2, md.alpha, src,
                           [&](int i) { return T.primes[md.first_p + i].q; },
                           [](int) { return false; }, md.w + wo, md.wq + wo, P);
    };
    fwd_cols_fpd<LOG_M>(sm, col, tt, c, log_n, T.fwd_col + ((long long)j << LOG_M), P, filld,
                        store);
  } else {
    const ulonglong2 *tw = T.fwd + (long long)j * N;
    if (P.q < kFwdLazyBound) fwd_cols<LOG_M, true>(sm, col, tt, c, log_n, tw, P, fill, store);
    else fwd_cols<LOG_M, false>(sm, col, tt, c, log_n, tw, P, fill, store);
  }
}

// Per-member buffers of a group for the ModDown row pass (by value).
struct MdGroup {
  long long z_bstride, cx_bstride;
  u64 *ct0[kMaxGroup], *ct1[kMaxGroup];
  const u64 *g0[kMaxGroup];
};

// FP64 row twiddles of the ModDown row pass from the global table through L1
// (each CTA uses its rows' twiddles once) with no shared-memory twiddle
// block: 4 CTAs per SM.
constexpr bool kMdRowsStageTw = false;
// Row pass of z with the ModDown finish fused into the epilogue.
template <int LOG_M>
__global__ void __launch_bounds__(kThreads, kMdRowsStageTw ? 3 : 4)
    k_moddown_rows(const u64 *__restrict__ z, int n_q, const int *__restrict__ q_index,
                   const int *__restrict__ cx_slot, const u64 *__restrict__ cx,
                   long long cx_stride_poly, const __grid_constant__ MdGroup grp, int rotate,
                   const u64 *__restrict__ diag, ModDownDev md, NttTables T) {
  using G = RowGeom<LOG_M>;
  const int mb = blockIdx.z;  // member of the group
  z += mb * grp.z_bstride;
  cx += mb * grp.cx_bstride;
  u64 *const ct0 = grp.ct0[mb], *const ct1 = grp.ct1[mb];
  const u64 *const g0 = grp.g0[mb];
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
  if (kMdRowsStageTw && fp)
    stage_row_twiddles<LOG_M, G::R>(smtw, T.fwd_fp + (long long)j * N, log_n, row0);
  // Pull the epilogue operands into L2 while the butterflies run: one
  // prefetch per 128-byte line of the tile (4096 words = 256 lines).
  {
    const int line = threadIdx.x * 16;  // words; kThreads * 16 == kTile
    asm volatile("prefetch.global.L2 [%0];" ::"l"(cxp + line));
    if (base) asm volatile("prefetch.global.L2 [%0];" ::"l"(base + line));
  }
  u64 x[kEpt];
  if (fp) {
    if (kMdRowsStageTw) {
      cp_async_wait_all();
      __syncthreads();
      fwd_rows_regs_fp<LOG_M>(x, sm, smtw, tile, t, rr, row, row0, P);
    } else {
      const TwRowsGlobal<LOG_M> twg{T.fwd_fp + (long long)j * N, log_n, P.qinv};
      fwd_rows_regs_fp_tw<LOG_M, true>(x, sm, twg, tile, t, rr, row, P);
    }
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
template <int LOG_N>
__global__ void __launch_bounds__(kThreads, 3)
    k_rescale_cols(const u64 *__restrict__ last, u64 q_last, int last_fp, u64 *z, int n_q,
                   const int *__restrict__ q_index, NttTables T) {
  constexpr int LOG_M = LOG_N / 2;  // column pass of 2^LOG_M points, stride M2
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int p = blockIdx.y / n_q, s = blockIdx.y % n_q;
  const int j = q_index[s];
  const PrimeDev P = T.primes[j];
  constexpr int log_n = LOG_N, N = 1 << LOG_N, M2 = N >> LOG_M;
  const int c = threadIdx.x % G::C, tt = (threadIdx.x / G::C) & (G::TT - 1);  // tt < TT (known range)
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
                               long long cx_stride_poly, const MdGroup &grp, int rot,
                               const u64 *diag, const ModDownDev &md, const NttTables &T) {
  constexpr size_t smem =
      kMdRowsStageTw ? row_smem_bytes<LOG_M>() : (size_t)RowGeom<LOG_M>::SMEM * 8;
  static std::atomic<unsigned> attr_done{0};
  cudaError_t e = ensure_dynamic_smem(k_moddown_rows<LOG_M>, smem, attr_done);
  if (e != cudaSuccess) return e;
  k_moddown_rows<LOG_M><<<grid, kThreads, smem, s>>>(z, n_q, q_index, cx_slot, cx, cx_stride_poly,
                                                     grp, rot, diag, md, T);
  return cudaGetLastError();
}

template <int LOG_M>
cudaError_t launch_modup_rows_ip(cudaStream_t s, const RowsIpArgs &A, int group,
                                 const ModUpDev &mu, const KsLayout &lay, const NttTables &T,
                                 cudaStream_t side, cudaEvent_t ev_fork, cudaEvent_t ev_join) {
  constexpr size_t smem_fp = rows_ip_smem_bytes<LOG_M, true>();
  constexpr size_t smem_int = rows_ip_smem_bytes<LOG_M, false>();
  static std::atomic<unsigned> attr_fp{0}, attr_int{0};
  cudaError_t e = ensure_dynamic_smem(k_modup_rows_ip<LOG_M, true>, smem_fp, attr_fp);
  if (e == cudaSuccess) e = ensure_dynamic_smem(k_modup_rows_ip<LOG_M, false>, smem_int, attr_int);
  if (e != cudaSuccess) return e;
  // the integer slots (longer per tile, few tiles) on the side stream when
  // there is one, overlapping the FP64 launch on s
  const bool fork = side && ev_fork && ev_join && lay.n_slots_int > 0 && lay.n_slots_fp > 0;
  if (lay.n_slots_int > 0) {
    cudaStream_t si = s;
    if (fork) {
      if ((e = cudaEventRecord(ev_fork, s)) != cudaSuccess) return e;
      if ((e = cudaStreamWaitEvent(side, ev_fork, 0)) != cudaSuccess) return e;
      si = side;
    }
    const dim3 grid((1 << T.log_n) / kRipTile, lay.n_slots_int, group);
    k_modup_rows_ip<LOG_M, false><<<grid, kRipThreads, smem_int, si>>>(A, mu, lay, T);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (lay.n_slots_fp > 0) {
    const dim3 grid((1 << T.log_n) / kRipTile, lay.n_slots_fp, group);
    k_modup_rows_ip<LOG_M, true><<<grid, kRipThreads, smem_fp, s>>>(A, mu, lay, T);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (fork) {
    if ((e = cudaEventRecord(ev_join, side)) != cudaSuccess) return e;
    if ((e = cudaStreamWaitEvent(s, ev_join, 0)) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

inline int col_tiles(int log_n, int log_m) {
  const int M2 = (1 << log_n) >> log_m;
  return M2 / (kThreads / ((1 << log_m) / 16));
}

}  // namespace

cudaError_t ntt_inverse_scaled(const LimbMap &src, const LimbMap &dst, int n_limbs,
                               const ulonglong2 *scale, const NttTables &T, cudaStream_t s,
                               uint32_t elt, const MemberIn *mi, int group) {
  if (!ntt_supported_log_n(T.log_n) || n_limbs < 0 || n_limbs > 65535) return cudaErrorInvalidValue;
  if (group < 1 || group > kMaxGroup) return cudaErrorInvalidValue;
  if (n_limbs == 0) return cudaSuccess;
  // first pass: the ordinary inverse row pass, src (through elt) -> dst
  cudaError_t e = ntt_inverse_rows_only(src, n_limbs, T, s, &dst, elt, mi, group);
  if (e != cudaSuccess) return e;
  return ntt_inverse_cols_scaled(dst, n_limbs, scale, T, s, group);
}

cudaError_t ntt_inverse_scaled_pack(const LimbMap &src, const LimbMap &tmp, const LimbMap &dst,
                                    int n_limbs, const ulonglong2 *scale, const NttTables &T,
                                    cudaStream_t s, const MemberIn *mi, int group, int pack_from) {
  if (!ntt_supported_log_n(T.log_n) || n_limbs < 0 || n_limbs > 65535) return cudaErrorInvalidValue;
  if (group < 1 || group > kMaxGroup) return cudaErrorInvalidValue;
  if (n_limbs == 0) return cudaSuccess;
  cudaError_t e = ntt_inverse_rows_only(src, n_limbs, T, s, &tmp, 1, mi, group);
  if (e != cudaSuccess) return e;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), n_limbs, group);
  switch (T.log_n) {
    case 12: k_inv_cols_scaled_pack<12><<<grid, kThreads, 0, s>>>(tmp, dst, T, scale, pack_from); break;
    case 13: k_inv_cols_scaled_pack<13><<<grid, kThreads, 0, s>>>(tmp, dst, T, scale, pack_from); break;
    case 14: k_inv_cols_scaled_pack<14><<<grid, kThreads, 0, s>>>(tmp, dst, T, scale, pack_from); break;
    case 15: k_inv_cols_scaled_pack<15><<<grid, kThreads, 0, s>>>(tmp, dst, T, scale, pack_from); break;
    case 16: k_inv_cols_scaled_pack<16><<<grid, kThreads, 0, s>>>(tmp, dst, T, scale, pack_from); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t ntt_inverse_cols_scaled(const LimbMap &dst, int n_limbs, const ulonglong2 *scale,
                                    const NttTables &T, cudaStream_t s, int group) {
  if (!ntt_supported_log_n(T.log_n) || n_limbs < 0 || n_limbs > 65535) return cudaErrorInvalidValue;
  if (group < 1 || group > kMaxGroup) return cudaErrorInvalidValue;
  if (n_limbs == 0) return cudaSuccess;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), n_limbs, group);
  switch (T.log_n) {
    case 12: k_inv_cols_scaled<12><<<grid, kThreads, 0, s>>>(dst, T, scale); break;
    case 13: k_inv_cols_scaled<13><<<grid, kThreads, 0, s>>>(dst, T, scale); break;
    case 14: k_inv_cols_scaled<14><<<grid, kThreads, 0, s>>>(dst, T, scale); break;
    case 15: k_inv_cols_scaled<15><<<grid, kThreads, 0, s>>>(dst, T, scale); break;
    case 16: k_inv_cols_scaled<16><<<grid, kThreads, 0, s>>>(dst, T, scale); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t modup_fused_cols(const u64 *v_all, const long long *src_ref, u64 *t, const ModUpDev &mu,
                             const KsLayout &lay, const int *job_d, const int *job_s, int n_jobs,
                             int n_fp, const NttTables &T, cudaStream_t s, int group,
                             long long v_bstride, long long t_bstride, bool packed) {
  if (!ntt_supported_log_n(T.log_n) || n_jobs < 0 || n_jobs > 65535) return cudaErrorInvalidValue;
  if (mu.alpha > KS_MAX_ALPHA || n_fp < 0 || n_fp > n_jobs) return cudaErrorInvalidValue;
  if (group < 1 || group > kMaxGroup) return cudaErrorInvalidValue;
  if (n_jobs == 0) return cudaSuccess;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), n_jobs, group);
#define KS_MODUP_LAUNCH(LN)                                                                   \
  (packed ? k_modup_cols<LN, true><<<grid, kThreads, 0, s>>>(v_all, src_ref, t, mu, lay, job_d, \
                                                              job_s, 0, T, v_bstride, t_bstride) \
          : k_modup_cols<LN, false><<<grid, kThreads, 0, s>>>(v_all, src_ref, t, mu, lay, job_d, \
                                                               job_s, 0, T, v_bstride, t_bstride))
  switch (T.log_n) {
    case 12: KS_MODUP_LAUNCH(12); break;
    case 13: KS_MODUP_LAUNCH(13); break;
    case 14: KS_MODUP_LAUNCH(14); break;
    case 15: KS_MODUP_LAUNCH(15); break;
    case 16: KS_MODUP_LAUNCH(16); break;
    default: return cudaErrorInvalidValue;
  }
#undef KS_MODUP_LAUNCH
  return cudaGetLastError();
}

cudaError_t modup_rows_inner_product_group(const GroupArgs &G, const u64 *t, int key_limbs,
                                           u64 *cx, const ModUpDev &mu, const KsLayout &lay,
                                           const NttTables &T, cudaStream_t s, cudaStream_t side,
                                           cudaEvent_t ev_fork, cudaEvent_t ev_join) {
  if (G.n < 1 || G.n > kMaxGroup) return cudaErrorInvalidValue;
  for (int b = 0; b < G.n; ++b)
    if (!(G.in.elt[b] & 1u) || G.in.elt[b] >= (2u << T.log_n)) return cudaErrorInvalidValue;
  if (!ntt_supported_log_n(T.log_n) || lay.n_out < 0 || lay.n_out > 65535)
    return cudaErrorInvalidValue;
  if (lay.n_out == 0) return cudaSuccess;
  RowsIpArgs A{};
  A.t = t;
  A.cx = cx;
  A.t_bstride = G.t;
  A.cx_bstride = G.cx;
  A.key_limbs = key_limbs;
  for (int b = 0; b < G.n; ++b) {
    A.c_ntt[b] = G.in.in[b];
    A.elt[b] = G.in.elt[b];
    A.key[b] = G.key[b];
  }
  A.fold = G.fold;
  A.fold_bstride = G.fold_b;
  if (lay.fold_off && !G.fold) return cudaErrorInvalidValue;
  const int s2 = T.log_n - T.log_n / 2;
  switch (s2) {
    case 6: return launch_modup_rows_ip<6>(s, A, G.n, mu, lay, T, side, ev_fork, ev_join);
    case 7: return launch_modup_rows_ip<7>(s, A, G.n, mu, lay, T, side, ev_fork, ev_join);
    case 8: return launch_modup_rows_ip<8>(s, A, G.n, mu, lay, T, side, ev_fork, ev_join);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t modup_rows_inner_product(const u64 *t, const u64 *c_ntt, const u64 *key,
                                     int key_limbs, u64 *cx, const ModUpDev &mu,
                                     const KsLayout &lay, const NttTables &T, cudaStream_t s,
                                     uint32_t elt) {
  GroupArgs G{};
  G.n = 1;
  G.in.in[0] = c_ntt;
  G.in.elt[0] = elt;
  G.key[0] = key;
  return modup_rows_inner_product_group(G, t, key_limbs, cx, mu, lay, T, s);
}

cudaError_t moddown_fused_cols(const u64 *y_base, const long long *y_off, u64 *z, int n_q,
                               const int *q_index, const ModDownDev &md, const int *job_ps,
                               int n_fp, const NttTables &T, cudaStream_t s, int group,
                               long long y_bstride, long long z_bstride) {
  if (!ntt_supported_log_n(T.log_n) || n_q < 0 || 2 * n_q > 65535) return cudaErrorInvalidValue;
  if (md.alpha > KS_MAX_ALPHA || n_fp < 0 || n_fp > 2 * n_q) return cudaErrorInvalidValue;
  if (group < 1 || group > kMaxGroup) return cudaErrorInvalidValue;
  if (n_q == 0) return cudaSuccess;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), 2 * n_q, group);
  switch (T.log_n) {
    case 12: k_moddown_cols<12><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T, job_ps, 0, y_bstride, z_bstride); break;
    case 13: k_moddown_cols<13><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T, job_ps, 0, y_bstride, z_bstride); break;
    case 14: k_moddown_cols<14><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T, job_ps, 0, y_bstride, z_bstride); break;
    case 15: k_moddown_cols<15><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T, job_ps, 0, y_bstride, z_bstride); break;
    case 16: k_moddown_cols<16><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T, job_ps, 0, y_bstride, z_bstride); break;
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
  switch (T.log_n) {
    case 12: k_rescale_cols<12><<<grid, kThreads, 0, s>>>(last, q_last, fp, z, n_q, q_index, T); break;
    case 13: k_rescale_cols<13><<<grid, kThreads, 0, s>>>(last, q_last, fp, z, n_q, q_index, T); break;
    case 14: k_rescale_cols<14><<<grid, kThreads, 0, s>>>(last, q_last, fp, z, n_q, q_index, T); break;
    case 15: k_rescale_cols<15><<<grid, kThreads, 0, s>>>(last, q_last, fp, z, n_q, q_index, T); break;
    case 16: k_rescale_cols<16><<<grid, kThreads, 0, s>>>(last, q_last, fp, z, n_q, q_index, T); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

static cudaError_t moddown_rows_dispatch(const u64 *z, int n_q, const int *q_index,
                                         const int *cx_slot, const u64 *cx,
                                         long long cx_stride_poly, const MdGroup &grp, int group,
                                         bool rotate, const u64 *diag, const ModDownDev &md,
                                         const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_q < 0 || 2 * n_q > 65535) return cudaErrorInvalidValue;
  if (group < 1 || group > kMaxGroup) return cudaErrorInvalidValue;
  if (n_q == 0) return cudaSuccess;
  const int s2 = T.log_n - T.log_n / 2;
  dim3 grid((1 << T.log_n) / kTile, 2 * n_q, group);
  const int rot = rotate ? 1 : 0;
  switch (s2) {
    case 6: return launch_moddown_rows<6>(grid, s, z, n_q, q_index, cx_slot, cx, cx_stride_poly, grp, rot, diag, md, T);
    case 7: return launch_moddown_rows<7>(grid, s, z, n_q, q_index, cx_slot, cx, cx_stride_poly, grp, rot, diag, md, T);
    case 8: return launch_moddown_rows<8>(grid, s, z, n_q, q_index, cx_slot, cx, cx_stride_poly, grp, rot, diag, md, T);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t moddown_fused_rows(const u64 *z, int n_q, const int *q_index, const int *cx_slot,
                               const u64 *cx, long long cx_stride_poly, u64 *ct0, u64 *ct1,
                               const u64 *g0, bool rotate, const u64 *diag,
                               const ModDownDev &md, const NttTables &T, cudaStream_t s) {
  MdGroup grp{};
  grp.ct0[0] = ct0;
  grp.ct1[0] = ct1;
  grp.g0[0] = g0;
  return moddown_rows_dispatch(z, n_q, q_index, cx_slot, cx, cx_stride_poly, grp, 1, rotate,
                               diag, md, T, s);
}

cudaError_t moddown_fused_rows_group(const GroupArgs &G, const u64 *z, int n_q,
                                     const int *q_index, const int *cx_slot, const u64 *cx,
                                     long long cx_stride_poly, bool rotate, const ModDownDev &md,
                                     const NttTables &T, cudaStream_t s) {
  if (G.n < 1 || G.n > kMaxGroup) return cudaErrorInvalidValue;
  MdGroup grp{};
  grp.z_bstride = G.z;
  grp.cx_bstride = G.cx;
  for (int b = 0; b < G.n; ++b) {
    grp.ct0[b] = G.ct0[b];
    grp.ct1[b] = G.ct1[b];
    grp.g0[b] = G.g0p[b];
  }
  return moddown_rows_dispatch(z, n_q, q_index, cx_slot, cx, cx_stride_poly, grp, G.n, rotate,
                               nullptr, md, T, s);
}

}  // namespace ksb
