// ks_fused.cu -- fused key-switch kernels (sm_100a).
//
// ModUp base extension fused into the first NTT pass: every element of a
// column tile is produced from the alpha scaled coefficient limbs of its
// digit (5 L2-resident loads + 5 multiply-accumulates + one Barrett
// reduction) and fed straight into the butterflies, so the extended limbs in
// coefficient form never touch HBM.  The scaled inputs
// v_i = [x_i * (Q_d/q_i)^-1]_{q_i} come out of the input INTT, whose last
// stage already multiplies by N^-1 and now also by (Q_d/q_i)^-1.
//
// ModDown: the P -> Q conversion is fused the same way into the first pass,
// and the second pass ends with (cx - z) * P^-1 and the add to the
// ciphertext, so the converted limbs never reach HBM in NTT form either.
#include "ks_fused.cuh"
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
    // scale entries of FP64 primes hold the bits of {s, fl(s/q)}
    inv_cols_fp<LOG_M>(sm, col, t, c, log_n, T.inv_fp + (long long)prime * N, P,
                       make_double2(as_fp(s0.x), as_fp(s0.y)), make_double2(as_fp(s1.x), as_fp(s1.y)),
                       load, store);
  } else if (P.q < kInvLazyBound) {
    inv_cols<LOG_M, true>(sm, col, t, c, log_n, tw, P, s0, s1, load, store);
  } else {
    inv_cols<LOG_M, false>(sm, col, t, c, log_n, tw, P, s0, s1, load, store);
  }
}

// ---------------------------------------------------------------------------
// ModUp: base conversion + forward column pass
// ---------------------------------------------------------------------------
template <int LOG_M>
__global__ void __launch_bounds__(kThreads)
    k_modup_cols(const u64 *__restrict__ v_all, const int *__restrict__ src_slot, u64 *t,
                 ModUpDev mu, KsLayout lay, const int *__restrict__ job_d,
                 const int *__restrict__ job_s, NttTables T) {
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int d = job_d[blockIdx.y], s = job_s[blockIdx.y];
  const int j = lay.out_j[s];
  const int prime = mu.prime_of[j];
  const PrimeDev P = T.primes[prime];
  const int log_n = T.log_n, N = 1 << log_n, M2 = N >> LOG_M;
  const ulonglong2 *tw = T.fwd + (long long)prime * N;
  const int c = threadIdx.x % G::C, tt = threadIdx.x / G::C;
  const int col = blockIdx.x * G::C + c;
  const int n_src = min(mu.alpha, mu.Ql - d * mu.alpha);
  const u64 *src[KS_MAX_ALPHA];
  u64 w[KS_MAX_ALPHA];
#pragma unroll
  for (int i = 0; i < KS_MAX_ALPHA; ++i) {
    if (i < n_src) {
      src[i] = v_all + (long long)src_slot[d * mu.alpha + i] * N;
      w[i] = mu.w[((long long)d * mu.QlP + j) * mu.alpha + i];
    }
  }
  auto load = [&](int r, int cl) {
    const long long k = (long long)r * M2 + cl;
    u128v acc = {0, 0};
#pragma unroll
    for (int i = 0; i < KS_MAX_ALPHA; ++i)
      if (i < n_src) mac(acc, __ldg(src[i] + k), w[i]);
    return barrett128(acc, P.q, P.br_hi, P.br_lo);
  };
  u64 *out = t + ((long long)d * lay.n_out + s) * N;
  auto store = [&](int r, int cl, u64 v) { out[(long long)r * M2 + cl] = v; };
  if (P.q < kFpBound)
    fwd_cols_fp<LOG_M>(sm, col, tt, c, log_n, T.fwd_fp + (long long)prime * N, P, load, store);
  else if (P.q < kFwdLazyBound) fwd_cols<LOG_M, true>(sm, col, tt, c, log_n, tw, P, load, store);
  else fwd_cols<LOG_M, false>(sm, col, tt, c, log_n, tw, P, load, store);
}

// ---------------------------------------------------------------------------
// ModDown: base conversion P -> q_j + forward column pass
// ---------------------------------------------------------------------------
template <int LOG_M>
__global__ void __launch_bounds__(kThreads)
    k_moddown_cols(const u64 *__restrict__ y_base, const long long *__restrict__ y_off, u64 *z,
                   int n_q, const int *__restrict__ q_index, ModDownDev md, NttTables T) {
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int p = blockIdx.y / n_q, s = blockIdx.y % n_q;
  const int j = q_index[s];
  const PrimeDev P = T.primes[j];
  const int log_n = T.log_n, N = 1 << log_n, M2 = N >> LOG_M;
  const ulonglong2 *tw = T.fwd + (long long)j * N;
  const int c = threadIdx.x % G::C, tt = threadIdx.x / G::C;
  const int col = blockIdx.x * G::C + c;
  const u64 *src[KS_MAX_ALPHA];
  u64 w[KS_MAX_ALPHA];
#pragma unroll
  for (int i = 0; i < KS_MAX_ALPHA; ++i) {
    if (i < md.alpha) {
      src[i] = y_base + y_off[p * md.alpha + i];
      w[i] = md.w[(long long)j * md.alpha + i];
    }
  }
  auto load = [&](int r, int cl) {
    const long long k = (long long)r * M2 + cl;
    u128v acc = {0, 0};
#pragma unroll
    for (int i = 0; i < KS_MAX_ALPHA; ++i)
      if (i < md.alpha) mac(acc, __ldg(src[i] + k), w[i]);
    return barrett128(acc, P.q, P.br_hi, P.br_lo);
  };
  u64 *out = z + ((long long)p * n_q + s) * N;
  auto store = [&](int r, int cl, u64 v) { out[(long long)r * M2 + cl] = v; };
  if (P.q < kFpBound)
    fwd_cols_fp<LOG_M>(sm, col, tt, c, log_n, T.fwd_fp + (long long)j * N, P, load, store);
  else if (P.q < kFwdLazyBound) fwd_cols<LOG_M, true>(sm, col, tt, c, log_n, tw, P, load, store);
  else fwd_cols<LOG_M, false>(sm, col, tt, c, log_n, tw, P, load, store);
}

// Row pass of z with the ModDown finish fused into the epilogue.
template <int LOG_M>
__global__ void __launch_bounds__(kThreads)
    k_moddown_rows(const u64 *__restrict__ z, int n_q, const int *__restrict__ q_index,
                   const int *__restrict__ cx_slot, const u64 *__restrict__ cx,
                   long long cx_stride_poly, u64 *ct0, u64 *ct1, const u64 *g0, int rotate,
                   ModDownDev md, NttTables T) {
  using G = RowGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  const int p = blockIdx.y / n_q, s = blockIdx.y % n_q;
  const int j = q_index[s];
  const PrimeDev P = T.primes[j];
  const int log_n = T.log_n, N = 1 << log_n;
  const ulonglong2 *tw = T.fwd + (long long)j * N;
  const int t = threadIdx.x % G::TT, rr = threadIdx.x / G::TT;
  const long long tile0 = (long long)blockIdx.x * kTile;
  const u64 *tile = z + ((long long)p * n_q + s) * N + tile0;
  const long long row = (long long)blockIdx.x * G::R + rr;
  u64 x[kEpt];
  if (P.q < kFpBound)
    fwd_rows_regs_fp<LOG_M>(x, sm, tile, t, rr, row, log_n, T.fwd_fp + (long long)j * N, P);
  else if (P.q < kFwdLazyBound) fwd_rows_regs<LOG_M, true>(x, sm, tile, t, rr, row, log_n, tw, P);
  else fwd_rows_regs<LOG_M, false>(x, sm, tile, t, rr, row, log_n, tw, P);
  const ulonglong2 pinv = md.pinv[j];
  const u64 *cxp = cx + p * cx_stride_poly + (long long)cx_slot[s] * N;
  u64 *dst = (p == 0 ? ct0 : ct1) + (long long)s * N;
  const u64 *base = (p == 0) ? (rotate ? g0 + (long long)s * N : dst) : (rotate ? nullptr : dst);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) {
    const long long k = row * G::M + lidx<LOG_M, 0, G::NLO>(t, e);
    const u64 o = mul_shoup(cxp[k] + P.q - x[e], pinv.x, pinv.y, P.q);
    dst[k] = base ? add_mod(base[k], o, P.q) : o;
  }
}

inline int col_tiles(int log_n, int log_m) {
  const int M2 = (1 << log_n) >> log_m;
  return M2 / (kThreads / ((1 << log_m) / 16));
}

}  // namespace

cudaError_t ntt_inverse_scaled(const LimbMap &m, int n_limbs, const ulonglong2 *scale,
                               const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_limbs < 0 || n_limbs > 65535) return cudaErrorInvalidValue;
  if (n_limbs == 0) return cudaSuccess;
  // first pass: the ordinary inverse row pass
  cudaError_t e = ntt_inverse_rows_only(m, n_limbs, T, s);
  if (e != cudaSuccess) return e;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), n_limbs);
  switch (s1) {
    case 6: k_inv_cols_scaled<6><<<grid, kThreads, 0, s>>>(m, T, scale); break;
    case 7: k_inv_cols_scaled<7><<<grid, kThreads, 0, s>>>(m, T, scale); break;
    case 8: k_inv_cols_scaled<8><<<grid, kThreads, 0, s>>>(m, T, scale); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t modup_fused_cols(const u64 *v_all, const int *src_slot, u64 *t, const ModUpDev &mu,
                             const KsLayout &lay, const int *job_d, const int *job_s, int n_jobs,
                             const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_jobs < 0 || n_jobs > 65535) return cudaErrorInvalidValue;
  if (mu.alpha > KS_MAX_ALPHA) return cudaErrorInvalidValue;
  if (n_jobs == 0) return cudaSuccess;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), n_jobs);
  switch (s1) {
    case 6: k_modup_cols<6><<<grid, kThreads, 0, s>>>(v_all, src_slot, t, mu, lay, job_d, job_s, T); break;
    case 7: k_modup_cols<7><<<grid, kThreads, 0, s>>>(v_all, src_slot, t, mu, lay, job_d, job_s, T); break;
    case 8: k_modup_cols<8><<<grid, kThreads, 0, s>>>(v_all, src_slot, t, mu, lay, job_d, job_s, T); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t moddown_fused_cols(const u64 *y_base, const long long *y_off, u64 *z, int n_q,
                               const int *q_index, const ModDownDev &md, const NttTables &T,
                               cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_q < 0 || 2 * n_q > 65535) return cudaErrorInvalidValue;
  if (md.alpha > KS_MAX_ALPHA) return cudaErrorInvalidValue;
  if (n_q == 0) return cudaSuccess;
  const int s1 = T.log_n / 2;
  dim3 grid(col_tiles(T.log_n, s1), 2 * n_q);
  switch (s1) {
    case 6: k_moddown_cols<6><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T); break;
    case 7: k_moddown_cols<7><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T); break;
    case 8: k_moddown_cols<8><<<grid, kThreads, 0, s>>>(y_base, y_off, z, n_q, q_index, md, T); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t moddown_fused_rows(const u64 *z, int n_q, const int *q_index, const int *cx_slot,
                               const u64 *cx, long long cx_stride_poly, u64 *ct0, u64 *ct1,
                               const u64 *g0, bool rotate, const ModDownDev &md,
                               const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_q < 0 || 2 * n_q > 65535) return cudaErrorInvalidValue;
  if (n_q == 0) return cudaSuccess;
  const int s2 = T.log_n - T.log_n / 2;
  dim3 grid((1 << T.log_n) / kTile, 2 * n_q);
  const int rot = rotate ? 1 : 0;
  switch (s2) {
    case 6: k_moddown_rows<6><<<grid, kThreads, 0, s>>>(z, n_q, q_index, cx_slot, cx, cx_stride_poly, ct0, ct1, g0, rot, md, T); break;
    case 7: k_moddown_rows<7><<<grid, kThreads, 0, s>>>(z, n_q, q_index, cx_slot, cx, cx_stride_poly, ct0, ct1, g0, rot, md, T); break;
    case 8: k_moddown_rows<8><<<grid, kThreads, 0, s>>>(z, n_q, q_index, cx_slot, cx, cx_stride_poly, ct0, ct1, g0, rot, md, T); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace ksb
