// ks_ntt.cu -- batched negacyclic NTT/INTT kernels for N = 2^12 .. 2^16.
//
// Each transform is two launches (column pass, row pass) built from the
// blocks in ks_ntt_impl.cuh.  Every CTA serves one limb, so the prime and the
// choice between the lazy butterflies (small primes) and Harvey's reduced
// butterflies (60-bit primes) are CTA-uniform.
#include "ks_ntt.cuh"
#include "ks_launch.cuh"
#include "ks_launch.cuh"
#include "ks_ntt_impl.cuh"
#include "ks_galois.cuh"

namespace ksb {
namespace {

using namespace ntt;

__device__ __forceinline__ void limb_of(const LimbMap &m, int i, u64 *&ptr, int &prime) {
  ptr = m.base + (m.offsets ? m.offsets[i] : (long long)i * m.stride);
  prime = m.prime_tab ? m.prime_tab[i] : m.first_prime + (i % m.period);
}

template <int LOG_N, bool FWD>
__global__ void __launch_bounds__(kThreads, 4) ntt_cols(LimbMap m, NttTables T) {
  constexpr int LOG_M = LOG_N / 2;  // column pass of 2^LOG_M points; stride M2 is a constant
  using G = ColGeom<LOG_M>;
  __shared__ u64 sm[G::SMEM];
  u64 *a;
  int prime;
  limb_of(m, blockIdx.y, a, prime);
  if (prime < 0) return;
  const PrimeDev P = T.primes[prime];
  constexpr int log_n = LOG_N, N = 1 << LOG_N, M2 = N >> LOG_M;
  const ulonglong2 *tw = (FWD ? T.fwd : T.inv) + (long long)prime * N;
  const int c = threadIdx.x % G::C, t = (threadIdx.x / G::C) & (G::TT - 1);  // known range t < TT
  const int col = blockIdx.x * G::C + c;
  auto load = [&](int r, int cl) { return a[(long long)r * M2 + cl]; };
  auto fill = [&](u64 (&x)[kEpt]) { fill_cols<LOG_M>(x, t, col, load); };
  auto store = [&](int r, int cl, u64 v) { a[(long long)r * M2 + cl] = v; };
  if (P.q < kFpBound) {
    const double2 *twf = (FWD ? T.fwd_col : T.inv_col) + ((long long)prime << LOG_M);
    if (FWD) {
      fwd_cols_fp<LOG_M>(sm, col, t, c, log_n, twf, P, fill, store);
    } else {
      const double2 s0 = make_double2(P.ninv_d, P.ninv_q), s1 = make_double2(P.w1ninv_d, P.w1ninv_q);
      inv_cols_fp<LOG_M>(sm, col, t, c, log_n, twf, P, s0, s1, load, store);
    }
  } else if (FWD) {
    if (P.q < kFwdLazyBound) fwd_cols<LOG_M, true>(sm, col, t, c, log_n, tw, P, fill, store);
    else fwd_cols<LOG_M, false>(sm, col, t, c, log_n, tw, P, fill, store);
  } else {
    const ulonglong2 s0 = make_ulonglong2(P.ninv, P.ninv_sh);
    const ulonglong2 s1 = make_ulonglong2(P.w1ninv, P.w1ninv_sh);
    if (P.q < kInvLazyBound) inv_cols<LOG_M, true>(sm, col, t, c, log_n, tw, P, s0, s1, load, store);
    else inv_cols<LOG_M, false>(sm, col, t, c, log_n, tw, P, s0, s1, load, store);
  }
}

// elt (inverse direction only): the input is read through the automorphism
// X -> X^elt (input slot galois_src(i) feeds slot i; the tile gathers from
// one aligned source tile); elt = 1 reads it as it is.
// The row twiddles of FP64 primes: staged per CTA in shared memory (true)
// or read from the global table through L1 (false: no twiddle block, 4 CTAs
// per SM).  Each CTA uses its twiddles once, so staging only adds a copy:
// reading them from L1 took the config-2 forward transform from 2.20 to
// 1.99 ms and the inverse from 2.43 to 2.14 ms.
constexpr bool kRowsStageTw = false;
template <int LOG_M, bool FWD>
__global__ void __launch_bounds__(kThreads, kRowsStageTw ? 3 : 4)
    ntt_rows(LimbMap m, LimbMap mo, NttTables T,
                                                     uint32_t elt,
                                                     const __grid_constant__ MemberIn mi) {
  using G = RowGeom<LOG_M>;
  extern __shared__ __align__(16) u64 dsm[];
  u64 *sm = dsm;
  double *smtw = reinterpret_cast<double *>(dsm + G::SMEM);
  u64 *a, *o;
  int prime, prime_o;
  limb_of(m, blockIdx.y, a, prime);
  limb_of(mo, blockIdx.y, o, prime_o);  // output limb (== input limb when in place)
  if (prime < 0) return;
  const int mb = blockIdx.z;  // member of the group
  if (mi.in[0]) {
    a = const_cast<u64 *>(mi.in[mb]) + (a - m.base);
    elt = mi.elt[mb];
  } else {
    a += mb * m.bstride;
  }
  o += mb * mo.bstride;
  const PrimeDev P = T.primes[prime];
  const int log_n = T.log_n, N = 1 << log_n;
  const ulonglong2 *tw = (FWD ? T.fwd : T.inv) + (long long)prime * N;
  const int t = threadIdx.x % G::TT, rr = threadIdx.x / G::TT;
  const u64 *tile = a + (long long)blockIdx.x * kTile;
  u64 *otile = o + (long long)blockIdx.x * kTile;
  const long long row0 = (long long)blockIdx.x * G::R, row = row0 + rr;
  u64 x[kEpt];
  const bool fp = P.q < kFpBound;
  const double *twfp = (FWD ? T.fwd_fp : T.inv_fp) + (long long)prime * N;
  if (kRowsStageTw && fp) stage_row_twiddles<LOG_M, G::R>(smtw, twfp, log_n, row0);
  const TwRowsGlobal<LOG_M> twg{twfp, log_n, P.qinv};
  if (FWD) {
    if (fp) {
      if (kRowsStageTw) {
        cp_async_wait_all();
        __syncthreads();
        fwd_rows_regs_fp<LOG_M>(x, sm, smtw, tile, t, rr, row, row0, P);
      } else {
        fwd_rows_regs_fp_tw<LOG_M, true>(x, sm, twg, tile, t, rr, row, P);
      }
    } else if (P.q < kFwdLazyBound) {
      fwd_rows_regs<LOG_M, true>(x, sm, tile, t, rr, row, log_n, tw, P);
    } else {
      fwd_rows_regs<LOG_M, false>(x, sm, tile, t, rr, row, log_n, tw, P);
    }
#pragma unroll
    for (int e = 0; e < kEpt; ++e) sm[padx<LOG_M>(rr, lidx<LOG_M, 0, G::NLO>(t, e))] = x[e];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kEpt; ++i) {
      const int lin = threadIdx.x + i * kThreads;
      otile[lin] = sm[padx<LOG_M>(lin >> LOG_M, lin & (G::M - 1))];
    }
  } else {
    if (elt == 1u) {
#pragma unroll
      for (int i = 0; i < kEpt; ++i) {
        const int lin = threadIdx.x + i * kThreads;
        sm[padx<LOG_M>(lin >> LOG_M, lin & (G::M - 1))] = tile[lin];
      }
    } else {
      const uint32_t t0 = (uint32_t)blockIdx.x * kTile;
      const u64 *stile = a + (galois_src(t0, elt, log_n) & ~(uint32_t)(kTile - 1));
#pragma unroll
      for (int i = 0; i < kEpt; ++i) {
        const int lin = threadIdx.x + i * kThreads;
        sm[padx<LOG_M>(lin >> LOG_M, lin & (G::M - 1))] =
            stile[galois_src(t0 + lin, elt, log_n) & (uint32_t)(kTile - 1)];
      }
    }
    if (kRowsStageTw && fp) cp_async_wait_all();
    __syncthreads();
    if (fp) {
      if (kRowsStageTw) inv_rows_regs_fp<LOG_M>(x, sm, smtw, t, rr, row, row0, P);
      else inv_rows_regs_fp_tw<LOG_M>(x, sm, twg, t, rr, row, P);
    }
    else if (P.q < kInvLazyBound) inv_rows_regs<LOG_M, true>(x, sm, t, rr, row, log_n, tw, P);
    else inv_rows_regs<LOG_M, false>(x, sm, t, rr, row, log_n, tw, P);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) otile[rr * G::M + lidx<LOG_M, G::HI, 4>(t, e)] = x[e];
  }
}

template <int LOG_N, bool FWD>
cudaError_t launch_cols(const LimbMap &m, int n_limbs, const NttTables &T, cudaStream_t s) {
  constexpr int LOG_M = LOG_N / 2, M2 = (1 << LOG_N) >> LOG_M;
  dim3 grid(M2 / ColGeom<LOG_M>::C, n_limbs);
  ntt_cols<LOG_N, FWD><<<grid, kThreads, 0, s>>>(m, T);
  return cudaGetLastError();
}
template <int LOG_M, bool FWD>
cudaError_t launch_rows(const LimbMap &m, const LimbMap &mo, int n_limbs, const NttTables &T,
                        cudaStream_t s, uint32_t elt = 1, const MemberIn *mi = nullptr,
                        int group = 1) {
  constexpr size_t smem =
      kRowsStageTw ? row_smem_bytes<LOG_M>() : (size_t)RowGeom<LOG_M>::SMEM * 8;
  static std::atomic<unsigned> attr_done{0};
  cudaError_t e = ensure_dynamic_smem(ntt_rows<LOG_M, FWD>, smem, attr_done);
  if (e != cudaSuccess) return e;
  dim3 grid((1 << T.log_n) / kTile, n_limbs, group);
  const MemberIn none{};
  ntt_rows<LOG_M, FWD><<<grid, kThreads, smem, s>>>(m, mo, T, elt, mi ? *mi : none);
  return cudaGetLastError();
}

template <bool FWD>
cudaError_t launch_pass(bool cols, int log_m, const LimbMap &m, int n, const NttTables &T,
                        cudaStream_t s, const LimbMap *mo = nullptr, uint32_t elt = 1,
                        const MemberIn *mi = nullptr, int group = 1) {
  const LimbMap &o = mo ? *mo : m;
  if (cols) {
    switch (T.log_n) {
      case 12: return launch_cols<12, FWD>(m, n, T, s);
      case 13: return launch_cols<13, FWD>(m, n, T, s);
      case 14: return launch_cols<14, FWD>(m, n, T, s);
      case 15: return launch_cols<15, FWD>(m, n, T, s);
      case 16: return launch_cols<16, FWD>(m, n, T, s);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (log_m) {
    case 6: return launch_rows<6, FWD>(m, o, n, T, s, elt, mi, group);
    case 7: return launch_rows<7, FWD>(m, o, n, T, s, elt, mi, group);
    case 8: return launch_rows<8, FWD>(m, o, n, T, s, elt, mi, group);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool ntt_supported_log_n(int log_n) { return log_n >= 12 && log_n <= 16; }

cudaError_t ntt_forward(const LimbMap &m, int n_limbs, const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_limbs < 0 || n_limbs > 65535) return cudaErrorInvalidValue;
  if (n_limbs == 0) return cudaSuccess;
  const int s1 = T.log_n / 2, s2 = T.log_n - s1;
  cudaError_t e = launch_pass<true>(true, s1, m, n_limbs, T, s);
  if (e != cudaSuccess) return e;
  return launch_pass<true>(false, s2, m, n_limbs, T, s);
}

cudaError_t ntt_forward_rows_only(const LimbMap &m, int n_limbs, const NttTables &T,
                                  cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_limbs < 0 || n_limbs > 65535) return cudaErrorInvalidValue;
  if (n_limbs == 0) return cudaSuccess;
  return launch_pass<true>(false, T.log_n - T.log_n / 2, m, n_limbs, T, s);
}

cudaError_t ntt_inverse_rows_only(const LimbMap &m, int n_limbs, const NttTables &T,
                                  cudaStream_t s, const LimbMap *out, uint32_t elt,
                                  const MemberIn *mi, int group) {
  if (!ntt_supported_log_n(T.log_n) || n_limbs < 0 || n_limbs > 65535) return cudaErrorInvalidValue;
  if (group < 1 || group > kMaxGroup) return cudaErrorInvalidValue;
  if (mi && mi->in[0]) {  // per-member inputs: every member's element checked, output separate
    for (int b = 0; b < group; ++b)
      if (!mi->in[b] || !(mi->elt[b] & 1u) || mi->elt[b] >= (2u << T.log_n))
        return cudaErrorInvalidValue;
    if (!out) return cudaErrorInvalidValue;
  } else {
    if (!(elt & 1u) || elt >= (2u << T.log_n)) return cudaErrorInvalidValue;
    if (elt != 1u && (!out || out->base == m.base)) return cudaErrorInvalidValue;  // gather needs a separate output
  }
  if (n_limbs == 0) return cudaSuccess;
  return launch_pass<false>(false, T.log_n - T.log_n / 2, m, n_limbs, T, s, out, elt, mi, group);
}

cudaError_t ntt_inverse(const LimbMap &m, int n_limbs, const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_limbs < 0 || n_limbs > 65535) return cudaErrorInvalidValue;
  if (n_limbs == 0) return cudaSuccess;
  const int s1 = T.log_n / 2, s2 = T.log_n - s1;
  cudaError_t e = launch_pass<false>(false, s2, m, n_limbs, T, s);
  if (e != cudaSuccess) return e;
  return launch_pass<false>(true, s1, m, n_limbs, T, s);
}

}  // namespace ksb
