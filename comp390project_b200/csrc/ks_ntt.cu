// ks_ntt.cu -- two-pass batched NTT/INTT for N = 2^12 .. 2^16.
//
// The length-N transform is split as N = M1 * M2 (M1 = 2^(logN/2)).  The
// column pass runs the logN/2 stages whose butterflies span the high index
// bits (each column of M1 elements at stride M2 is an independent sub-
// transform); the row pass runs the remaining stages inside contiguous rows
// of M2 elements.  Every thread keeps 16 elements in registers and runs four
// butterfly stages on them (a radix-16 step); one shared-memory exchange
// re-partitions the sub-transform for the next four stages.
//
// Column-pass tiles are 16 adjacent columns wide (for M1 = 256) with the lane
// index running along the contiguous column direction, so every global access
// is a full 128-byte row segment.  Row-pass tiles are 4096 contiguous words.
#include "ks_ntt.cuh"

namespace ksb {
namespace {

constexpr int kThreads = 256;
constexpr int kEpt = 16;                     // elements per thread
constexpr int kTile = kThreads * kEpt;       // 4096 words per CTA

__device__ __forceinline__ void limb_of(const LimbMap &m, int i, u64 *&ptr, int &prime) {
  ptr = m.base + (m.offsets ? m.offsets[i] : (long long)i * m.stride);
  prime = m.prime_tab ? m.prime_tab[i] : m.first_prime + (i % m.period);
}

// Register e = (g << NB) | v holds the local index
//   ((u >> LO) << (LO + NB)) | (v << LO) | (u & ((1 << LO) - 1)),  u = (g << LOG_T) | t.
template <int LOG_M, int LO, int NB>
__device__ __forceinline__ int lidx(int t, int e) {
  constexpr int LOG_T = LOG_M - 4;
  const int g = e >> NB, v = e & ((1 << NB) - 1);
  const int u = (g << LOG_T) | t;
  return ((u >> LO) << (LO + NB)) | (v << LO) | (u & ((1 << LO) - 1));
}

// Forward stages on local bits [LO, LO+NB), high bit first.  Global bit of
// local bit b is b + gofs; the twiddle of the pair whose lower element has
// local index i is tw[(1 << (logN-1-b-gofs)) + (((prefix << LOG_M) | i) >> (b+1))].
template <int LOG_M, int LO, int NB>
__device__ __forceinline__ void fwd_round(u64 (&x)[kEpt], int t, long long prefix, int gofs,
                                          int log_n, const ulonglong2 *__restrict__ tw, u64 q,
                                          u64 two_q) {
#pragma unroll
  for (int k = NB - 1; k >= 0; --k) {
    const int b = LO + k;
    const int base = 1 << (log_n - 1 - b - gofs);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) {
      if (e & (1 << k)) continue;
      const long long H = (prefix << LOG_M) | lidx<LOG_M, LO, NB>(t, e);
      const ulonglong2 w = __ldg(&tw[base + (int)(H >> (b + 1))]);
      ct_bfly(x[e], x[e | (1 << k)], w.x, w.y, q, two_q);
    }
  }
}

// Inverse stages on local bits [LO, LO+NB), low bit first.  If LAST, the top
// stage of this round is the final stage of the transform (N^-1 folded in).
template <int LOG_M, int LO, int NB, bool LAST>
__device__ __forceinline__ void inv_round(u64 (&x)[kEpt], int t, long long prefix, int gofs,
                                          int log_n, const ulonglong2 *__restrict__ tw,
                                          const PrimeDev &P) {
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const int b = LO + k;
    const int base = 1 << (log_n - 1 - b - gofs);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) {
      if (e & (1 << k)) continue;
      if (LAST && k == NB - 1) {
        gs_bfly_last(x[e], x[e | (1 << k)], P);
      } else {
        const long long H = (prefix << LOG_M) | lidx<LOG_M, LO, NB>(t, e);
        const ulonglong2 w = __ldg(&tw[base + (int)(H >> (b + 1))]);
        gs_bfly(x[e], x[e | (1 << k)], w.x, w.y, P.q, P.two_q);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Column pass: sub-transforms of length M = 2^LOG_M at stride M2 = N / M.
// ---------------------------------------------------------------------------
template <int LOG_M, bool FWD>
__global__ void __launch_bounds__(kThreads) ntt_cols(LimbMap m, NttTables T) {
  constexpr int M = 1 << LOG_M, LOG_T = LOG_M - 4, TT = 1 << LOG_T, C = kThreads / TT;
  constexpr int HI = LOG_M - 4, NLO = LOG_M - 4;  // high round: bits [HI, LOG_M); low: [0, NLO)
  __shared__ u64 sm[M * C];
  u64 *a;
  int prime;
  limb_of(m, blockIdx.y, a, prime);
  if (prime < 0) return;
  const PrimeDev P = T.primes[prime];
  const int log_n = T.log_n, N = 1 << log_n, M2 = N >> LOG_M, gofs = log_n - LOG_M;
  const ulonglong2 *tw = (FWD ? T.fwd : T.inv) + (long long)prime * N;
  const int c = threadIdx.x % C, t = threadIdx.x / C;
  const int col = blockIdx.x * C + c;
  u64 x[kEpt];
  if (FWD) {
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = a[(long long)lidx<LOG_M, HI, 4>(t, e) * M2 + col];
    fwd_round<LOG_M, HI, 4>(x, t, 0, gofs, log_n, tw, P.q, P.two_q);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) sm[lidx<LOG_M, HI, 4>(t, e) * C + c] = x[e];
    __syncthreads();
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = sm[lidx<LOG_M, 0, NLO>(t, e) * C + c];
    fwd_round<LOG_M, 0, NLO>(x, t, 0, gofs, log_n, tw, P.q, P.two_q);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) a[(long long)lidx<LOG_M, 0, NLO>(t, e) * M2 + col] = x[e];
  } else {
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = a[(long long)lidx<LOG_M, 0, NLO>(t, e) * M2 + col];
    inv_round<LOG_M, 0, NLO, false>(x, t, 0, gofs, log_n, tw, P);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) sm[lidx<LOG_M, 0, NLO>(t, e) * C + c] = x[e];
    __syncthreads();
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = sm[lidx<LOG_M, HI, 4>(t, e) * C + c];
    inv_round<LOG_M, HI, 4, true>(x, t, 0, gofs, log_n, tw, P);
#pragma unroll
    for (int e = 0; e < kEpt; ++e)
      a[(long long)lidx<LOG_M, HI, 4>(t, e) * M2 + col] = csub(x[e], P.q);
  }
}

// ---------------------------------------------------------------------------
// Row pass: sub-transforms of M = 2^LOG_M contiguous words.
// ---------------------------------------------------------------------------
template <int LOG_M>
__device__ __forceinline__ int padx(int r, int i) {
  constexpr int M = 1 << LOG_M;
  return r * (M + M / 16) + i + (i >> 4);
}

template <int LOG_M, bool FWD>
__global__ void __launch_bounds__(kThreads) ntt_rows(LimbMap m, NttTables T) {
  constexpr int M = 1 << LOG_M, LOG_T = LOG_M - 4, TT = 1 << LOG_T, R = kThreads / TT;
  constexpr int HI = LOG_M - 4, NLO = LOG_M - 4;
  __shared__ u64 sm[R * (M + M / 16)];
  u64 *a;
  int prime;
  limb_of(m, blockIdx.y, a, prime);
  if (prime < 0) return;
  const PrimeDev P = T.primes[prime];
  const int log_n = T.log_n, N = 1 << log_n;
  const ulonglong2 *tw = (FWD ? T.fwd : T.inv) + (long long)prime * N;
  const int t = threadIdx.x % TT, rr = threadIdx.x / TT;
  u64 *tile = a + (long long)blockIdx.x * kTile;
  const long long row = (long long)blockIdx.x * R + rr;
  u64 x[kEpt];
  if (FWD) {
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = tile[rr * M + lidx<LOG_M, HI, 4>(t, e)];
    fwd_round<LOG_M, HI, 4>(x, t, row, 0, log_n, tw, P.q, P.two_q);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) sm[padx<LOG_M>(rr, lidx<LOG_M, HI, 4>(t, e))] = x[e];
    __syncwarp();
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = sm[padx<LOG_M>(rr, lidx<LOG_M, 0, NLO>(t, e))];
    fwd_round<LOG_M, 0, NLO>(x, t, row, 0, log_n, tw, P.q, P.two_q);
#pragma unroll
    for (int e = 0; e < kEpt; ++e)
      sm[padx<LOG_M>(rr, lidx<LOG_M, 0, NLO>(t, e))] = reduce4(x[e], P.q, P.two_q);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kEpt; ++i) {
      const int lin = threadIdx.x + i * kThreads;
      tile[lin] = sm[padx<LOG_M>(lin >> LOG_M, lin & (M - 1))];
    }
  } else {
#pragma unroll
    for (int i = 0; i < kEpt; ++i) {
      const int lin = threadIdx.x + i * kThreads;
      sm[padx<LOG_M>(lin >> LOG_M, lin & (M - 1))] = tile[lin];
    }
    __syncthreads();
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = sm[padx<LOG_M>(rr, lidx<LOG_M, 0, NLO>(t, e))];
    inv_round<LOG_M, 0, NLO, false>(x, t, row, 0, log_n, tw, P);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) sm[padx<LOG_M>(rr, lidx<LOG_M, 0, NLO>(t, e))] = x[e];
    __syncwarp();
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = sm[padx<LOG_M>(rr, lidx<LOG_M, HI, 4>(t, e))];
    inv_round<LOG_M, HI, 4, false>(x, t, row, 0, log_n, tw, P);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) tile[rr * M + lidx<LOG_M, HI, 4>(t, e)] = x[e];
  }
}

template <int LOG_M, bool FWD>
cudaError_t launch_cols(const LimbMap &m, int n_limbs, const NttTables &T, cudaStream_t s) {
  constexpr int TT = 1 << (LOG_M - 4), C = kThreads / TT;
  const int M2 = (1 << T.log_n) >> LOG_M;
  dim3 grid(M2 / C, n_limbs);
  ntt_cols<LOG_M, FWD><<<grid, kThreads, 0, s>>>(m, T);
  return cudaGetLastError();
}
template <int LOG_M, bool FWD>
cudaError_t launch_rows(const LimbMap &m, int n_limbs, const NttTables &T, cudaStream_t s) {
  dim3 grid((1 << T.log_n) / kTile, n_limbs);
  ntt_rows<LOG_M, FWD><<<grid, kThreads, 0, s>>>(m, T);
  return cudaGetLastError();
}

template <bool FWD>
cudaError_t launch_pass(bool cols, int log_m, const LimbMap &m, int n, const NttTables &T,
                        cudaStream_t s) {
  switch (log_m) {
    case 6: return cols ? launch_cols<6, FWD>(m, n, T, s) : launch_rows<6, FWD>(m, n, T, s);
    case 7: return cols ? launch_cols<7, FWD>(m, n, T, s) : launch_rows<7, FWD>(m, n, T, s);
    case 8: return cols ? launch_cols<8, FWD>(m, n, T, s) : launch_rows<8, FWD>(m, n, T, s);
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

cudaError_t ntt_inverse(const LimbMap &m, int n_limbs, const NttTables &T, cudaStream_t s) {
  if (!ntt_supported_log_n(T.log_n) || n_limbs < 0 || n_limbs > 65535) return cudaErrorInvalidValue;
  if (n_limbs == 0) return cudaSuccess;
  const int s1 = T.log_n / 2, s2 = T.log_n - s1;
  cudaError_t e = launch_pass<false>(false, s2, m, n_limbs, T, s);
  if (e != cudaSuccess) return e;
  return launch_pass<false>(true, s1, m, n_limbs, T, s);
}

}  // namespace ksb
