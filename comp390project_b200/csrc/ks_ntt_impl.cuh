// ks_ntt_impl.cuh -- the device building blocks of the two-pass NTT, shared
// by the plain batched transform (ks_ntt.cu) and the fused key-switch
// kernels (ks_fused.cu).
//
// The length-N transform is split as N = M1 * M2 (M1 = 2^(logN/2)).  The
// column pass runs the stages whose butterflies span the high index bits
// (each column of M1 elements at stride M2 is an independent sub-transform);
// the row pass runs the remaining stages inside contiguous rows of M2
// elements.  Every thread keeps 16 elements in registers and runs four
// butterfly stages on them (a radix-16 step); one shared-memory exchange
// re-partitions the sub-transform for the next four stages.
//
// Column-pass tiles are 4096/M1 adjacent columns wide with the lane index
// running along the contiguous column direction, so every global access is
// a full row segment (128 bytes for M1 = 256).  Row-pass tiles are 4096
// contiguous words.
#pragma once
#include "ks_arith.cuh"
#include "ks_ntt.cuh"

namespace ksb {
namespace ntt {

constexpr int kThreads = 256;
constexpr int kEpt = 16;                // elements per thread
constexpr int kTile = kThreads * kEpt;  // 4096 words per CTA

// Register e = (g << NB) | v holds the local index
//   ((u >> LO) << (LO + NB)) | (v << LO) | (u & ((1 << LO) - 1)),  u = (g << LOG_T) | t.
// The fields of t and of e occupy disjoint bits, so the index is the sum
// lidx_t(t) + lidx_e(e): the e part is a compile-time constant that folds
// into immediate offsets, and only the t part is computed at run time.  Every
// round has LO <= LOG_T.
template <int LOG_M, int LO, int NB>
__device__ __forceinline__ int lidx_t(int t) {
  static_assert(LO <= LOG_M - 4, "round below the thread bits");
  return ((t >> LO) << (LO + NB)) + (t & ((1 << LO) - 1));
}
template <int LOG_M, int LO, int NB>
__host__ __device__ constexpr int lidx_e(int e) {
  return (((e >> NB) << (LOG_M - 4 - LO)) << (LO + NB)) + ((e & ((1 << NB) - 1)) << LO);
}
template <int LOG_M, int LO, int NB>
__device__ __forceinline__ int lidx(int t, int e) {
  return lidx_t<LOG_M, LO, NB>(t) + lidx_e<LOG_M, LO, NB>(e);
}

// Twiddle addressing.  The pair whose lower element has local index
// i = lidx(t, e) at local bit b of a pass over rows of 2^LOG_M words uses
// the twiddle at index (1 << (logN-1-b-gofs)) + (((prefix << LOG_M) + i) >> (b+1)).
// Because the t and e fields are disjoint, i >> (b + 1) =
// (lidx_t >> (b + 1)) + (lidx_e >> (b + 1)): the first part (with the prefix)
// gives one per-thread base per stage, the second a compile-time offset, so a
// butterfly's twiddle is one load at a constant offset from the stage base.
// The FP64 getters below keep that split (their tables may permute the
// within-row index by row_tw_pos, a bit permutation, which distributes over
// the two disjoint parts).

// Forward stages on local bits [LO, LO+NB), high bit first; integer tables
// {w, w_shoup} in natural order.
template <int LOG_M, int LO, int NB, bool LAZY>
__device__ __forceinline__ void fwd_round(u64 (&x)[kEpt], int t, long long prefix, int gofs,
                                          int log_n, const ulonglong2 *__restrict__ tw, u64 q,
                                          u64 two_q) {
  const int lt = lidx_t<LOG_M, LO, NB>(t);
#pragma unroll
  for (int k = NB - 1; k >= 0; --k) {
    const int b = LO + k;
    const int twk =  // stage base (an index below N)
        (1 << (log_n - 1 - b - gofs)) + (int)(prefix << (LOG_M - b - 1)) + (lt >> (b + 1));
#pragma unroll
    for (int e = 0; e < kEpt; ++e) {
      if (e & (1 << k)) continue;
      const ulonglong2 w = __ldg(&tw[twk + (lidx_e<LOG_M, LO, NB>(e) >> (b + 1))]);
      if (LAZY) ct_bfly_lazy(x[e], x[e | (1 << k)], w.x, w.y, q, two_q);
      else ct_bfly(x[e], x[e | (1 << k)], w.x, w.y, q, two_q);
    }
  }
}

// Inverse stages on local bits [LO, LO+NB), low bit first.  If LAST, the top
// stage of this round is the final stage of the transform, with the output
// scale folded in (scale = N^-1 and psi^-brev(1) N^-1, Shoup pairs).
template <int LOG_M, int LO, int NB, bool LAZY, bool LAST>
__device__ __forceinline__ void inv_round(u64 (&x)[kEpt], int t, long long prefix, int gofs,
                                          int log_n, const ulonglong2 *__restrict__ tw,
                                          const PrimeDev &P, ulonglong2 s0, ulonglong2 s1) {
  const int lt = lidx_t<LOG_M, LO, NB>(t);
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const int b = LO + k;
    const int gb = b + gofs;
    const int twk =  // stage base (an index below N)
        (1 << (log_n - 1 - gb)) + (int)(prefix << (LOG_M - b - 1)) + (lt >> (b + 1));
    const u64 K = P.q << gb;  // >= bound of the operands entering this stage (lazy path)
#pragma unroll
    for (int e = 0; e < kEpt; ++e) {
      if (e & (1 << k)) continue;
      u64 &X = x[e], &Y = x[e | (1 << k)];
      if (LAST && k == NB - 1) {
        const u64 s = LAZY ? X + Y : X + Y;  // < 2^64 on both paths
        const u64 d = LAZY ? X + K - Y : X - Y + P.two_q;
        X = mul_shoup_lazy(s, s0.x, s0.y, P.q);
        Y = mul_shoup_lazy(d, s1.x, s1.y, P.q);
      } else {
        const ulonglong2 w = __ldg(&tw[twk + (lidx_e<LOG_M, LO, NB>(e) >> (b + 1))]);
        if (LAZY) gs_bfly_lazy(X, Y, w.x, w.y, P.q, K);
        else gs_bfly(X, Y, w.x, w.y, P.q, P.two_q);
      }
    }
  }
}

template <int LOG_M>
__device__ __forceinline__ int padx(int r, int i) {
  constexpr int M = 1 << LOG_M;
  return r * (M + M / 16) + i + (i >> 4);
}

template <int LOG_M>
struct ColGeom {
  static constexpr int M = 1 << LOG_M, LOG_T = LOG_M - 4, TT = 1 << LOG_T, C = kThreads / TT;
  static constexpr int HI = LOG_M - 4, NLO = LOG_M - 4;
  static constexpr int SMEM = M * C;  // words
};
// 42-bit packing of one thread's column values (the kEpt = 16 words at rows
// lidx<LOG_M, HI, 4>(t, e) of its column, each below 2^42): five triplets in
// two words each (a | b << 42, b >> 22 | c << 20) and the last value alone,
// 11 words; word w of thread t of a column sits at row t * 11 + w of the
// packed limb (11 N / 16 words).  The input all-gather of input broadcast
// moves limbs in this form (kPackWords, ks_ntt.cuh).
__device__ __forceinline__ void pack42(const u64 (&v)[16], u64 (&w)[kPackWords]) {
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const u64 a = v[3 * k], b = v[3 * k + 1], c = v[3 * k + 2];
    w[2 * k] = a | (b << 42);
    w[2 * k + 1] = (b >> 22) | (c << 20);
  }
  w[10] = v[15];
}
__device__ __forceinline__ void unpack42(const u64 (&w)[kPackWords], u64 (&v)[16]) {
  constexpr u64 m42 = (1ull << 42) - 1, m20 = (1ull << 20) - 1;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    v[3 * k] = w[2 * k] & m42;
    v[3 * k + 1] = (w[2 * k] >> 42) | ((w[2 * k + 1] & m20) << 22);
    v[3 * k + 2] = w[2 * k + 1] >> 20;
  }
  v[15] = w[10];
}

template <int LOG_M>
struct RowGeom {
  static constexpr int M = 1 << LOG_M, LOG_T = LOG_M - 4, TT = 1 << LOG_T, R = kThreads / TT;
  static constexpr int HI = LOG_M - 4, NLO = LOG_M - 4;
  static constexpr int SMEM = R * (M + M / 16);
};

// ---------------------------------------------------------------------------
// Forward column pass.  load(r, col) gives the input of row r (< q for the
// lazy path, < 4q otherwise); store(r, col, v) receives the output (< 17q lazy,
// < 4q Harvey).  Rows r index the column sub-transform, col < M2.
// ---------------------------------------------------------------------------
// fill(x) sets x[e] to the input of column row lidx<LOG_M, HI, 4>(t, e).
template <int LOG_M, class Load>
__device__ __forceinline__ void fill_cols(u64 (&x)[kEpt], int t, int col, Load &&load) {
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = load(lidx<LOG_M, ColGeom<LOG_M>::HI, 4>(t, e), col);
}

template <int LOG_M, bool LAZY, class Fill, class Store>
__device__ __forceinline__ void fwd_cols(u64 *sm, int col, int t, int c, int log_n,
                                         const ulonglong2 *tw, const PrimeDev &P, Fill &&fill,
                                         Store &&store) {
  using G = ColGeom<LOG_M>;
  const int gofs = log_n - LOG_M;
  u64 x[kEpt];
  fill(x);
  fwd_round<LOG_M, G::HI, 4, LAZY>(x, t, 0, gofs, log_n, tw, P.q, P.two_q);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) sm[lidx<LOG_M, G::HI, 4>(t, e) * G::C + c] = x[e];
  __syncthreads();
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = sm[lidx<LOG_M, 0, G::NLO>(t, e) * G::C + c];
  fwd_round<LOG_M, 0, G::NLO, LAZY>(x, t, 0, gofs, log_n, tw, P.q, P.two_q);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) store(lidx<LOG_M, 0, G::NLO>(t, e), col, x[e]);
}

// Inverse column pass (the second pass of an inverse transform); outputs are
// canonical and multiplied by the scale of the last stage.
template <int LOG_M, bool LAZY, class Load, class Store>
__device__ __forceinline__ void inv_cols(u64 *sm, int col, int t, int c, int log_n,
                                         const ulonglong2 *tw, const PrimeDev &P, ulonglong2 s0,
                                         ulonglong2 s1, Load &&load, Store &&store) {
  using G = ColGeom<LOG_M>;
  const int gofs = log_n - LOG_M;
  u64 x[kEpt];
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = load(lidx<LOG_M, 0, G::NLO>(t, e), col);
  inv_round<LOG_M, 0, G::NLO, LAZY, false>(x, t, 0, gofs, log_n, tw, P, s0, s1);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) sm[lidx<LOG_M, 0, G::NLO>(t, e) * G::C + c] = x[e];
  __syncthreads();
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = sm[lidx<LOG_M, G::HI, 4>(t, e) * G::C + c];
  inv_round<LOG_M, G::HI, 4, LAZY, true>(x, t, 0, gofs, log_n, tw, P, s0, s1);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) store(lidx<LOG_M, G::HI, 4>(t, e), col, csub(x[e], P.q));
}

// ---------------------------------------------------------------------------
// Forward row pass over one 4096-word tile (R rows of M).  The thread's
// 16 outputs (canonical) are handed to finish(rr, i, v) for local row rr,
// index i in the row; the tile is then written by the caller from smem.
// ---------------------------------------------------------------------------
// The 16 inputs of thread t of local row rr of a row tile (pattern HI), for
// callers that load them ahead of the transform.
template <int LOG_M>
__device__ __forceinline__ void load_rows_tile(u64 (&x)[kEpt], const u64 *tile, int t, int rr) {
#pragma unroll
  for (int e = 0; e < kEpt; ++e)
    x[e] = tile[rr * RowGeom<LOG_M>::M + lidx<LOG_M, RowGeom<LOG_M>::HI, 4>(t, e)];
}

// fwd_rows_regs on inputs already in x (load_rows_tile).
template <int LOG_M, bool LAZY>
__device__ __forceinline__ void fwd_rows_inregs(u64 (&x)[kEpt], u64 *sm, int t, int rr,
                                                long long row, int log_n, const ulonglong2 *tw,
                                                const PrimeDev &P) {
  using G = RowGeom<LOG_M>;
  fwd_round<LOG_M, G::HI, 4, LAZY>(x, t, row, 0, log_n, tw, P.q, P.two_q);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) sm[padx<LOG_M>(rr, lidx<LOG_M, G::HI, 4>(t, e))] = x[e];
  __syncwarp();
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = sm[padx<LOG_M>(rr, lidx<LOG_M, 0, G::NLO>(t, e))];
  fwd_round<LOG_M, 0, G::NLO, LAZY>(x, t, row, 0, log_n, tw, P.q, P.two_q);
#pragma unroll
  for (int e = 0; e < kEpt; ++e)
    x[e] = LAZY ? reduce_full(x[e], P.q, P.mu) : reduce4(x[e], P.q, P.two_q);
  __syncwarp();
}

template <int LOG_M, bool LAZY>
__device__ __forceinline__ void fwd_rows_regs(u64 (&x)[kEpt], u64 *sm, const u64 *tile, int t,
                                              int rr, long long row, int log_n,
                                              const ulonglong2 *tw, const PrimeDev &P) {
  load_rows_tile<LOG_M>(x, tile, t, rr);
  fwd_rows_inregs<LOG_M, LAZY>(x, sm, t, rr, row, log_n, tw, P);
}


// Inverse row pass (the first pass of an inverse transform) over one tile
// already staged in smem (padx layout); outputs in registers, pattern HI.
template <int LOG_M, bool LAZY>
__device__ __forceinline__ void inv_rows_regs(u64 (&x)[kEpt], u64 *sm, int t, int rr,
                                              long long row, int log_n, const ulonglong2 *tw,
                                              const PrimeDev &P) {
  using G = RowGeom<LOG_M>;
  const ulonglong2 none = make_ulonglong2(0, 0);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = sm[padx<LOG_M>(rr, lidx<LOG_M, 0, G::NLO>(t, e))];
  inv_round<LOG_M, 0, G::NLO, LAZY, false>(x, t, row, 0, log_n, tw, P, none, none);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) sm[padx<LOG_M>(rr, lidx<LOG_M, 0, G::NLO>(t, e))] = x[e];
  __syncwarp();
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = sm[padx<LOG_M>(rr, lidx<LOG_M, G::HI, 4>(t, e))];
  inv_round<LOG_M, G::HI, 4, LAZY, false>(x, t, row, 0, log_n, tw, P, none, none);
}

// ===========================================================================
// FP64 variants (primes below kFpBound).  Values travel between the passes as
// the bits of signed integer-valued doubles; the pass inputs and the final
// outputs are canonical uint64.  A twiddle getter (stage / get, see the
// twiddle addressing note above) returns {w, wq} for the pair at local bit b:
// w = psi^(+-brev) and wq the quotient factor,
// either fl(w/q) from the column tables (2^(logN/2) pairs per prime) or
// w * fl(1/q) formed next to its use from the row tables (w only, to keep the
// staged row blocks small); both keep the estimate error below
// |y| 2^-52 <= 2^-4 for |y| <= 2^48 (every product input of these passes
// stays below 2^48 for q < kFpBound).
// ===========================================================================
__device__ __forceinline__ double as_fp(u64 b) { return __longlong_as_double((long long)b); }
__device__ __forceinline__ u64 fp_bits(double d) { return (u64)__double_as_longlong(d); }

// Column-pass getter: the prime's {w, fl(w/q)} column table (index
// 2^(LOG_M-1-b) + (i >> (b+1)) < 2^LOG_M; every column of a CTA shares them;
// the prefix is 0).  stage(b, prefix, ts) is the per-thread base of local bit
// b (ts = lidx_t >> (b + 1)), get(base, b, es) the twiddle at the constant
// offset es = lidx_e >> (b + 1).
template <int LOG_M>
struct TwCols {
  const double2 *tw;
  __device__ __forceinline__ int stage(int b, long long, int ts) const {
    return (1 << (LOG_M - 1 - b)) + ts;
  }
  __device__ __forceinline__ double2 get(int base, int, int es) const {
    return __ldg(tw + base + es);
  }
};

// Shared-memory getter for a row pass over rows [row0, row0 + R): the block
// of local bit b holds R * 2^u twiddles, u = LOG_M - 1 - b, at offset
// R (2^u - 1); the within-row index is permuted by row_tw_pos.
template <int LOG_M, int R>
struct TwRowsSmem {
  const double *sm;
  long long row0;
  double qinv;
  __device__ __forceinline__ int stage(int b, long long prefix, int ts) const {
    const int u = LOG_M - 1 - b;
    return R * ((1 << u) - 1) + (int)((prefix - row0) << u) + row_tw_pos(LOG_M, b, ts);
  }
  __device__ __forceinline__ double2 get(int base, int b, int es) const {
    const double w = sm[base + row_tw_pos(LOG_M, b, es)];
    return make_double2(w, __dmul_rn(w, qinv));
  }
};

// Global-table getter for a row pass (rows of 2^LOG_M words, permuted
// row-pass region of the FP64 table).
template <int LOG_M>
struct TwRowsGlobal {
  const double *tw;
  int log_n;
  double qinv;
  __device__ __forceinline__ int stage(int b, long long prefix, int ts) const {
    const int u = LOG_M - 1 - b;  // an index below N
    return (1 << (log_n - 1 - b)) + (int)(prefix << u) + row_tw_pos(LOG_M, b, ts);
  }
  __device__ __forceinline__ double2 get(int base, int b, int es) const {
    const double w = __ldg(tw + base + row_tw_pos(LOG_M, b, es));
    return make_double2(w, __dmul_rn(w, qinv));
  }
};

// Issues cp.async copies (by the NTHR threads of the CTA) of the row-pass
// twiddle block (R (M - 1) doubles) of rows [row0, row0 + R) into sm; the caller waits with cp_async_wait_all.
// Block u (u = 0..LOG_M-1) is tw[2^(logN-LOG_M+u) + row0 2^u, +R 2^u); with R
// even every block starts and ends on a 16-byte boundary.
template <int LOG_M, int R, int NTHR = kThreads>
__device__ __forceinline__ void stage_row_twiddles(double *sm, const double *tw, int log_n,
                                                   long long row0) {
  constexpr int M = 1 << LOG_M, TOTAL = R * (M - 1);
  static_assert(R % 2 == 0, "row blocks must be 16-byte multiples");
  for (int ch = threadIdx.x; ch < TOTAL / 2; ch += NTHR) {
    const int e = 2 * ch;
    const int u = 31 - __clz(e / R + 1);
    const int o = e - R * ((1 << u) - 1);
    const double *g = tw + (1ll << (log_n - LOG_M + u)) + (row0 << u) + o;
    const unsigned s = (unsigned)__cvta_generic_to_shared(sm + e);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(g) : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Bound: operands < B on entry -> < B + 4 * 0.57q on exit (additive growth).
template <int LOG_M, int LO, int NB, class Tw>
__device__ __forceinline__ void fwd_round_fp(double (&x)[kEpt], int t, long long prefix,
                                             const Tw &tw, double q, double qinv) {
  const int lt = lidx_t<LOG_M, LO, NB>(t);
#pragma unroll
  for (int k = NB - 1; k >= 0; --k) {
    const int b = LO + k;
    const int base = tw.stage(b, prefix, lt >> (b + 1));
#pragma unroll
    for (int e = 0; e < kEpt; ++e) {
      if (e & (1 << k)) continue;
      const double2 w = tw.get(base, b, lidx_e<LOG_M, LO, NB>(e) >> (b + 1));
      fp_ct_bfly(x[e], x[e | (1 << k)], w.x, w.y, q);
    }
  }
}

// Every operand is reduced to |x| <= q/2 (+1) on entry, so within the round
// the sums stay below 2^NB * 0.57q and every product input below 2^48.
template <int LOG_M, int LO, int NB, bool LAST, class Tw>
__device__ __forceinline__ void inv_round_fp(double (&x)[kEpt], int t, long long prefix,
                                             const Tw &tw, const PrimeDev &P, double2 s0,
                                             double2 s1) {
  const int lt = lidx_t<LOG_M, LO, NB>(t);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = fp_reduce_sym(x[e], P.qd, P.qinv);
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const int b = LO + k;
    const int base = tw.stage(b, prefix, lt >> (b + 1));
#pragma unroll
    for (int e = 0; e < kEpt; ++e) {
      if (e & (1 << k)) continue;
      double &X = x[e], &Y = x[e | (1 << k)];
      if (LAST && k == NB - 1) {
        const double s = __dadd_rn(X, Y), d = __dsub_rn(X, Y);
        X = fp_mulmod(s, s0.x, s0.y, P.qd);
        Y = fp_mulmod(d, s1.x, s1.y, P.qd);
      } else {
        const double2 w = tw.get(base, b, lidx_e<LOG_M, LO, NB>(e) >> (b + 1));
        fp_gs_bfly(X, Y, w.x, w.y, P.qd);
      }
    }
  }
}

// filld(x) fills signed integer-valued doubles (|x| < 8q).
template <int LOG_M, class FillD, class Store>
__device__ __forceinline__ void fwd_cols_fpd(u64 *sm, int col, int t, int c, int log_n,
                                             const double2 *tw, const PrimeDev &P, FillD &&filld,
                                             Store &&store) {
  using G = ColGeom<LOG_M>;
  const TwCols<LOG_M> twg{tw};
  double x[kEpt];
  filld(x);
  fwd_round_fp<LOG_M, G::HI, 4>(x, t, 0, twg, P.qd, P.qinv);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) sm[lidx<LOG_M, G::HI, 4>(t, e) * G::C + c] = fp_bits(x[e]);
  __syncthreads();
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = as_fp(sm[lidx<LOG_M, 0, G::NLO>(t, e) * G::C + c]);
  fwd_round_fp<LOG_M, 0, G::NLO>(x, t, 0, twg, P.qd, P.qinv);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) store(lidx<LOG_M, 0, G::NLO>(t, e), col, fp_bits(x[e]));
}

template <int LOG_M, class Fill, class Store>
__device__ __forceinline__ void fwd_cols_fp(u64 *sm, int col, int t, int c, int log_n,
                                            const double2 *tw, const PrimeDev &P, Fill &&fill,
                                            Store &&store) {
  auto filld = [&](double (&x)[kEpt]) {
    u64 xin[kEpt];
    fill(xin);
#pragma unroll
    for (int e = 0; e < kEpt; ++e) x[e] = u64_to_fp(xin[e]);
  };
  fwd_cols_fpd<LOG_M>(sm, col, t, c, log_n, tw, P, filld, store);
}

// Inverse column pass (second pass); load() gives the bits of the first
// pass result, store() receives canonical uint64 times the last-stage scale
// (CANON_FP: the bits of that canonical value as a double instead).
template <int LOG_M, bool CANON_FP = false, class Load, class Store>
__device__ __forceinline__ void inv_cols_fp(u64 *sm, int col, int t, int c, int log_n,
                                            const double2 *tw, const PrimeDev &P, double2 s0,
                                            double2 s1, Load &&load, Store &&store) {
  using G = ColGeom<LOG_M>;
  const TwCols<LOG_M> twg{tw};
  double x[kEpt];
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = as_fp(load(lidx<LOG_M, 0, G::NLO>(t, e), col));
  inv_round_fp<LOG_M, 0, G::NLO, false>(x, t, 0, twg, P, s0, s1);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) sm[lidx<LOG_M, 0, G::NLO>(t, e) * G::C + c] = fp_bits(x[e]);
  __syncthreads();
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = as_fp(sm[lidx<LOG_M, G::HI, 4>(t, e) * G::C + c]);
  inv_round_fp<LOG_M, G::HI, 4, true>(x, t, 0, twg, P, s0, s1);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) {
    if (CANON_FP)  // the last stage's fp_mulmod leaves |x| < 0.57q: one add makes it canonical
      store(lidx<LOG_M, G::HI, 4>(t, e), col, fp_bits(x[e] < 0.0 ? __dadd_rn(x[e], P.qd) : x[e]));
    else
      store(lidx<LOG_M, G::HI, 4>(t, e), col, fp_to_canon(x[e], P.qd, P.qinv));
  }
}

// inv_cols_fp with the canonical outputs (times the last-stage scale) left
// in registers: out[e] is row lidx<LOG_M, HI, 4>(t, e) of the column.
template <int LOG_M, class Load>
__device__ __forceinline__ void inv_cols_fp_regs(u64 *sm, int col, int t, int c, int log_n,
                                                 const double2 *tw, const PrimeDev &P, double2 s0,
                                                 double2 s1, Load &&load, u64 (&out)[kEpt]) {
  using G = ColGeom<LOG_M>;
  const TwCols<LOG_M> twg{tw};
  double x[kEpt];
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = as_fp(load(lidx<LOG_M, 0, G::NLO>(t, e), col));
  inv_round_fp<LOG_M, 0, G::NLO, false>(x, t, 0, twg, P, s0, s1);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) sm[lidx<LOG_M, 0, G::NLO>(t, e) * G::C + c] = fp_bits(x[e]);
  __syncthreads();
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = as_fp(sm[lidx<LOG_M, G::HI, 4>(t, e) * G::C + c]);
  inv_round_fp<LOG_M, G::HI, 4, true>(x, t, 0, twg, P, s0, s1);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) out[e] = fp_to_canon(x[e], P.qd, P.qinv);
}

// Forward row pass; the tile holds first-pass bits; canonical outputs in xo
// (CANON), else the bits of the unreduced doubles (|x| < 12q < 2^47).
// tw: twiddle getter (TwRowsSmem over a staged block, or TwRowsGlobal).
// fwd_rows_regs_fp_tw on inputs already in xo (load_rows_tile).
template <int LOG_M, bool CANON, class Tw>
__device__ __forceinline__ void fwd_rows_fp_inregs(u64 (&xo)[kEpt], u64 *sm, const Tw &tw, int t,
                                                   int rr, long long row, const PrimeDev &P) {
  using G = RowGeom<LOG_M>;
  double x[kEpt];
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = as_fp(xo[e]);
  fwd_round_fp<LOG_M, G::HI, 4>(x, t, row, tw, P.qd, P.qinv);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) sm[padx<LOG_M>(rr, lidx<LOG_M, G::HI, 4>(t, e))] = fp_bits(x[e]);
  __syncwarp();
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = as_fp(sm[padx<LOG_M>(rr, lidx<LOG_M, 0, G::NLO>(t, e))]);
  fwd_round_fp<LOG_M, 0, G::NLO>(x, t, row, tw, P.qd, P.qinv);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) xo[e] = CANON ? fp_to_canon(x[e], P.qd, P.qinv) : fp_bits(x[e]);
  __syncwarp();
}

template <int LOG_M, bool CANON, class Tw>
__device__ __forceinline__ void fwd_rows_regs_fp_tw(u64 (&xo)[kEpt], u64 *sm, const Tw &tw,
                                                    const u64 *tile, int t, int rr, long long row,
                                                    const PrimeDev &P) {
  load_rows_tile<LOG_M>(xo, tile, t, rr);
  fwd_rows_fp_inregs<LOG_M, CANON>(xo, sm, tw, t, rr, row, P);
}

// smtw: this CTA's twiddle block, staged by stage_row_twiddles (the caller
// waits for it and synchronises before calling).
template <int LOG_M, bool CANON = true>
__device__ __forceinline__ void fwd_rows_regs_fp(u64 (&xo)[kEpt], u64 *sm, const double *smtw,
                                                 const u64 *tile, int t, int rr, long long row,
                                                 long long row0, const PrimeDev &P) {
  const TwRowsSmem<LOG_M, RowGeom<LOG_M>::R> tw{smtw, row0, P.qinv};
  fwd_rows_regs_fp_tw<LOG_M, CANON>(xo, sm, tw, tile, t, rr, row, P);
}

// Inverse row pass (first pass) over a tile staged in smem as canonical
// uint64; outputs (bits of doubles, |x| <= q/2 + 1) in xo, pattern HI.
template <int LOG_M, class Tw>
__device__ __forceinline__ void inv_rows_regs_fp_tw(u64 (&xo)[kEpt], u64 *sm, const Tw &tw,
                                                    int t, int rr, long long row,
                                                    const PrimeDev &P) {
  using G = RowGeom<LOG_M>;
  const double2 none = make_double2(0, 0);
  double x[kEpt];
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = u64_to_fp(sm[padx<LOG_M>(rr, lidx<LOG_M, 0, G::NLO>(t, e))]);
  inv_round_fp<LOG_M, 0, G::NLO, false>(x, t, row, tw, P, none, none);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) sm[padx<LOG_M>(rr, lidx<LOG_M, 0, G::NLO>(t, e))] = fp_bits(x[e]);
  __syncwarp();
#pragma unroll
  for (int e = 0; e < kEpt; ++e) x[e] = as_fp(sm[padx<LOG_M>(rr, lidx<LOG_M, G::HI, 4>(t, e))]);
  inv_round_fp<LOG_M, G::HI, 4, false>(x, t, row, tw, P, none, none);
#pragma unroll
  for (int e = 0; e < kEpt; ++e) xo[e] = fp_bits(fp_reduce_sym(x[e], P.qd, P.qinv));
}
template <int LOG_M>
__device__ __forceinline__ void inv_rows_regs_fp(u64 (&xo)[kEpt], u64 *sm, const double *smtw,
                                                 int t, int rr, long long row, long long row0,
                                                 const PrimeDev &P) {
  const TwRowsSmem<LOG_M, RowGeom<LOG_M>::R> tw{smtw, row0, P.qinv};
  inv_rows_regs_fp_tw<LOG_M>(xo, sm, tw, t, rr, row, P);
}

// Shared memory of a row-pass CTA: the exchange buffer then (FP64 path) the
// twiddle block.
template <int LOG_M>
__host__ __device__ constexpr size_t row_smem_bytes() {
  return (size_t)RowGeom<LOG_M>::SMEM * 8 + (size_t)RowGeom<LOG_M>::R * ((1 << LOG_M) - 1) * 8;
}

}  // namespace ntt
}  // namespace ksb
