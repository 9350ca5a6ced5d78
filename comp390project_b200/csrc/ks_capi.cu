// ks_capi.cu -- context set-up, key management, the hybrid key-switch
// pipeline and the extern "C" entry points declared in include/ks_capi.h.
//
// Pipeline of one key switch on rank g of G (input-broadcast mode; G = 1 is
// the single-GPU path), following the stage order of the reference's
// keyswitching_output_aggregation (output_aggregation.cu:197-294) and
// Phantom's keyswitch_inplace (input_broadcast.cu:172):
//   1. automorphism of c0, c1 (rotation only)            -> g0, g1
//   2. INTT of the input limbs, all-gather over ranks     -> coefficient form
//   3. ModUp base extension of every digit to the owned QlP limbs, NTT
//   4. inner product with the evaluation-key shard        -> cx (owned limbs)
//   5. INTT of the owned P limbs of cx, all-gather        -> P part, coefficient form
//   6. conversion P -> owned Q limbs, NTT
//   7. (cx - conv) * P^-1, add to the ciphertext          -> ct (in place)
#include <cuda_runtime.h>
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "../../include/ks_capi.h"
#include "ks_context.hpp"
#include "ks_fused.cuh"
#include "ks_hostmath.hpp"

using namespace ksb;

struct ks_ctx {
  Ctx c;
};

struct ks_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int device = 0;
};

namespace {

std::mutex g_err_mu;
std::string g_err;

void set_global_err(const std::string &s) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  g_err = s;
}

struct KsError {
  int code;
  std::string msg;
};

#define KS_CUDA(expr)                                                                     \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    if (_e != cudaSuccess)                                                                \
      throw KsError{KS_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)};     \
  } while (0)
#define KS_NCCL(expr)                                                                     \
  do {                                                                                    \
    ncclResult_t _r = (expr);                                                             \
    if (_r != ncclSuccess)                                                                \
      throw KsError{KS_ERR_NCCL, std::string(#expr) + ": " + ncclGetErrorString(_r)};     \
  } while (0)
#define KS_REQUIRE(cond, msg)                                                             \
  do {                                                                                    \
    if (!(cond)) throw KsError{KS_ERR_INVALID, msg};                                      \
  } while (0)

// A failed call during a graph capture ends (and discards) the capture, so
// the caller's stream is usable again.
inline void abort_capture(ks_ctx *ctx) {
  if (!ctx || !ctx->c.capturing) return;
  cudaGraph_t g = nullptr;
  cudaStreamEndCapture(ctx->c.capture_stream, &g);
  if (g) cudaGraphDestroy(g);
  cudaGetLastError();
  ctx->c.capturing = false;
}

template <class F>
int guarded(ks_ctx *ctx, F &&f) {
  try {
    f();
    return KS_OK;
  } catch (const KsError &e) {
    if (ctx) ctx->c.err = e.msg;
    set_global_err(e.msg);
    abort_capture(ctx);
    return e.code;
  } catch (const std::bad_alloc &) {
    if (ctx) ctx->c.err = "host allocation failed";
    set_global_err("host allocation failed");
    abort_capture(ctx);
    return KS_ERR_ALLOC;
  } catch (const std::exception &e) {
    if (ctx) ctx->c.err = e.what();
    set_global_err(e.what());
    abort_capture(ctx);
    return KS_ERR_INVALID;
  } catch (...) {
    if (ctx) ctx->c.err = "unknown exception";
    set_global_err("unknown exception");
    abort_capture(ctx);
    return KS_ERR_INVALID;
  }
}

template <class T>
T *dev_alloc(size_t n) {
  void *p = nullptr;
  if (n == 0) n = 1;
  cudaError_t e = cudaMalloc(&p, n * sizeof(T));
  if (e != cudaSuccess)
    throw KsError{KS_ERR_ALLOC, std::string("cudaMalloc ") + std::to_string(n * sizeof(T)) +
                                    " bytes: " + cudaGetErrorString(e)};
  return static_cast<T *>(p);
}

template <class T>
T *upload(const std::vector<T> &v) {
  T *d = dev_alloc<T>(v.size());
  if (!v.empty()) KS_CUDA(cudaMemcpy(d, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
  return d;
}

void up_ints(DevInts &t) { t.d = upload(t.h); }
void up_i64(DevI64 &t) { t.d = upload(t.h); }

// Temporary device buffer of a set-up call, freed on every exit path.
template <class T>
struct DevBuf {
  T *p = nullptr;
  explicit DevBuf(size_t n) : p(dev_alloc<T>(n)) {}
  DevBuf(const DevBuf &) = delete;
  DevBuf &operator=(const DevBuf &) = delete;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

inline bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

int n_local(int g, int G, int total) { return g < total ? (total - g - 1) / G + 1 : 0; }

// Merges two job lists with the `rare` jobs at evenly spaced positions, the
// first of them at the front (the rare jobs are the long-running ones).
template <class T>
std::vector<T> interleave_jobs(const std::vector<T> &common, const std::vector<T> &rare) {
  std::vector<T> out;
  const size_t n = common.size() + rare.size();
  out.reserve(n);
  size_t ic = 0, ir = 0;
  for (size_t k = 0; k < n; ++k) {
    // rare job ir belongs at position floor(ir * n / rare.size())
    if (ir < rare.size() && k >= ir * n / rare.size()) out.push_back(rare[ir++]);
    else if (ic < common.size()) out.push_back(common[ic++]);
    else out.push_back(rare[ir++]);
  }
  return out;
}

u64 mix64h(u64 z) {
  z ^= z >> 30;
  z *= 0xBF58476D1CE4E5B9ull;
  z ^= z >> 27;
  z *= 0x94D049BB133111EBull;
  z ^= z >> 31;
  return z;
}
// Per-(seed, domain) key of the counter hash prng(seed, dom, idx) =
// mix64(key + (idx + 1) * golden); the CPU oracle uses the same definition.
u64 prng_stream(u64 seed, u64 dom) { return mix64h(seed ^ mix64h(dom + 0x9E3779B97F4A7C15ull)); }
u64 prng_at(u64 seed, u64 dom, u64 idx) {
  return mix64h(prng_stream(seed, dom) + (idx + 1) * 0x9E3779B97F4A7C15ull);
}
enum : u64 { DOM_SECRET = 1, DOM_SECRET_SIGN = 2, DOM_KEY_A = 3, DOM_KEY_E = 4 };

// ---------------------------------------------------------------------------
// Context construction
// ---------------------------------------------------------------------------
void build_tables(Ctx &c) {
  const int N = c.N, K = c.K;
  std::vector<PrimeDev> pd(K);
  std::vector<ulonglong2> fwd((size_t)K * N), inv((size_t)K * N);
  std::vector<double> fwd_fp((size_t)K * N, 0.0), inv_fp((size_t)K * N, 0.0);
  const int NC = 1 << (c.log_n / 2);  // column-pass twiddle indices
  std::vector<double2> fwd_col((size_t)K * NC, make_double2(0, 0)), inv_col(fwd_col);
  std::vector<std::thread> th;
  auto work = [&](int k) {
    const u64 q = c.primes[k];
    const u64 psi = h_min_psi(q, (u64)N), psii = h_invmod(psi, q);
    std::vector<u64> pw(N), pwi(N);
    pw[0] = pwi[0] = 1;
    for (int i = 1; i < N; ++i) {
      pw[i] = h_mulmod(pw[i - 1], psi, q);
      pwi[i] = h_mulmod(pwi[i - 1], psii, q);
    }
    for (int i = 0; i < N; ++i) {
      const uint32_t r = h_brev((uint32_t)i, c.log_n);
      fwd[(size_t)k * N + i] = make_ulonglong2(pw[r], h_shoup(pw[r], q));
      inv[(size_t)k * N + i] = make_ulonglong2(pwi[r], h_shoup(pwi[r], q));
    }
    if (q < kFpBound) {
      // FP64 tables: w as a double, row-pass blocks permuted by row_tw_pos
      const int lm = c.log_n - c.log_n / 2;
      for (int i = 0; i < N; ++i) {
        size_t dst = (size_t)i;
        const int b = c.log_n - 1 - (31 - __builtin_clz((unsigned)std::max(i, 1)));
        if (i > 0 && b < lm) {  // row-pass local bit b: i = 2^(logN-1-b) + row 2^u + kk
          const int u = lm - 1 - b;
          const size_t off = (size_t)i - ((size_t)1 << (c.log_n - 1 - b));
          const int kk = (int)(off & (((size_t)1 << u) - 1));
          dst = ((size_t)1 << (c.log_n - 1 - b)) + (off >> u << u) + row_tw_pos(lm, b, kk);
        }
        fwd_fp[(size_t)k * N + dst] = (double)fwd[(size_t)k * N + i].x;
        inv_fp[(size_t)k * N + dst] = (double)inv[(size_t)k * N + i].x;
      }
      for (int i = 0; i < NC; ++i) {
        const double wf = (double)fwd[(size_t)k * N + i].x, wi = (double)inv[(size_t)k * N + i].x;
        fwd_col[(size_t)k * NC + i] = make_double2(wf, wf / (double)q);
        inv_col[(size_t)k * NC + i] = make_double2(wi, wi / (double)q);
      }
    }
    PrimeDev &P = pd[k];
    P.q = q;
    P.two_q = 2 * q;
    h_barrett_ratio(q, P.br_hi, P.br_lo);
    P.ninv = h_invmod((u64)N % q, q);
    P.ninv_sh = h_shoup(P.ninv, q);
    P.w1ninv = h_mulmod(pwi[N / 2], P.ninv, q);
    P.w1ninv_sh = h_shoup(P.w1ninv, q);
    P.mu = (u64)((~(u128)0 >> 64) / q);  // floor((2^64 - 1) / q) == floor(2^64 / q)
    P.pad_ = 0;
    P.qd = (double)q;
    P.qinv = 1.0 / (double)q;
    P.ninv_d = (double)P.ninv;
    P.ninv_q = (double)P.ninv / (double)q;
    P.w1ninv_d = (double)P.w1ninv;
    P.w1ninv_q = (double)P.w1ninv / (double)q;
  };
  const int nth = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  for (int t0 = 0; t0 < nth; ++t0)
    th.emplace_back([&, t0] {
      for (int k = t0; k < K; k += nth) work(k);
    });
  for (auto &t : th) t.join();
  c.h_primes = pd;
  c.d_primes = upload(pd);
  c.d_tw_fwd = upload(fwd);
  c.d_tw_inv = upload(inv);
  c.d_tw_fwd_fp = upload(fwd_fp);
  c.d_tw_inv_fp = upload(inv_fp);
  c.d_tw_fwd_col = upload(fwd_col);
  c.d_tw_inv_col = upload(inv_col);

  // Discrete Gaussian CDT (sigma 3.2, |e| <= 19) for the synthetic keys.
  std::vector<u64> T(20);
  {
    const double sigma = 3.2;
    double rho[20], Z = 0, cum = 0;
    for (int x = 0; x < 20; ++x) {
      rho[x] = std::exp(-(double)x * x / (2 * sigma * sigma));
      Z += (x == 0 ? 1.0 : 2.0) * rho[x];
    }
    for (int x = 0; x < 20; ++x) {
      cum += (x == 0 ? 1.0 : 2.0) * rho[x];
      T[x] = (x == 19) ? (1ull << 63) : (u64)(cum / Z * 9223372036854775808.0);
    }
  }
  c.d_gauss = upload(T);
}

void build_moddown(Ctx &c) {
  const int a = c.alpha, L = c.L;
  if (a == 0) return;
  std::vector<ulonglong2> phatinv(a), pinv(L);
  std::vector<u64> w((size_t)L * a);
  for (int i = 0; i < a; ++i) {
    const u64 pi = c.primes[L + i];
    u64 prod = 1;
    for (int t = 0; t < a; ++t)
      if (t != i) prod = h_mulmod(prod, c.primes[L + t] % pi, pi);
    const u64 v = h_invmod(prod, pi);
    phatinv[i] = make_ulonglong2(v, h_shoup(v, pi));
  }
  for (int j = 0; j < L; ++j) {
    const u64 q = c.primes[j];
    u64 P = 1;
    for (int t = 0; t < a; ++t) P = h_mulmod(P, c.primes[L + t] % q, q);
    const u64 v = h_invmod(P, q);
    pinv[j] = make_ulonglong2(v, h_shoup(v, q));
    for (int i = 0; i < a; ++i) {
      u64 r = 1;
      for (int t = 0; t < a; ++t)
        if (t != i) r = h_mulmod(r, c.primes[L + t] % q, q);
      w[(size_t)j * a + i] = r;
    }
  }
  c.d_phatinv = upload(phatinv);
  c.d_pinv = upload(pinv);
  std::vector<ulonglong2> pmodq(L);
  for (int j = 0; j < L; ++j) {
    const u64 q = c.primes[j];
    u64 P = 1;
    for (int t = 0; t < a; ++t) P = h_mulmod(P, c.primes[L + t] % q, q);
    pmodq[j] = make_ulonglong2(P, h_shoup(P, q));
  }
  c.d_pmodq = upload(pmodq);
  std::vector<u64> wsh(w.size());
  for (int j = 0; j < L; ++j)
    for (int i = 0; i < a; ++i) wsh[(size_t)j * a + i] = h_shoup(w[(size_t)j * a + i], c.primes[j]);
  std::vector<double> wq(w.size(), 0.0);
  for (int j = 0; j < L; ++j)
    if (c.primes[j] < kFpBound)
      for (int i = 0; i < a; ++i)
        wq[(size_t)j * a + i] = (double)w[(size_t)j * a + i] / (double)c.primes[j];
  c.d_mdw = upload(w);
  c.d_mdwsh = upload(wsh);
  c.d_mdwq = upload(wq);
  c.md = ModDownDev{a, L, c.d_phatinv, c.d_mdw, c.d_pinv, c.d_mdwsh, c.d_mdwq};
}

void build_level(Ctx &c, Level &lv, int Ql) {
  // Output aggregation keeps the whole ciphertext on every rank: its limb
  // layout is the single-GPU one, and only the digits (d % world == rank)
  // are split.
  const bool oa = c.oa();
  const int a = c.alpha, L = c.L, G = oa ? 1 : c.world, g = oa ? 0 : c.rank;
  lv.Ql = Ql;
  lv.QlP = Ql + a;
  lv.beta = (Ql + a - 1) / a;
  lv.prime_of.h.resize(lv.QlP);
  for (int j = 0; j < lv.QlP; ++j) lv.prime_of.h[j] = j < Ql ? j : L + (j - Ql);
  // owned output limbs: Q limbs j = g, g+G, ... then P limbs with key index (L+i) % G == g
  for (int j = g; j < Ql; j += G) lv.out_j.h.push_back(j);
  lv.n_q = (int)lv.out_j.h.size();
  std::vector<int> own_p;
  for (int i = 0; i < a; ++i)
    if ((L + i) % G == g) own_p.push_back(i);
  lv.n_p = (int)own_p.size();
  for (int i : own_p) lv.out_j.h.push_back(Ql + i);
  lv.n_out = (int)lv.out_j.h.size();
  for (int s = 0; s < lv.n_out; ++s) {
    const int j = lv.out_j.h[s];
    lv.key_slot.h.push_back(lv.prime_of.h[j] / G);
    lv.c_slot.h.push_back(j < Ql ? j / G : -1);
  }
  lv.coef_ml = (Ql + G - 1) / G;
  auto my_digit = [&](int d) { return !oa || d % c.world == c.rank; };
  for (int d = 0; d < lv.beta; ++d)
    if (my_digit(d)) lv.digits.h.push_back(d);
  for (int d = 0; d < lv.beta; ++d)
    for (int s = 0; s < lv.n_out; ++s) {
      const int j = lv.out_j.h[s];
      const bool in_digit = j < Ql && j / a == d;
      lv.t_jobs.h.push_back(in_digit || !my_digit(d) ? -1 : lv.prime_of.h[j]);
    }
  for (int s = 0; s < lv.n_q; ++s) {
    lv.q_index.h.push_back(lv.out_j.h[s]);
    lv.cx_slot_q.h.push_back(s);
  }
  for (int p = 0; p < 2; ++p)
    for (int s = 0; s < lv.n_out; ++s) lv.cx_prime.h.push_back(lv.prime_of.h[lv.out_j.h[s]]);
  // input INTT: owned Q limbs, or (output aggregation) the limbs of this rank's digits
  for (int s = 0; s < lv.n_q; ++s) {
    const int j = lv.out_j.h[s];
    if (!my_digit(j / a)) continue;
    lv.intt_off.h.push_back((long long)s * c.N);
    lv.intt_prime.h.push_back(j);
  }
  lv.n_intt = (int)lv.intt_prime.h.size();
  for (int p = 0; p < 2; ++p)
    for (int s = 0; s < lv.n_q; ++s) lv.z_jobs.h.push_back(lv.out_j.h[s]);
  // P part: offsets of the owned P slots that get inverse-transformed
  const long long N = c.N;
  for (int p = 0; p < 2; ++p)
    for (int k = 0; k < lv.n_p; ++k) {
      lv.p_jobs.h.push_back(L + own_p[k]);
      lv.p_cx_offsets.h.push_back(((long long)p * lv.n_out + lv.n_q + k) * N);
      if (G == 1) lv.p_offsets.h.push_back(((long long)p * lv.n_out + lv.n_q + k) * N);
      else lv.p_offsets.h.push_back(((long long)k * 2 + p) * N);  // ysend [max_p][2][N]
    }
  // The integer launch of the fused row pass also runs the inverse row pass
  // of the owned P slots (the first half of step 5) when every P prime takes
  // the non-lazy integer inverse path; output aggregation sums cx over the
  // ranks first, so it keeps the separate pass.
  bool fold = !oa && lv.n_p > 0;
  for (int k = 0; k < lv.n_p; ++k) fold = fold && c.primes[L + own_p[k]] >= kInvLazyBound;
  if (fold)
    for (int s = 0; s < lv.n_out; ++s)
      for (int p = 0; p < 2; ++p)
        lv.fold_off.h.push_back(s < lv.n_q ? -1 : lv.p_offsets.h[p * lv.n_p + (s - lv.n_q)]);
  // where P limb i of poly p lives after the (optional) all-gather
  for (int p = 0; p < 2; ++p)
    for (int i = 0; i < a; ++i) {
      if (G == 1) {
        lv.y_off.h.push_back(((long long)p * lv.n_out + lv.n_q + i) * N);
      } else {
        const int owner = (L + i) % G;
        int pslot = 0;
        for (int i2 = 0; i2 < i; ++i2)
          if ((L + i2) % G == owner) ++pslot;
        lv.y_off.h.push_back((((long long)owner * c.max_p_own + pslot) * 2 + p) * N);
      }
    }
  // ModUp constants
  std::vector<ulonglong2> qhi((size_t)lv.beta * a, make_ulonglong2(0, 0));
  std::vector<u64> w((size_t)lv.beta * lv.QlP * a, 0);
  for (int d = 0; d < lv.beta; ++d) {
    const int lo = d * a, hi = std::min(Ql, lo + a);
    for (int i = lo; i < hi; ++i) {
      const u64 qi = c.primes[i];
      u64 prod = 1;
      for (int t = lo; t < hi; ++t)
        if (t != i) prod = h_mulmod(prod, c.primes[t] % qi, qi);
      const u64 v = h_invmod(prod, qi);
      qhi[(size_t)d * a + (i - lo)] = make_ulonglong2(v, h_shoup(v, qi));
    }
    for (int j = 0; j < lv.QlP; ++j) {
      const u64 m = c.primes[lv.prime_of.h[j]];
      for (int i = lo; i < hi; ++i) {
        u64 r = 1 % m;
        for (int t = lo; t < hi; ++t)
          if (t != i) r = h_mulmod(r, c.primes[t] % m, m);
        w[((size_t)d * lv.QlP + j) * a + (i - lo)] = r;
      }
    }
  }
  // fused ModUp jobs and the scaled-INTT constants
  auto scale_pair = [&](int prime, u64 cst, std::vector<ulonglong2> &out) {
    const PrimeDev &P = c.h_primes[prime];
    const u64 q = P.q;
    const u64 a0 = h_mulmod(P.ninv, cst, q), a1 = h_mulmod(P.w1ninv, cst, q);
    if (q < kFpBound) {  // FP64 primes: the bits of {s, fl(s/q)}
      auto bits = [](double d) {
        u64 b;
        std::memcpy(&b, &d, 8);
        return b;
      };
      out.push_back(make_ulonglong2(bits((double)a0), bits((double)a0 / (double)q)));
      out.push_back(make_ulonglong2(bits((double)a1), bits((double)a1 / (double)q)));
    } else {
      out.push_back(make_ulonglong2(a0, h_shoup(a0, q)));
      out.push_back(make_ulonglong2(a1, h_shoup(a1, q)));
    }
  };
  // Input all-gather layout: rank r's share of the coefficient-form input
  // is coef_words words at r * coef_words; its local slot k sits at
  // slot_off(k), packed (pack42) for k >= 1 when the context packs.
  {
    const long long N = c.N, P = c.pk_words;
    auto slot_off = [&](int k) {
      return c.pack ? (k == 0 ? 0 : N + (long long)(k - 1) * P) : (long long)k * N;
    };
    lv.coef_words = c.pack ? N + (long long)(lv.coef_ml - 1) * P : (long long)lv.coef_ml * N;
    for (int d = 0; d < lv.beta; ++d)
      for (int i = 0; i < a; ++i) {
        const int j = d * a + i;
        const int k = j / G;
        const long long w = (long long)(j % G) * lv.coef_words + slot_off(k);
        lv.src_ref.h.push_back(j < Ql ? (w << 1) | (c.pack && k >= 1 ? 1 : 0) : 0);
      }
    if (c.pack)
      for (int s = 0; s < lv.n_q; ++s) lv.coef_off.h.push_back(slot_off(s));
  }
  // Job order of the fused column passes: jobs whose target prime takes the
  // integer path (q_0 and the 60-bit special primes) run 2-3x longer than
  // the FP64 ones and use the integer pipes, so they are spread evenly over
  // the list (the first at the front): co-resident CTAs then keep the FP64
  // and integer pipes busy at the same time, and no wave at the end runs
  // integer work alone.
  std::vector<std::pair<int, int>> fp_jobs, int_jobs;  // (d, s)
  for (int d = 0; d < lv.beta; ++d)
    for (int s = 0; s < lv.n_out; ++s) {
      const int pj = lv.t_jobs.h[(size_t)d * lv.n_out + s];
      if (pj < 0) continue;
      (c.primes[pj] < kFpBound ? fp_jobs : int_jobs).push_back({d, s});
    }
  for (const auto &ds : interleave_jobs(fp_jobs, int_jobs)) {
    const int d = ds.first, s = ds.second, pj = lv.t_jobs.h[(size_t)d * lv.n_out + s];
    lv.job_d.h.push_back(d);
    lv.job_s.h.push_back(s);
    lv.job_prime.h.push_back(pj);
    lv.job_off.h.push_back(((long long)d * lv.n_out + s) * N);
    if (c.primes[pj] < kFpBound) ++lv.n_jobs_fp;
  }
  lv.n_jobs = (int)lv.job_d.h.size();
  std::vector<int> md_fp, md_int;
  for (int p = 0; p < 2; ++p)
    for (int s = 0; s < lv.n_q; ++s)
      (c.primes[lv.out_j.h[s]] < kFpBound ? md_fp : md_int).push_back(p * lv.n_q + s);
  lv.md_job_ps.h = interleave_jobs(md_fp, md_int);
  lv.n_md_fp = (int)md_fp.size();
  // the fused row pass + inner product runs one launch over the FP64 output
  // slots and one over the integer ones
  for (int s = 0; s < lv.n_out; ++s)
    (c.primes[lv.prime_of.h[lv.out_j.h[s]]] < kFpBound ? lv.rip_fp : lv.rip_int).h.push_back(s);
  std::vector<ulonglong2> sin, sp;
  for (int i = 0; i < lv.n_intt; ++i) {
    const int j = lv.intt_prime.h[i], d = j / a;
    scale_pair(j, qhi[(size_t)d * a + (j - d * a)].x, sin);
  }
  for (int p = 0; p < 2; ++p)
    for (int k = 0; k < lv.n_p; ++k) {
      const int i = own_p[k];
      const u64 pi = c.primes[L + i];
      u64 prod = 1;
      for (int t = 0; t < a; ++t)
        if (t != i) prod = h_mulmod(prod, c.primes[L + t] % pi, pi);
      scale_pair(L + i, h_invmod(prod, pi), sp);
    }
  // rescale by the last prime of this level
  if (Ql >= 2) {
    const int last = Ql - 1;
    const u64 ql = c.primes[last];
    std::vector<ulonglong2> rpinv(L, make_ulonglong2(0, 0)), rsc;
    for (int j = 0; j < last; ++j) {
      const u64 qj = c.primes[j], v = h_invmod(ql % qj, qj);
      rpinv[j] = make_ulonglong2(v, h_shoup(v, qj));
    }
    scale_pair(last, 1, rsc);
    scale_pair(last, 1, rsc);
    const bool have_last = (last % G) == g;
    for (int p = 0; p < 2; ++p) {
      lv.rs_off.h.push_back(((long long)p * lv.n_q + (have_last ? last / G : 0)) * c.N);
      lv.rs_prime.h.push_back(last);
    }
    lv.rs_pinv = upload(rpinv);
    lv.rs_scale = upload(rsc);
    up_i64(lv.rs_off);
    up_ints(lv.rs_prime);
    lv.rs_md = ModDownDev{1, last, nullptr, nullptr, lv.rs_pinv, nullptr, nullptr};
  }
  up_i64(lv.src_ref);
  up_i64(lv.coef_off);
  up_ints(lv.rip_fp);
  up_ints(lv.rip_int);
  up_ints(lv.digits);
  up_ints(lv.cx_prime);
  up_ints(lv.intt_prime);
  up_i64(lv.intt_off);
  up_ints(lv.md_job_ps);
  up_ints(lv.job_d);
  up_ints(lv.job_s);
  up_ints(lv.job_prime);
  up_i64(lv.job_off);
  lv.scale_in = upload(sin);
  lv.scale_p = upload(sp);
  up_ints(lv.prime_of);
  up_ints(lv.out_j);
  up_ints(lv.key_slot);
  up_ints(lv.c_slot);
  up_ints(lv.t_jobs);
  up_ints(lv.q_index);
  up_ints(lv.z_jobs);
  up_ints(lv.cx_slot_q);
  up_ints(lv.p_jobs);
  up_i64(lv.p_offsets);
  up_i64(lv.p_cx_offsets);
  up_i64(lv.fold_off);
  up_i64(lv.y_off);
  lv.qhatinv = upload(qhi);
  std::vector<u64> wsh(w.size());
  std::vector<double> wq(w.size(), 0.0);
  for (int d = 0; d < lv.beta; ++d)
    for (int j = 0; j < lv.QlP; ++j)
      for (int i = 0; i < a; ++i) {
        const size_t o = ((size_t)d * lv.QlP + j) * a + i;
        const u64 m = c.primes[lv.prime_of.h[j]];
        wsh[o] = h_shoup(w[o], m);
        if (m < kFpBound) wq[o] = (double)w[o] / (double)m;
      }
  lv.w = upload(w);
  lv.wsh = upload(wsh);
  lv.wq = upload(wq);
  lv.mu = ModUpDev{Ql, lv.QlP, lv.beta, a, lv.prime_of.d, lv.qhatinv, lv.w, lv.wsh, lv.wq};
  lv.lay = KsLayout{lv.n_out,  lv.out_j.d,  lv.key_slot.d,           lv.c_slot.d, G,
                    lv.coef_ml, lv.digits.d, (int)lv.digits.h.size(), lv.rip_fp.d,
                    lv.rip_int.d, (int)lv.rip_fp.h.size(), (int)lv.rip_int.h.size(),
                    lv.fold_off.h.empty() ? nullptr : lv.fold_off.d};
}

void ctx_init(Ctx &c, const ks_params *prm, int device, int rank, int world, ncclComm_t comm,
              const void *nccl_id) {
  KS_REQUIRE(prm != nullptr, "params is null");
  KS_REQUIRE(ntt_supported_log_n((int)prm->log_n), "log_n must be in [12, 16]");
  KS_REQUIRE(prm->n_q >= 1 && prm->q != nullptr, "need at least one Q prime");
  KS_REQUIRE(prm->n_p >= 0 && prm->n_p <= KS_MAX_ALPHA, "alpha must be in [0, 8]");
  KS_REQUIRE(prm->n_p == 0 || prm->p != nullptr, "P primes missing");
  KS_REQUIRE(world >= 1 && rank >= 0 && rank < world, "bad rank/world");
  KS_REQUIRE(prm->n_q + prm->n_p <= KS_MAX_PRIMES, "too many primes");
  c.device = device;
  c.rank = rank;
  c.world = world;
  c.mode = world > 1 ? prm->mode : KS_MODE_INPUT_BROADCAST;
  KS_REQUIRE(c.mode == KS_MODE_INPUT_BROADCAST || c.mode == KS_MODE_OUTPUT_AGGREGATION,
             "unknown mode");
  c.max_batch = std::max(1, prm->max_batch);
  c.group = std::max(1, prm->group);
  KS_REQUIRE(c.group <= kMaxGroup, "group must be in [1, 8]");
  c.log_n = (int)prm->log_n;
  c.N = 1 << c.log_n;
  c.L = prm->n_q;
  c.alpha = prm->n_p;
  c.K = c.L + c.alpha;
  for (int i = 0; i < c.L; ++i) c.primes.push_back(prm->q[i]);
  for (int i = 0; i < c.alpha; ++i) c.primes.push_back(prm->p[i]);
  for (int k = 0; k < c.K; ++k) {
    const u64 q = c.primes[k];
    KS_REQUIRE(q > 2 && q < (1ull << 61), "primes must be below 2^61");
    KS_REQUIRE(q % (2ull * c.N) == 1, "primes must be 1 mod 2N");
    KS_REQUIRE(h_is_prime(q), "modulus is not prime");
    for (int k2 = 0; k2 < k; ++k2) KS_REQUIRE(c.primes[k2] != q, "primes must be distinct");
  }
  KS_CUDA(cudaSetDevice(device));
  build_tables(c);
  // key shard: cyclic key-basis limbs of all digits (input broadcast), or
  // all limbs of the digits d % world == rank (output aggregation)
  for (int kj = c.oa() ? 0 : rank; kj < c.K; kj += c.oa() ? 1 : world) c.own_key.push_back(kj);
  c.own_key_prime.h = c.own_key;
  up_ints(c.own_key_prime);
  if (c.alpha > 0) {
    const int beta = (c.L + c.alpha - 1) / c.alpha;
    for (int d = 0; d < beta; ++d)
      if (!c.oa() || d % world == rank) c.key_digits.push_back(d);
  }
  if (c.alpha > 0) {
    for (int g = 0; g < world; ++g) {
      int cnt = 0;
      for (int i = 0; i < c.alpha; ++i)
        if ((c.L + i) % world == g) ++cnt;
      c.max_p_own = std::max(c.max_p_own, cnt);
    }
    build_moddown(c);
    // pack the input all-gather when every limb after q_0 fits 42 bits
    if (world > 1 && !c.oa() && c.L >= 2) {
      bool fits = true;
      for (int j = 1; j < c.L; ++j) fits = fits && c.primes[j] < (1ull << 42);
      c.pack = fits;
      c.pk_words = fits ? (long long)kPackWords * c.N / 16 : 0;
    }
    c.levels.resize(c.L + 1);
    for (int Ql = 1; Ql <= c.L; ++Ql) build_level(c, c.levels[Ql], Ql);
    // scratch, sized for the top level
    const Level &top = c.levels[c.L];
    const size_t N = c.N;
    const bool ib = !c.replicated();  // input broadcast over world > 1 ranks
    const size_t nq = ib ? n_local(rank, world, c.L) : c.L;
    const size_t n_key_own = c.own_key.size();
    // per member of a group (member strides of the group layout): automorphism
    // output g0, coefficient input (send buffer of the all-gather) and its
    // gathered form [G][ml][N], extended digits t, cx, the P limbs sent and
    // gathered before ModDown, z, and the staging of a host ciphertext
    const size_t g = c.group;
    c.st_g = 2 * nq * N;
    c.st_coef = top.coef_words;
    c.st_coef_all = ib ? world * c.st_coef : c.st_coef;
    c.st_t = (size_t)top.beta * top.n_out * N;
    c.st_cx = 2 * (size_t)top.n_out * N;
    c.st_ys = ib ? (size_t)c.max_p_own * 2 * N : 0;
    c.st_ya = ib ? (size_t)world * c.st_ys : 0;
    c.st_z = 2 * nq * N;
    c.st_ct = 2 * nq * N;
    size_t w_g = g * c.st_g, w_coef = g * c.st_coef, w_coef_all = ib ? g * c.st_coef_all : 0;
    size_t w_t = std::max<size_t>(g * c.st_t, 3 * n_key_own * N);  // key generation borrows lane 0's t
    size_t w_cx = g * c.st_cx;
    size_t w_ys = g * c.st_ys;
    size_t w_ya = g * c.st_ya;
    size_t w_z = g * c.st_z;
    size_t w_ct = g * c.st_ct;  // device copies of host ciphertexts (ks_rotate_batch_host)
    c.arena_words = w_g + w_coef + w_coef_all + w_t + w_cx + w_ys + w_ya + w_z + w_ct;
    // one scratch arena per lane; lanes = max_batch (1..8), each for `group` key switches
    // (contexts made by ks_ctx_create_all are set up one after another on one
    // thread, where splitting communicators would block, so they keep one lane)
    c.lanes.resize(comm ? 1 : std::min(8, c.max_batch));
    for (size_t li = 0; li < c.lanes.size(); ++li) {
      Ctx::Lane &ln = c.lanes[li];
      ln.arena = dev_alloc<u64>(c.arena_words);
      u64 *p = ln.arena;
      ln.s_g = p; p += w_g;
      ln.s_coef = p; p += w_coef;
      ln.s_coef_all = ib ? p : ln.s_coef; p += w_coef_all;
      ln.s_t = p; p += w_t;
      ln.s_cx = p; p += w_cx;
      ln.s_ysend = p; p += w_ys;
      ln.s_yall = p; p += w_ya;
      ln.s_z = p; p += w_z;
      ln.s_ct = p; p += w_ct;
      if (li > 0) KS_CUDA(cudaStreamCreateWithFlags(&ln.stream, cudaStreamNonBlocking));
      KS_CUDA(cudaEventCreateWithFlags(&ln.done, cudaEventDisableTiming));
      KS_CUDA(cudaStreamCreateWithFlags(&ln.side, cudaStreamNonBlocking));
      KS_CUDA(cudaEventCreateWithFlags(&ln.ev_fork, cudaEventDisableTiming));
      KS_CUDA(cudaEventCreateWithFlags(&ln.ev_join, cudaEventDisableTiming));
      KS_CUDA(cudaStreamCreateWithFlags(&ln.copy, cudaStreamNonBlocking));
      for (int h = 0; h < 2; ++h) {
        KS_CUDA(cudaEventCreateWithFlags(&ln.ev_in[h], cudaEventDisableTiming));
        KS_CUDA(cudaEventCreateWithFlags(&ln.ev_out[h], cudaEventDisableTiming));
      }
    }
    KS_CUDA(cudaEventCreateWithFlags(&c.ev_fork, cudaEventDisableTiming));
  }
  if (world > 1) {
    if (comm) {
      c.comm = comm;
    } else {
      KS_REQUIRE(nccl_id != nullptr, "world > 1 needs an NCCL unique id");
      ncclUniqueId id;
      std::memcpy(&id, nccl_id, sizeof(id));
      KS_NCCL(ncclCommInitRank(&c.comm, world, id, rank));
    }
    c.own_comm = true;
    // every lane gets its own communicator so collectives of different key
    // switches never share one (all ranks create them in the same order)
    for (size_t li = 0; li < c.lanes.size(); ++li) {
      if (li == 0) c.lanes[li].comm = c.comm;
      else KS_NCCL(ncclCommSplit(c.comm, 0, rank, &c.lanes[li].comm, nullptr));
    }
  }
  KS_CUDA(cudaDeviceSynchronize());
}

void ctx_free(Ctx &c) {
  if (c.wd_thread.joinable()) {
    c.wd_stop = true;
    c.wd_thread.join();
  }
  cudaSetDevice(c.device);
  cudaDeviceSynchronize();
  for (auto &w : c.wd_pending) cudaEventDestroy(w.ev);
  for (cudaEvent_t e : c.wd_free) cudaEventDestroy(e);
  c.wd_pending.clear();
  c.wd_free.clear();
  auto f = [](void *p) {
    if (p) cudaFree(p);
  };
  for (auto &kv : c.keys) f(kv.second.d);
  c.keys.clear();
  for (auto &lv : c.levels) {
    for (DevInts *t : {&lv.prime_of, &lv.out_j, &lv.key_slot, &lv.c_slot, &lv.t_jobs,
                       &lv.q_index, &lv.z_jobs, &lv.cx_slot_q, &lv.p_jobs})
      f(t->d);
    f(lv.p_offsets.d);
    f(lv.p_cx_offsets.d);
    f(lv.fold_off.d);
    f(lv.y_off.d);
    f(lv.qhatinv);
    f(lv.src_ref.d);
    f(lv.coef_off.d);
    for (DevInts *t : {&lv.job_d, &lv.job_s, &lv.job_prime, &lv.md_job_ps,
                       &lv.digits, &lv.cx_prime, &lv.intt_prime, &lv.rip_fp, &lv.rip_int})
      f(t->d);
    f(lv.job_off.d);
    f(lv.intt_off.d);
    f(lv.rs_off.d);
    f(lv.rs_prime.d);
    f(lv.rs_pinv);
    f(lv.rs_scale);
    f(lv.scale_in);
    f(lv.scale_p);
    f(lv.w);
    f(lv.wsh);
    f(lv.wq);
  }
  f(c.own_key_prime.d);
  f(c.d_primes);
  f(c.d_tw_fwd);
  f(c.d_tw_inv);
  f(c.d_tw_fwd_fp);
  f(c.d_tw_inv_fp);
  f(c.d_tw_fwd_col);
  f(c.d_tw_inv_col);
  f(c.d_gauss);
  f(c.d_phatinv);
  f(c.d_pinv);
  f(c.d_pmodq);
  f(c.d_mdw);
  f(c.d_mdwsh);
  f(c.d_mdwq);
  for (size_t li = 0; li < c.lanes.size(); ++li) {
    Ctx::Lane &ln = c.lanes[li];
    f(ln.arena);
    if (ln.stream) cudaStreamDestroy(ln.stream);
    if (ln.done) cudaEventDestroy(ln.done);
    if (ln.side) cudaStreamDestroy(ln.side);
    if (ln.ev_fork) cudaEventDestroy(ln.ev_fork);
    if (ln.ev_join) cudaEventDestroy(ln.ev_join);
    if (ln.copy) cudaStreamDestroy(ln.copy);
    for (int h = 0; h < 2; ++h) {
      if (ln.ev_in[h]) cudaEventDestroy(ln.ev_in[h]);
      if (ln.ev_out[h]) cudaEventDestroy(ln.ev_out[h]);
    }
    if (li > 0 && ln.comm) ncclCommDestroy(ln.comm);
  }
  c.lanes.clear();
  if (c.ev_fork) cudaEventDestroy(c.ev_fork);
  for (auto &pe : c.prof_events) {
    cudaEventDestroy(pe.second.first);
    cudaEventDestroy(pe.second.second);
  }
  for (auto e : c.event_pool) cudaEventDestroy(e);
  if (c.comm && c.own_comm) ncclCommDestroy(c.comm);
  c.comm = nullptr;
}

// ---------------------------------------------------------------------------
// Keys
// ---------------------------------------------------------------------------
unsigned long long key_id(int kind, uint32_t elt) {
  return ((unsigned long long)(kind == KS_KEY_RELIN ? 0 : 1) << 32) |
         (kind == KS_KEY_RELIN ? 0u : elt);
}

void check_elt(const Ctx &c, uint32_t elt) {
  KS_REQUIRE((elt & 1u) && elt < 2u * (uint32_t)c.N, "galois element must be odd and < 2N");
}

KeyShard &key_alloc(Ctx &c, int kind, uint32_t elt) {
  KS_REQUIRE(c.alpha > 0, "context has no special primes (NTT-only context)");
  KS_REQUIRE(kind == KS_KEY_RELIN || kind == KS_KEY_GALOIS, "unknown key kind");
  if (kind == KS_KEY_GALOIS) check_elt(c, elt);
  auto id = key_id(kind, elt);
  auto it = c.keys.find(id);
  if (it != c.keys.end()) return it->second;
  KeyShard k;
  k.limbs = (int)c.own_key.size();
  k.beta = (int)c.key_digits.size();
  k.d = dev_alloc<u64>(std::max<size_t>(1, (size_t)k.beta * 2 * k.limbs * c.N));
  return c.keys[id] = k;
}

// Unregisters and frees key (kind, elt) when the call that fills it fails
// part-way (upload, generation or distribution), so no later key switch runs
// on a half-written key.  dismiss() on success.
struct KeyFillGuard {
  Ctx &c;
  unsigned long long id;
  bool ok = false;
  KeyFillGuard(Ctx &c_, int kind, uint32_t elt) : c(c_), id(key_id(kind, elt)) {}
  void dismiss() { ok = true; }
  ~KeyFillGuard() {
    if (ok) return;
    auto it = c.keys.find(id);
    if (it == c.keys.end()) return;
    cudaSetDevice(c.device);
    cudaFree(it->second.d);  // cudaFree synchronises with the device before releasing
    c.keys.erase(it);
  }
};

const KeyShard &key_get(Ctx &c, int kind, uint32_t elt) {
  auto it = c.keys.find(key_id(kind, elt));
  if (it == c.keys.end())
    throw KsError{KS_ERR_NO_KEY, kind == KS_KEY_RELIN
                                     ? std::string("no relinearisation key uploaded")
                                     : "no galois key for element " + std::to_string(elt)};
  return it->second;
}

size_t full_key_words(const Ctx &c) {
  return c.alpha ? (size_t)((c.L + c.alpha - 1) / c.alpha) * 2 * c.K * c.N : 0;
}

// Words of rank g's shard of a full key (the layout key_alloc gives rank g).
size_t shard_words(const Ctx &c, int g) {
  const int beta = (c.L + c.alpha - 1) / c.alpha;
  if (c.world == 1) return full_key_words(c);
  if (c.oa()) return (size_t)n_local(g, c.world, beta) * 2 * c.K * c.N;
  return (size_t)beta * 2 * n_local(g, c.world, c.K) * c.N;
}

// Copies rank g's shard of the full key src ([beta][2][K][N]) into dst:
// input broadcast keeps the key-basis limbs kj % G == g of every digit
// ([beta][2][limbs][N]); output aggregation the digits d % G == g, all limbs.
void extract_shard(const Ctx &c, int g, const u64 *src, u64 *dst, cudaMemcpyKind dir,
                   cudaStream_t s) {
  const size_t N = c.N;
  const int beta = (c.L + c.alpha - 1) / c.alpha, G = c.world;
  if (G == 1) {
    KS_CUDA(cudaMemcpyAsync(dst, src, full_key_words(c) * 8, dir, s));
  } else if (c.oa()) {
    int di = 0;
    for (int d = g; d < beta; d += G, ++di)
      KS_CUDA(cudaMemcpyAsync(dst + (size_t)2 * di * c.K * N, src + (size_t)2 * d * c.K * N,
                              (size_t)2 * c.K * N * 8, dir, s));
  } else {
    const int limbs = n_local(g, G, c.K);
    if (limbs == 0) return;
    for (int d = 0; d < beta; ++d)
      for (int p = 0; p < 2; ++p)
        KS_CUDA(cudaMemcpy2DAsync(dst + ((size_t)(2 * d + p) * limbs) * N, N * 8,
                                  src + (((size_t)(2 * d + p) * c.K) + g) * N,
                                  (size_t)G * N * 8, N * 8, limbs, dir, s));
  }
}

void key_upload(Ctx &c, int kind, uint32_t elt, const u64 *src, size_t n_words, bool from_dev,
                cudaStream_t s) {
  KS_REQUIRE(src != nullptr, "key pointer is null");
  KS_REQUIRE(n_words == full_key_words(c), "key size mismatch: expected " +
                                               std::to_string(full_key_words(c)) + " words");
  KS_CUDA(cudaSetDevice(c.device));
  KeyFillGuard guard(c, kind, elt);
  KeyShard &k = key_alloc(c, kind, elt);
  extract_shard(c, c.rank, src, k.d,
                from_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s);
  if (!from_dev) KS_CUDA(cudaStreamSynchronize(s));
  guard.dismiss();
}

void check_alive(const Ctx &c);
void watch_collective(Ctx &c, cudaStream_t s);
template <class F>
void enqueue_nccl(Ctx &c, ncclComm_t const &comm, cudaStream_t s, F &&call);

// Key distribution: the root holds the full key in its device memory and
// sends every rank its shard over NCCL point-to-point (the root packs each
// shard into a staging buffer first); the others receive straight into their
// key shard.  Collective over the context's ranks; synchronous on return.
void key_distribute(Ctx &c, int kind, uint32_t elt, const u64 *full_dev, int root,
                    cudaStream_t s) {
  KS_REQUIRE(root >= 0 && root < c.world, "root out of range");
  KS_CUDA(cudaSetDevice(c.device));
  KeyFillGuard guard(c, kind, elt);
  if (c.world == 1) {
    KS_REQUIRE(full_dev != nullptr, "key pointer is null");
    KeyShard &k = key_alloc(c, kind, elt);
    extract_shard(c, 0, full_dev, k.d, cudaMemcpyDeviceToDevice, s);
    KS_CUDA(cudaStreamSynchronize(s));
    guard.dismiss();
    return;
  }
  check_alive(c);
  KeyShard &k = key_alloc(c, kind, elt);
  std::vector<std::unique_ptr<DevBuf<u64>>> staging(c.world);
  if (c.rank == root) {
    KS_REQUIRE(full_dev != nullptr, "the root needs the full key on its device");
    for (int g = 0; g < c.world; ++g) {
      if (g == root) {
        extract_shard(c, g, full_dev, k.d, cudaMemcpyDeviceToDevice, s);
      } else if (shard_words(c, g)) {
        staging[g].reset(new DevBuf<u64>(shard_words(c, g)));
        extract_shard(c, g, full_dev, staging[g]->p, cudaMemcpyDeviceToDevice, s);
      }
    }
  }
  enqueue_nccl(c, c.comm, s, [&](ncclComm_t cm) {
    ncclResult_t r = ncclGroupStart();
    if (r != ncclSuccess) return r;
    if (c.rank == root) {
      for (int g = 0; g < c.world && r == ncclSuccess; ++g)
        if (g != root && staging[g]) r = ncclSend(staging[g]->p, shard_words(c, g), ncclUint64, g, cm, s);
    } else if (shard_words(c, c.rank)) {
      r = ncclRecv(k.d, shard_words(c, c.rank), ncclUint64, root, cm, s);
    }
    const ncclResult_t r2 = ncclGroupEnd();
    return r != ncclSuccess ? r : r2;
  });
  KS_CUDA(cudaStreamSynchronize(s));  // the staging buffers are freed after this
  check_alive(c);
  guard.dismiss();
}

void key_generate(Ctx &c, int kind, uint32_t elt, const int8_t *sk_host, u64 seed,
                  cudaStream_t s) {
  KS_REQUIRE(sk_host != nullptr, "secret is null");
  KS_CUDA(cudaSetDevice(c.device));
  KeyFillGuard guard(c, kind, elt);
  KeyShard &k = key_alloc(c, kind, elt);
  const int n = k.limbs, N = c.N;
  const NttTables T = c.tables();
  DevBuf<int8_t> sk_buf(N);
  int8_t *d_sk = sk_buf.p;
  KS_CUDA(cudaMemcpyAsync(d_sk, sk_host, N, cudaMemcpyHostToDevice, s));
  u64 *st = c.lanes[0].s_t;
  u64 *s_ntt = st, *snew = st + (size_t)n * N, *e = st + 2 * (size_t)n * N;
  const int *prime = c.own_key_prime.d;
  KS_CUDA(expand_ternary(d_sk, s_ntt, n, prime, c.d_primes, c.log_n, s));
  LimbMap ms{s_ntt, N, nullptr, prime, 0, 1};
  KS_CUDA(ntt_forward(ms, n, T, s));
  if (kind == KS_KEY_GALOIS) KS_CUDA(galois_ntt(s_ntt, snew, n, c.log_n, elt, s));
  else KS_CUDA(mul_pointwise(s_ntt, s_ntt, snew, n, prime, c.d_primes, c.log_n, s));
  // per-slot constants
  std::vector<int> in_digit(n);
  std::vector<u64> pmodq(n);
  DevBuf<u64> pmq_buf(n);
  DevBuf<int> in_buf(n);
  u64 *d_pmq = pmq_buf.p;
  int *d_in = in_buf.p;
  for (int sl = 0; sl < n; ++sl) {
    const int kj = c.own_key[sl];
    const u64 q = c.primes[kj];
    u64 P = 1;
    for (int i = 0; i < c.alpha; ++i) P = h_mulmod(P, c.primes[c.L + i] % q, q);
    pmodq[sl] = P;
  }
  KS_CUDA(cudaMemcpyAsync(d_pmq, pmodq.data(), n * 8, cudaMemcpyHostToDevice, s));
  const u64 sa = prng_stream(seed, DOM_KEY_A), se = prng_stream(seed, DOM_KEY_E);
  std::vector<std::vector<int>> flags(k.beta, std::vector<int>(n));
  for (int di = 0; di < k.beta; ++di) {
    const int d = c.key_digits[di];  // the digit's samples do not depend on the shard
    for (int sl = 0; sl < n; ++sl) {
      const int kj = c.own_key[sl];
      flags[di][sl] = (kj < c.L && kj / c.alpha == d) ? 1 : 0;
    }
    KS_CUDA(cudaMemcpyAsync(d_in, flags[di].data(), n * sizeof(int), cudaMemcpyHostToDevice, s));
    KS_CUDA(sample_gauss(e, n, prime, c.d_primes, c.d_gauss, se, (u64)d * N, c.log_n, s));
    LimbMap me{e, N, nullptr, prime, 0, 1};
    KS_CUDA(ntt_forward(me, n, T, s));
    u64 *kb = k.d + (size_t)(2 * di) * n * N, *ka = k.d + (size_t)(2 * di + 1) * n * N;
    KS_CUDA(keygen_digit(kb, ka, s_ntt, snew, e, n, prime, prime, d_in, d_pmq, sa, d, c.K,
                         c.d_primes, c.log_n, s));
    KS_CUDA(cudaStreamSynchronize(s));  // flags buffer is reused per digit
  }
  guard.dismiss();
}

// ---------------------------------------------------------------------------
// Optional per-stage timing (bench accounting; off by default)
// ---------------------------------------------------------------------------
enum Stage {
  ST_GALOIS = 0, ST_INTT_IN, ST_MODUP_COLS, ST_MODUP_ROWS_IP, ST_INTT_P, ST_MODDOWN_COLS,
  ST_MODDOWN_ROWS, ST_COMM, ST_MODUP_ROWS, ST_INNER_PROD, ST_PLAIN_MAC, ST_COUNT
};
// modup_rows and inner_product are the two halves of modup_rows_ip that the
// hoisted path and the BSGS giant steps run apart (one row pass, one inner
// product per rotation); plain_mac is the plaintext products of the BSGS matmul.
static const char *kStageNames[ST_COUNT] = {
    "galois",       "intt_input",   "modup_cols",   "modup_rows_ip", "intt_p",
    "moddown_cols", "moddown_rows", "collective",   "modup_rows",    "inner_product",
    "plain_mac"};

cudaEvent_t pool_event(Ctx &c) {
  if (!c.event_pool.empty()) {
    cudaEvent_t e = c.event_pool.back();
    c.event_pool.pop_back();
    return e;
  }
  cudaEvent_t e;
  KS_CUDA(cudaEventCreate(&e));
  return e;
}

struct StageTimer {
  Ctx &c;
  int st;
  cudaStream_t s;
  cudaEvent_t a = nullptr;
  StageTimer(Ctx &c_, int st_, cudaStream_t s_) : c(c_), st(st_), s(s_) {
    if (c.profile) {
      a = pool_event(c);
      KS_CUDA(cudaEventRecord(a, s));
    }
  }
  ~StageTimer() noexcept(false) {
    if (c.profile && a) {
      cudaEvent_t b = pool_event(c);
      KS_CUDA(cudaEventRecord(b, s));
      c.prof_events.push_back({st, {a, b}});
    }
  }
};

// ---------------------------------------------------------------------------
// Collectives
// ---------------------------------------------------------------------------
// Collective deadline.  Every collective of the hot path is followed by an
// event (watch_collective); the context's watchdog thread polls those events
// and, when one is still pending timeout_ms after it was enqueued (a rank
// that never joined, a broken link), aborts all of the context's NCCL
// communicators -- ncclCommAbort makes the waiting NCCL kernels return --
// and marks the context failed: every later call returns KS_ERR_TIMEOUT and
// the context can only be destroyed.  Nothing is watched during a graph
// capture or with timeout_ms <= 0.
void abort_comms(Ctx &c, const char *why) {
  std::lock_guard<std::mutex> g(c.nccl_mu);
  if (c.aborted.load()) return;
  // the message is written before the flag, and only here: check_alive reads
  // it once the flag is set, never racing the calling thread's c.err
  c.abort_msg = why;
  c.aborted.store(true);
  for (size_t li = 0; li < c.lanes.size(); ++li) {
    if (c.lanes[li].comm && c.lanes[li].comm != c.comm) ncclCommAbort(c.lanes[li].comm);
    c.lanes[li].comm = nullptr;
  }
  if (c.comm) ncclCommAbort(c.comm);
  c.comm = nullptr;
  set_global_err(why);
}

void watchdog_loop(Ctx *c) {
  cudaSetDevice(c->device);
  while (!c->wd_stop.load()) {
    std::this_thread::sleep_for(std::chrono::milliseconds(2));
    bool late = false;
    {
      std::lock_guard<std::mutex> g(c->wd_mu);
      const auto now = std::chrono::steady_clock::now();
      for (size_t i = 0; i < c->wd_pending.size();) {
        const cudaError_t q = cudaEventQuery(c->wd_pending[i].ev);
        if (q == cudaErrorNotReady) {
          late = late || now > c->wd_pending[i].deadline;
          ++i;
        } else {
          if (q != cudaSuccess) cudaGetLastError();
          c->wd_free.push_back(c->wd_pending[i].ev);
          c->wd_pending[i] = c->wd_pending.back();
          c->wd_pending.pop_back();
        }
      }
    }
    if (late) {
      abort_comms(*c, "a collective did not complete within the deadline (ks_set_timeout_ms); "
                      "communicators aborted, destroy the context");
      std::lock_guard<std::mutex> g(c->wd_mu);
      for (auto &w : c->wd_pending) c->wd_free.push_back(w.ev);
      c->wd_pending.clear();
    }
  }
}

void watch_collective(Ctx &c, cudaStream_t s) {
  if (c.timeout_ms <= 0 || c.capturing) return;
  cudaEvent_t e = nullptr;
  {
    std::lock_guard<std::mutex> g(c.wd_mu);
    if (!c.wd_free.empty()) {
      e = c.wd_free.back();
      c.wd_free.pop_back();
    }
  }
  if (!e) KS_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  KS_CUDA(cudaEventRecord(e, s));
  std::lock_guard<std::mutex> g(c.wd_mu);
  c.wd_pending.push_back(
      {e, std::chrono::steady_clock::now() + std::chrono::milliseconds(c.timeout_ms)});
  if (!c.wd_thread.joinable()) c.wd_thread = std::thread(watchdog_loop, &c);
}

void check_alive(const Ctx &c) {
  if (c.aborted.load())
    throw KsError{KS_ERR_TIMEOUT, "context failed: " + c.abort_msg};
}

// Enqueues one NCCL call on the communicator held in `comm` (a lane's or the
// context's field).  The field is read under nccl_mu, the lock the watchdog
// holds while it aborts and clears the communicators, after re-checking the
// aborted flag: a communicator that ncclCommAbort has freed is never used.
template <class F>
void enqueue_nccl(Ctx &c, ncclComm_t const &comm, cudaStream_t s, F &&call) {
  {
    std::lock_guard<std::mutex> g(c.nccl_mu);
    check_alive(c);
    if (comm == nullptr) throw KsError{KS_ERR_TIMEOUT, "context failed: no communicator"};
    KS_NCCL(call(comm));
  }
  watch_collective(c, s);
}

void allgather(Ctx &c, ncclComm_t const &comm, const u64 *send, u64 *recv, size_t words,
               cudaStream_t s) {
  enqueue_nccl(c, comm, s, [&](ncclComm_t cm) {
    return ncclAllGather(send, recv, words, ncclUint64, cm, s);
  });
}

// ---------------------------------------------------------------------------
// The key switch
// ---------------------------------------------------------------------------
// One member of a group of key switches that share every launch (grid z =
// member; at most kMaxGroup).  The switched polynomial `in` (this rank's Q
// limbs, NTT form) is read through X -> X^elt; the result goes to ct0, ct1:
// with rotate, ct0 = g0 + ks0 (g0 null: ct0 = ks0) and ct1 = ks1; otherwise
// ct0 += ks0, ct1 += ks1.
struct KsMember {
  const u64 *in = nullptr;
  uint32_t elt = 1;
  const KeyShard *key = nullptr;
  u64 *ct0 = nullptr, *ct1 = nullptr;
  const u64 *g0 = nullptr;
};

// g all-gathers of `words` words per rank, member b from send + b sst into
// recv + b rst, as one NCCL group (one launch).
void allgather_group(Ctx &c, ncclComm_t const &comm, const u64 *send, long long sst, u64 *recv,
                     long long rst, size_t words, int g, cudaStream_t s) {
  enqueue_nccl(c, comm, s, [&](ncclComm_t cm) {
    ncclResult_t r = ncclGroupStart();
    for (int b = 0; b < g && r == ncclSuccess; ++b)
      r = ncclAllGather(send + b * sst, recv + b * rst, words, ncclUint64, cm, s);
    const ncclResult_t r2 = ncclGroupEnd();
    return r != ncclSuccess ? r : r2;
  });
}

// Steps 2-3 for a group: scaled coefficient form v_j = [x_j (Q_d/q_j)^-1]_{q_j}
// of the input limbs this rank extends (input broadcast all-gathers them),
// then the base extension fused into the column pass -> the lane's t.
void ks_modup_cols(Ctx &c, Ctx::Lane &L, const Level &lv, const KsMember *m, int g,
                   cudaStream_t s) {
  const NttTables T = c.tables();
  {
    StageTimer tm(c, ST_INTT_IN, s);
    MemberIn mi{};
    for (int b = 0; b < g; ++b) {
      mi.in[b] = m[b].in;
      mi.elt[b] = m[b].elt;
    }
    LimbMap min{const_cast<u64 *>(m[0].in), 0, lv.intt_off.d, lv.intt_prime.d, 0, 1, 0};
    if (c.pack) {
      // row pass into the lane's t (free until the column pass below), column
      // pass into the send buffer with the limbs after slot 0 packed
      LimbMap tmp{L.s_t, 0, lv.intt_off.d, lv.intt_prime.d, 0, 1, c.st_t};
      LimbMap mc{L.s_coef, 0, lv.coef_off.d, lv.intt_prime.d, 0, 1, c.st_coef};
      KS_CUDA(ntt_inverse_scaled_pack(min, tmp, mc, lv.n_intt, lv.scale_in, T, s, &mi, g, 1));
    } else {
      LimbMap mc{L.s_coef, 0, lv.intt_off.d, lv.intt_prime.d, 0, 1, c.st_coef};
      KS_CUDA(ntt_inverse_scaled(min, mc, lv.n_intt, lv.scale_in, T, s, 1, &mi, g));
    }
    c.launches += lv.n_intt > 0 ? 2 : 0;
  }
  if (!c.replicated()) {
    StageTimer tm(c, ST_COMM, s);
    allgather_group(c, L.comm, L.s_coef, c.st_coef, L.s_coef_all, c.st_coef_all,
                    (size_t)lv.coef_words, g, s);
  }
  {
    StageTimer tm(c, ST_MODUP_COLS, s);
    KS_CUDA(modup_fused_cols(L.s_coef_all, lv.src_ref.d, L.s_t, lv.mu, lv.lay, lv.job_d.d,
                             lv.job_s.d, lv.n_jobs, lv.n_jobs_fp, T, s, g, c.st_coef_all, c.st_t,
                             c.pack));
    c.launches += lv.n_jobs > 0 ? 1 : 0;
  }
}

// Output aggregation: sum the partial inner products of all ranks (every
// rank then holds all of cx; G q < 2^64) and reduce mod the limb primes.
void ks_aggregate(Ctx &c, Ctx::Lane &L, const Level &lv, int g, cudaStream_t s) {
  if (!c.oa()) return;
  {
    StageTimer tm(c, ST_COMM, s);
    const size_t words = (size_t)(g - 1) * c.st_cx + (size_t)2 * lv.n_out * c.N;
    enqueue_nccl(c, L.comm, s, [&](ncclComm_t cm) {
      return ncclAllReduce(L.s_cx, L.s_cx, words, ncclUint64, ncclSum, cm, s);
    });
  }
  for (int b = 0; b < g; ++b) {
    KS_CUDA(mod_reduce(L.s_cx + b * c.st_cx, 2 * lv.n_out, lv.cx_prime.d, c.d_primes, c.log_n, s));
    c.launches += 1;
  }
}

// Steps 5-7 for a group: ModDown of each member's cx into its ciphertext
// (see moddown_fused_rows for rotate).
void ks_moddown(Ctx &c, Ctx::Lane &L, const Level &lv, const KsMember *m, int g, bool rotate,
                cudaStream_t s, bool p_rows_done = false) {
  const size_t N = c.N;
  const NttTables T = c.tables();
  // 5. P part to scaled coefficient form [y_i (P/p_i)^-1]_{p_i}
  const u64 *y_base;
  long long y_bstride;
  if (c.replicated()) {
    StageTimer tm(c, ST_INTT_P, s);
    LimbMap mp{L.s_cx, 0, lv.p_offsets.d, lv.p_jobs.d, 0, 1, c.st_cx};
    if (p_rows_done) {  // the fused row pass has run the inverse row pass in place
      KS_CUDA(ntt_inverse_cols_scaled(mp, 2 * lv.n_p, lv.scale_p, T, s, g));
      c.launches += lv.n_p > 0 ? 1 : 0;
    } else {
      KS_CUDA(ntt_inverse_scaled(mp, mp, 2 * lv.n_p, lv.scale_p, T, s, 1, nullptr, g));
      c.launches += lv.n_p > 0 ? 2 : 0;
    }
    y_base = L.s_cx;
    y_bstride = c.st_cx;
  } else {
    if (lv.n_p > 0) {  // the owned P limbs of cx, inverse-transformed into the send buffer
      StageTimer tm(c, ST_INTT_P, s);
      LimbMap src{L.s_cx, 0, lv.p_cx_offsets.d, lv.p_jobs.d, 0, 1, c.st_cx};
      LimbMap dst{L.s_ysend, 0, lv.p_offsets.d, lv.p_jobs.d, 0, 1, c.st_ys};
      if (p_rows_done) {  // the fused row pass has written the row-passed limbs to ysend
        KS_CUDA(ntt_inverse_cols_scaled(dst, 2 * lv.n_p, lv.scale_p, T, s, g));
        c.launches += 1;
      } else {
        KS_CUDA(ntt_inverse_scaled(src, dst, 2 * lv.n_p, lv.scale_p, T, s, 1, nullptr, g));
        c.launches += 2;
      }
    }
    StageTimer tm(c, ST_COMM, s);
    allgather_group(c, L.comm, L.s_ysend, c.st_ys, L.s_yall, c.st_ya,
                    (size_t)c.max_p_own * 2 * N, g, s);
    y_base = L.s_yall;
    y_bstride = c.st_ya;
  }
  // 6. P -> Q conversion fused into the column pass
  {
    StageTimer tm(c, ST_MODDOWN_COLS, s);
    KS_CUDA(moddown_fused_cols(y_base, lv.y_off.d, L.s_z, lv.n_q, lv.q_index.d, c.md,
                               lv.md_job_ps.d, lv.n_md_fp, T, s, g, y_bstride, c.st_z));
    c.launches += lv.n_q > 0 ? 1 : 0;
  }
  // 7. row pass with (cx - z) * P^-1 and the add to the ciphertext in the epilogue
  {
    StageTimer tm(c, ST_MODDOWN_ROWS, s);
    GroupArgs G{};
    G.n = g;
    G.z = c.st_z;
    G.cx = c.st_cx;
    for (int b = 0; b < g; ++b) {
      G.ct0[b] = m[b].ct0;
      G.ct1[b] = m[b].ct1;
      G.g0p[b] = m[b].g0;
    }
    KS_CUDA(moddown_fused_rows_group(G, L.s_z, lv.n_q, lv.q_index.d, lv.cx_slot_q.d, L.s_cx,
                                     (long long)lv.n_out * N, rotate, c.md, T, s));
    c.launches += lv.n_q > 0 ? 1 : 0;
  }
}

// The key switch of a group of g members on lane L (steps 2-7; the caller has
// done step 1, the automorphism of c0, where it rotates).
void keyswitch_group(Ctx &c, Ctx::Lane &L, const Level &lv, const KsMember *m, int g,
                     bool rotate, cudaStream_t s) {
  KS_REQUIRE(g >= 1 && g <= c.group, "group larger than the context's scratch");
  const NttTables T = c.tables();
  bool p_rows_done = false;
  ks_modup_cols(c, L, lv, m, g, s);
  // 4. row pass of every extended limb fused with the inner product
  {
    StageTimer tm(c, ST_MODUP_ROWS_IP, s);
    if (lv.lay.n_digits > 0) {
      GroupArgs G{};
      G.n = g;
      G.t = c.st_t;
      G.cx = c.st_cx;
      // folded inverse row pass of the P slots: in place in cx (one GPU) or
      // into the all-gather send buffer (input broadcast)
      p_rows_done = lv.lay.fold_off != nullptr;
      G.fold = c.world == 1 ? L.s_cx : L.s_ysend;
      G.fold_b = c.world == 1 ? c.st_cx : c.st_ys;
      for (int b = 0; b < g; ++b) {
        G.in.in[b] = m[b].in;
        G.in.elt[b] = m[b].elt;
        G.key[b] = m[b].key->d;
      }
      // the integer launch on the lane's side stream; the stage timer's
      // events on s bracket the fork and the join, so a profiled stage is
      // timed as it runs (both launches overlapped)
      KS_CUDA(modup_rows_inner_product_group(G, L.s_t, m[0].key->limbs, L.s_cx, lv.mu, lv.lay,
                                             T, s, L.side, L.ev_fork, L.ev_join));
      c.launches += (lv.lay.n_slots_fp > 0 ? 1 : 0) + (lv.lay.n_slots_int > 0 ? 1 : 0);
    } else {  // output aggregation with more ranks than digits: a zero partial sum
      for (int b = 0; b < g; ++b)
        KS_CUDA(cudaMemsetAsync(L.s_cx + b * c.st_cx, 0, (size_t)2 * lv.n_out * c.N * 8, s));
    }
  }
  ks_aggregate(c, L, lv, g, s);
  ks_moddown(c, L, lv, m, g, rotate, s, p_rows_done);
}

// One key switch (a group of one).
void keyswitch_core(Ctx &c, Ctx::Lane &L, const Level &lv, const KeyShard &key, const u64 *in_ntt,
                    u64 *ct0, u64 *ct1, const u64 *g0, bool rotate, cudaStream_t s,
                    uint32_t elt = 1) {
  KsMember m;
  m.in = in_ntt;
  m.elt = elt;
  m.key = &key;
  m.ct0 = ct0;
  m.ct1 = ct1;
  m.g0 = g0;
  keyswitch_group(c, L, lv, &m, 1, rotate, s);
}

const Level &level_of(Ctx &c, int Ql) {
  KS_REQUIRE(c.alpha > 0, "context has no special primes (NTT-only context)");
  KS_REQUIRE(Ql >= 1 && Ql <= c.L, "level_limbs out of range");
  return c.levels[Ql];
}

// Rotations of a group of g ciphertexts cts[b] ([2][n_q][N], in place) by
// their Galois elements elts[b], pushed through every launch together.
void do_apply_galois_group(Ctx &c, Ctx::Lane &L, u64 *const *cts, const uint32_t *elts, int g,
                           int Ql, cudaStream_t s) {
  check_alive(c);
  KS_REQUIRE(g >= 1 && g <= c.group, "group larger than the context's scratch");
  const Level &lv = level_of(c, Ql);
  const size_t nq = lv.n_q, N = c.N;
  KsMember m[kMaxGroup];
  MemberIn mi{};
  for (int b = 0; b < g; ++b) {
    u64 *ct = cts[b];
    KS_REQUIRE(aligned16(ct) && (ct != nullptr || nq == 0),
               "ciphertext pointer null or not 16-byte aligned");
    check_elt(c, elts[b]);
    m[b].in = nq ? ct + nq * N : nullptr;
    m[b].elt = elts[b];
    m[b].key = &key_get(c, KS_KEY_GALOIS, elts[b]);
    m[b].ct0 = ct;
    m[b].ct1 = nq ? ct + nq * N : nullptr;
    m[b].g0 = L.s_g + b * c.st_g;
    mi.in[b] = ct;
    mi.elt[b] = elts[b];
  }
  KS_CUDA(cudaSetDevice(c.device));
  // 1. automorphism of every c0 -> g0 (c1 is read through the automorphism by
  //    the input INTT and the inner product; it is overwritten only at the end)
  if (nq > 0) {
    StageTimer tm(c, ST_GALOIS, s);
    KS_CUDA(galois_ntt_group(mi, g, L.s_g, c.st_g, (int)nq, c.log_n, s));
    c.launches += 1;
  }
  keyswitch_group(c, L, lv, m, g, true, s);
}

void do_apply_galois(Ctx &c, Ctx::Lane &L, u64 *ct, int Ql, uint32_t elt, cudaStream_t s) {
  do_apply_galois_group(c, L, &ct, &elt, 1, Ql, s);
}

uint32_t elt_of_step(const Ctx &c, int step) {
  const long long slots = c.N / 2;
  long long st = ((step % slots) + slots) % slots;
  return (uint32_t)h_powmod(3, (u64)st, 2ull * c.N);
}

// Hoisted rotations of one ciphertext ct [2][n_q][N] (not modified):
//   shared by all rotations: INTT of c1, base extension + column pass, and
//   the row pass of every extended limb -> lane 0's t (NTT form);
//   outs != null, rotation i (galois element g_i): the inner product reads the
//     extended digits through the automorphism (k_inner_product with elt g_i),
//     all-reduce (output aggregation), ModDown: outs[i] = (c0 o g_i + ks0, ks1).
//     Rotations run on the lanes round-robin (each lane has its own cx /
//     ModDown scratch and communicator).  This is the hoisting of Halevi-Shoup
//     (decompose and extend once, permute the extended digits per rotation).
//   diags != null (linear transform, double hoisting as in Bossuat et al.,
//     Eurocrypt 2021): every rotation's inner product, plus [P] c0 o g_i on the
//     Q limbs, is multiplied by diags[i] (extended basis, [n_out][N]) and
//     accumulated in lane 0's cx; one all-reduce (output aggregation) and one
//     ModDown at the end: out = sum_i diags[i] * rot_i(ct).
void do_hoisted(Ctx &c, const u64 *ct, int Ql, const int *steps, int n, u64 *const *outs,
                const u64 *const *diags, u64 *out, cudaStream_t s) {
  check_alive(c);
  KS_REQUIRE(aligned16(ct) && (ct != nullptr || n_local(c.rank, c.replicated() ? 1 : c.world, Ql) == 0),
             "ciphertext pointer null or not 16-byte aligned");
  KS_REQUIRE(steps != nullptr && n >= 0, "bad rotation list");
  KS_REQUIRE((outs != nullptr) != (out != nullptr), "give either outs or out");
  const Level &lv = level_of(c, Ql);
  const size_t nq = lv.n_q, N = c.N;
  // a rank that owns no limb of this level passes null buffers
  const bool have_q = nq > 0, have_out = lv.n_out > 0;
  std::vector<uint32_t> elts(n);
  std::vector<const KeyShard *> keys(n);
  for (int i = 0; i < n; ++i) {
    elts[i] = elt_of_step(c, steps[i]);
    keys[i] = &key_get(c, KS_KEY_GALOIS, elts[i]);
    if (outs)
      KS_REQUIRE(aligned16(outs[i]) && (outs[i] != nullptr || !have_q),
                 "output pointer null or misaligned");
    else
      KS_REQUIRE(diags && aligned16(diags[i]) && (diags[i] != nullptr || !have_out),
                 "diagonal pointer null or misaligned");
  }
  KS_CUDA(cudaSetDevice(c.device));
  if (out) KS_CUDA(cudaMemsetAsync(out, 0, 2 * nq * N * 8, s));
  if (n == 0) return;
  const NttTables T = c.tables();
  Ctx::Lane &L0 = c.lanes[0];
  const u64 *c1 = ct + nq * N;
  KsMember m0;
  m0.in = c1;
  ks_modup_cols(c, L0, lv, &m0, 1, s);
  {
    StageTimer tm(c, ST_MODUP_ROWS, s);
    LimbMap mt{L0.s_t, 0, lv.job_off.d, lv.job_prime.d, 0, 1};
    KS_CUDA(ntt_forward_rows_only(mt, lv.n_jobs, T, s));
    c.launches += lv.n_jobs > 0 ? 1 : 0;
  }
  if (!outs) {
    const bool add_c0 = !c.oa() || c.rank == 0;  // the c0 term once over the ranks
    for (int i = 0; i < n; ++i) {
      StageTimer tm(c, ST_INNER_PROD, s);
      if (lv.lay.n_digits > 0) {
        KS_CUDA(inner_product_acc(L0.s_t, c1, keys[i]->d, keys[i]->limbs, L0.s_cx, diags[i], ct,
                                  c.d_pmodq, add_c0, i == 0, lv.mu, lv.lay, c.d_primes,
                                  c.log_n, elts[i], s));
        c.launches += lv.lay.n_out > 0 ? 1 : 0;
      } else if (i == 0) {
        KS_CUDA(cudaMemsetAsync(L0.s_cx, 0, (size_t)2 * lv.n_out * N * 8, s));
      }
    }
    ks_aggregate(c, L0, lv, 1, s);
    KsMember mo;
    mo.ct0 = out;
    mo.ct1 = out + nq * N;
    ks_moddown(c, L0, lv, &mo, 1, true, s);  // rotate without g0: out = ModDown(acc)
    return;
  }
  const int nl = std::min<int>((int)c.lanes.size(), n);
  if (nl > 1) {
    KS_CUDA(cudaEventRecord(c.ev_fork, s));
    for (int li = 1; li < nl; ++li) KS_CUDA(cudaStreamWaitEvent(c.lanes[li].stream, c.ev_fork, 0));
  }
  for (int i = 0; i < n; ++i) {
    const int li = i % nl;
    Ctx::Lane &L = c.lanes[li];
    const cudaStream_t ls = li == 0 ? s : L.stream;
    {
      StageTimer tm(c, ST_GALOIS, ls);
      KS_CUDA(galois_ntt(ct, L.s_g, (int)nq, c.log_n, elts[i], ls));
      c.launches += 1;
    }
    {
      StageTimer tm(c, ST_INNER_PROD, ls);
      if (lv.lay.n_digits > 0) {
        KS_CUDA(inner_product(L0.s_t, c1, keys[i]->d, keys[i]->limbs, L.s_cx, lv.mu, lv.lay,
                              c.d_primes, c.log_n, elts[i], ls));
        c.launches += lv.lay.n_out > 0 ? 1 : 0;
      } else {
        KS_CUDA(cudaMemsetAsync(L.s_cx, 0, (size_t)2 * lv.n_out * N * 8, ls));
      }
    }
    ks_aggregate(c, L, lv, 1, ls);
    KsMember mo;
    mo.ct0 = outs[i];
    mo.ct1 = outs[i] + nq * N;
    mo.g0 = L.s_g;
    ks_moddown(c, L, lv, &mo, 1, true, ls);
  }
  for (int li = 1; li < nl; ++li) {
    KS_CUDA(cudaEventRecord(c.lanes[li].done, c.lanes[li].stream));
    KS_CUDA(cudaStreamWaitEvent(s, c.lanes[li].done, 0));
  }
}

// Rescale by the last prime (Phantom rescale_to_next_inplace, reference
// dist_rescale_to_next_inplace, distributed_eval.cu:265-273, which gathers
// the ciphertext on GPU 0 for it): the owner of limb Ql-1 INTTs it (both
// polys) and, with input broadcast, broadcasts the 2N coefficient words;
// every rank then finishes its own limbs j < Ql-1 with the ModDown column
// and row kernels, q_{Ql-1} playing the special prime:
//   out_j = (ct_j - NTT_j([c + h]_{q_last} mod q_j - [h]_{q_j})) * q_last^-1,  h = q_last / 2.
void do_rescale(Ctx &c, Ctx::Lane &L, const u64 *ct, int Ql, u64 *out, cudaStream_t s) {
  check_alive(c);
  KS_REQUIRE(aligned16(ct) && aligned16(out), "pointers not 16-byte aligned");
  KS_REQUIRE(ct == nullptr || ct != out, "out must not alias ct");
  KS_REQUIRE(Ql >= 2 && Ql <= c.L, "level_limbs must be in [2, L]");
  KS_REQUIRE((ct != nullptr && out != nullptr) ||
                 n_local(c.rank, c.replicated() ? 1 : c.world, Ql) == 0,
             "ciphertext pointers are null");
  const Level &lv = level_of(c, Ql), &lo = level_of(c, Ql - 1);
  const int last = Ql - 1, G = c.replicated() ? 1 : c.world;
  const bool have_last = G == 1 || last % G == c.rank;
  const size_t N = c.N;
  const NttTables T = c.tables();
  const u64 ql = c.primes[last];
  KS_CUDA(cudaSetDevice(c.device));
  u64 *buf = L.s_t;  // [2][N], coefficient form of the last limb
  if (have_last) {
    StageTimer tm(c, ST_INTT_IN, s);
    LimbMap src{const_cast<u64 *>(ct), 0, lv.rs_off.d, lv.rs_prime.d, 0, 1};
    LimbMap dst{buf, (long long)N, nullptr, lv.rs_prime.d, 0, 1};
    KS_CUDA(ntt_inverse_scaled(src, dst, 2, lv.rs_scale, T, s));
    c.launches += 2;
  }
  if (G > 1) {
    StageTimer tm(c, ST_COMM, s);
    enqueue_nccl(c, L.comm, s, [&](ncclComm_t cm) {
      return ncclBroadcast(buf, buf, 2 * N, ncclUint64, last % G, cm, s);
    });
  }
  {
    StageTimer tm(c, ST_MODDOWN_COLS, s);
    KS_CUDA(rescale_fused_cols(buf, ql, ql < kFpBound, L.s_z, lo.n_q, lo.q_index.d, T, s));
    c.launches += lo.n_q > 0 ? 1 : 0;
  }
  {
    StageTimer tm(c, ST_MODDOWN_ROWS, s);
    KS_CUDA(moddown_fused_rows(L.s_z, lo.n_q, lo.q_index.d, lo.cx_slot_q.d, ct,
                               (long long)lv.n_q * N, out, out + (size_t)lo.n_q * N, nullptr,
                               true, nullptr, lv.rs_md, T, s));
    c.launches += lo.n_q > 0 ? 1 : 0;
  }
}

// Words of the BSGS matmul workspace: the baby-step rotations of every input
// and kMacMaxOut giant-step partial sums, each [2][n_q][N].
size_t bsgs_workspace_words(Ctx &c, int Ql, int n_in, int n_baby) {
  const Level &lv = level_of(c, Ql);
  return ((size_t)n_in * (n_baby - 1) + kMacMaxOut) * 2 * lv.n_q * c.N;
}

// Block matrix product by the diagonal method with baby and giant steps
// (Halevi-Shoup diagonals, BSGS split as in Halevi-Shoup 2018):
//   y[o] = sum_{g in [g_lo, g_hi)} rot_{g B u}( sum_{i < n_in} sum_{b < B}
//            pts[((o n_in + i) G + g) B + b] (.) rot_{b u}(x[i]) ),
// B = n_baby, G = n_giant, u = unit.  The baby-step rotations of each input
// share one ModUp (do_hoisted); the plaintext products of up to kMacMaxOut
// giant steps are one k_mac_plain pass over the baby-step ciphertexts; each
// giant-step partial sum g > 0 is rotated by g B u and added to y[o].  The
// product runs limb-locally in every mode; the key switches do their own
// communication.  A giant-step range [g_lo, g_hi) smaller than [0, G) gives a
// partial product (the callers' partition of the giant steps over GPUs).
void do_bsgs_matmul(Ctx &c, const u64 *const *x, const u64 *const *baby, int n_in, int Ql,
                    int unit, int n_baby, int n_giant, int g_lo, int g_hi,
                    const u64 *const *pts, u64 *const *y, int n_out, u64 *work,
                    cudaStream_t s) {
  check_alive(c);
  KS_REQUIRE(x != nullptr && y != nullptr && pts != nullptr, "null pointer list");
  KS_REQUIRE(n_in >= 1 && n_out >= 1 && n_baby >= 1 && n_giant >= 1, "empty matmul shape");
  KS_REQUIRE(0 <= g_lo && g_lo < g_hi && g_hi <= n_giant, "giant-step range out of bounds");
  KS_REQUIRE(unit != 0, "unit rotation step must be nonzero");
  const Level &lv = level_of(c, Ql);
  const int nq = lv.n_q;
  const size_t N = c.N, ct_words = 2 * (size_t)nq * N;
  const bool have = nq > 0;
  for (int i = 0; i < n_in; ++i)
    KS_REQUIRE(aligned16(x[i]) && (x[i] != nullptr || !have), "input pointer null or misaligned");
  for (int o = 0; o < n_out; ++o) {
    KS_REQUIRE(aligned16(y[o]) && (y[o] != nullptr || !have), "output pointer null or misaligned");
    for (int i = 0; i < n_in; ++i) KS_REQUIRE(!have || y[o] != x[i], "an output aliases an input");
    KS_REQUIRE(!have || y[o] != work, "an output aliases the workspace");
    for (int i = 0; i < n_in; ++i)
      for (int g = g_lo; g < g_hi; ++g)
        for (int b = 0; b < n_baby; ++b) {
          const u64 *pt = pts[(((size_t)o * n_in + i) * n_giant + g) * n_baby + b];
          KS_REQUIRE(aligned16(pt) && (pt != nullptr || !have),
                     "plaintext pointer null or misaligned");
        }
  }
  KS_REQUIRE(aligned16(work) && (work != nullptr || !have), "workspace null or misaligned");
  if (baby)
    for (size_t r = 0; r < (size_t)n_in * (n_baby - 1); ++r)
      KS_REQUIRE(aligned16(baby[r]) && (baby[r] != nullptr || !have),
                 "baby-step pointer null or misaligned");
  // every key first, so that a missing one fails before any launch
  std::vector<int> steps(n_baby > 1 && !baby ? n_baby - 1 : 0);
  for (size_t b = 0; b < steps.size(); ++b) steps[b] = (int)(b + 1) * unit;
  for (int st : steps) (void)key_get(c, KS_KEY_GALOIS, elt_of_step(c, st));
  for (int g = std::max(g_lo, 1); g < g_hi; ++g)
    (void)key_get(c, KS_KEY_GALOIS, elt_of_step(c, g * n_baby * unit));
  KS_CUDA(cudaSetDevice(c.device));
  // rot(i, b) = rot_{b u}(x[i]): the caller's (baby != null) or computed into
  // the workspace, b = 1 .. B-1; the partial sums follow the rotations
  u64 *const own = work;
  auto rot = [&](int i, int b) -> const u64 * {
    if (b == 0) return x[i];
    const size_t r = (size_t)i * (n_baby - 1) + (b - 1);
    return baby ? baby[r] : own + r * ct_words;
  };
  u64 *part = work + (baby ? 0 : (size_t)n_in * (n_baby - 1) * ct_words);
  std::vector<u64 *> outs(steps.size());
  for (int i = 0; i < n_in && !steps.empty(); ++i) {
    for (int b = 1; b < n_baby; ++b) outs[b - 1] = const_cast<u64 *>(rot(i, b));
    do_hoisted(c, x[i], Ql, steps.data(), (int)steps.size(), outs.data(), nullptr, nullptr, s);
  }
  const int n_terms = n_in * n_baby;
  KS_REQUIRE(!c.lanes.empty(), "context has no special primes (NTT-only context)");
  Ctx::Lane &L = c.lanes[0];
  const NttTables T = c.tables();
  const bool add_c0 = !c.oa() || c.rank == 0;  // the c0 term once over the ranks
  for (int o = 0; o < n_out; ++o) {
    // g == 0 (if in range) is written straight into y[o] by the first pass;
    // otherwise y[o] starts from zero
    if (g_lo > 0 && have) KS_CUDA(cudaMemsetAsync(y[o], 0, ct_words * 8, s));
    bool acc_open = false;  // lane 0's cx holds this output's giant-step sum
    for (int g0 = g_lo; g0 < g_hi; g0 += kMacMaxOut) {
      const int ng = std::min(kMacMaxOut, g_hi - g0);
      MacTerms a{};
      a.n_out = ng;
      for (int j = 0; j < ng; ++j) a.out[j] = g0 + j == 0 ? y[o] : part + (size_t)j * ct_words;
      {
        StageTimer tm(c, ST_PLAIN_MAC, s);
        for (int m0 = 0; m0 < n_terms; m0 += kMacMaxTerms) {
          a.n_terms = std::min(kMacMaxTerms, n_terms - m0);
          a.accumulate = m0 > 0;
          for (int m = 0; m < a.n_terms; ++m) {
            const int i = (m0 + m) / n_baby, b = (m0 + m) % n_baby;
            a.ct[m] = rot(i, b);
            for (int j = 0; j < ng; ++j)
              a.pt[j][m] = pts[(((size_t)o * n_in + i) * n_giant + g0 + j) * n_baby + b];
          }
          KS_CUDA(mac_plain(a, nq, lv.q_index.d, c.d_primes, c.log_n, s));
          c.launches += have ? 1 : 0;
        }
      }
      // giant steps g > 0: ModUp of the partial sum's c1, then its inner
      // product with the giant step's key, read through the automorphism,
      // plus [P] g(c0), accumulated in the extended basis (lane 0's cx)
      for (int j = 0; j < ng; ++j) {
        const int g = g0 + j;
        if (g == 0) continue;
        const uint32_t elt = elt_of_step(c, g * n_baby * unit);
        const KeyShard &key = key_get(c, KS_KEY_GALOIS, elt);
        const u64 *c1 = have ? a.out[j] + nq * N : nullptr;
        KsMember mi;
        mi.in = c1;
        ks_modup_cols(c, L, lv, &mi, 1, s);
        {
          StageTimer tm(c, ST_MODUP_ROWS, s);
          LimbMap mt{L.s_t, 0, lv.job_off.d, lv.job_prime.d, 0, 1};
          KS_CUDA(ntt_forward_rows_only(mt, lv.n_jobs, T, s));
          c.launches += lv.n_jobs > 0 ? 1 : 0;
        }
        StageTimer tm(c, ST_INNER_PROD, s);
        if (lv.lay.n_digits > 0) {
          KS_CUDA(inner_product_acc(L.s_t, c1, key.d, key.limbs, L.s_cx, nullptr, a.out[j],
                                    c.d_pmodq, add_c0, !acc_open, lv.mu, lv.lay, c.d_primes,
                                    c.log_n, elt, s));
          c.launches += lv.lay.n_out > 0 ? 1 : 0;
        } else if (!acc_open) {
          KS_CUDA(cudaMemsetAsync(L.s_cx, 0, (size_t)2 * lv.n_out * N * 8, s));
        }
        acc_open = true;
      }
    }
    // one ModDown for all giant steps of the output: y[o] += ModDown(acc)
    if (acc_open) {
      ks_aggregate(c, L, lv, 1, s);
      KsMember mo;
      mo.ct0 = y[o];
      mo.ct1 = have ? y[o] + nq * N : nullptr;
      ks_moddown(c, L, lv, &mo, 1, false, s);
    }
  }
}

void do_relin(Ctx &c, Ctx::Lane &L, u64 *ct, int Ql, cudaStream_t s) {
  check_alive(c);
  KS_REQUIRE(aligned16(ct) && (ct != nullptr || n_local(c.rank, c.replicated() ? 1 : c.world, Ql) == 0),
             "ciphertext pointer null or not 16-byte aligned");
  const Level &lv = level_of(c, Ql);
  const KeyShard &key = key_get(c, KS_KEY_RELIN, 0);
  const size_t nq = lv.n_q, N = c.N;
  KS_CUDA(cudaSetDevice(c.device));
  keyswitch_core(c, L, lv, key, ct + 2 * nq * N, ct, ct + nq * N, nullptr, false, s);
}

Ctx::Lane &lane0(Ctx &c) {
  KS_REQUIRE(!c.lanes.empty(), "context has no special primes (NTT-only context)");
  return c.lanes[0];
}


}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int ks_gen_primes(uint32_t log_n, const int *bit_sizes, int n, uint64_t *out) {
  return guarded(nullptr, [&] {
    KS_REQUIRE(bit_sizes && out && n > 0, "bad arguments");
    KS_REQUIRE(log_n >= 1 && log_n <= 20, "log_n out of range");
    if (h_gen_primes((int)log_n, bit_sizes, n, out) != 0)
      throw KsError{KS_ERR_INVALID, "not enough primes of the requested sizes"};
  });
}

int ks_secret_generate(uint32_t log_n, uint64_t seed, int hamming_weight, int8_t *out) {
  // Same specification as the CPU oracle's synthetic secret: uniform ternary
  // (h <= 0) or exactly h nonzero +-1 entries chosen by a partial
  // Fisher-Yates shuffle driven by the counter hash.
  return guarded(nullptr, [&] {
    KS_REQUIRE(out != nullptr && log_n >= 1 && log_n <= 20, "bad arguments");
    const size_t N = (size_t)1 << log_n;
    KS_REQUIRE(hamming_weight <= (int)N, "hamming weight larger than N");
    if (hamming_weight <= 0) {
      for (size_t k = 0; k < N; ++k)
        out[k] = (int8_t)((int)(u64)(((unsigned __int128)prng_at(seed, DOM_SECRET, k) * 3) >> 64) - 1);
      return;
    }
    std::vector<uint32_t> pos(N);
    for (size_t k = 0; k < N; ++k) pos[k] = (uint32_t)k;
    std::memset(out, 0, N);
    for (int i = 0; i < hamming_weight; ++i) {
      const size_t j =
          i + (size_t)(u64)(((unsigned __int128)prng_at(seed, DOM_SECRET, (u64)i) * (N - i)) >> 64);
      std::swap(pos[i], pos[j]);
      out[pos[i]] = (prng_at(seed, DOM_SECRET_SIGN, (u64)i) & 1) ? -1 : 1;
    }
  });
}

int ks_nccl_unique_id(void *out, size_t n) {
  return guarded(nullptr, [&] {
    KS_REQUIRE(out != nullptr && n >= sizeof(ncclUniqueId), "buffer too small for an NCCL id");
    ncclUniqueId id;
    KS_NCCL(ncclGetUniqueId(&id));
    std::memcpy(out, &id, sizeof(id));
  });
}

int ks_ctx_create(const ks_params *prm, int device, int rank, int world, const void *nccl_id,
                  ks_ctx **out) {
  if (!out) {
    set_global_err("out pointer is null");
    return KS_ERR_INVALID;
  }
  *out = nullptr;
  ks_ctx *ctx = new (std::nothrow) ks_ctx();
  if (!ctx) {
    set_global_err("host allocation failed");
    return KS_ERR_ALLOC;
  }
  int rc = guarded(ctx, [&] { ctx_init(ctx->c, prm, device, rank, world, nullptr, nccl_id); });
  if (rc != KS_OK) {
    set_global_err(ctx->c.err);
    ctx_free(ctx->c);
    delete ctx;
    return rc;
  }
  *out = ctx;
  return KS_OK;
}

int ks_ctx_create_all(const ks_params *prm, const int *devices, int n, ks_ctx **outs) {
  if (!outs || !devices || n < 1) {
    set_global_err("bad arguments");
    return KS_ERR_INVALID;
  }
  std::vector<ncclComm_t> comms(n, nullptr);
  if (n > 1) {
    ncclResult_t r = ncclCommInitAll(comms.data(), n, devices);
    if (r != ncclSuccess) {
      set_global_err(std::string("ncclCommInitAll: ") + ncclGetErrorString(r));
      return KS_ERR_NCCL;
    }
  }
  for (int i = 0; i < n; ++i) outs[i] = nullptr;
  for (int i = 0; i < n; ++i) {
    outs[i] = new (std::nothrow) ks_ctx();
    int rc = KS_ERR_ALLOC;
    if (outs[i])
      rc = guarded(outs[i],
                   [&] { ctx_init(outs[i]->c, prm, devices[i], i, n, comms[i], nullptr); });
    else
      set_global_err("host allocation failed");
    if (rc != KS_OK) {
      if (outs[i]) set_global_err(outs[i]->c.err);
      // communicators a failed context did not adopt are destroyed here
      const bool adopted = outs[i] && outs[i]->c.comm == comms[i];
      for (int k = 0; k <= i; ++k) {
        if (!outs[k]) continue;
        ctx_free(outs[k]->c);
        delete outs[k];
        outs[k] = nullptr;
      }
      for (int k = adopted ? i + 1 : i; k < n; ++k)
        if (comms[k]) ncclCommDestroy(comms[k]);
      return rc;
    }
  }
  return KS_OK;
}

int ks_ctx_destroy(ks_ctx *ctx) {
  if (!ctx) return KS_ERR_INVALID;
  ctx_free(ctx->c);
  delete ctx;
  return KS_OK;
}

int ks_last_error(const ks_ctx *ctx, char *buf, size_t n) {
  if (!buf || n == 0) return KS_ERR_INVALID;
  std::string s;
  if (ctx) {
    s = ctx->c.err;
  } else {
    std::lock_guard<std::mutex> lk(g_err_mu);
    s = g_err;
  }
  std::snprintf(buf, n, "%s", s.c_str());
  return KS_OK;
}

int ks_set_timeout_ms(ks_ctx *ctx, int ms) {
  if (!ctx || ms < 0) return KS_ERR_INVALID;
  ctx->c.timeout_ms = ms;
  return KS_OK;
}

int ks_n_local_limbs(const ks_ctx *ctx, int total_limbs) {
  if (!ctx || total_limbs < 0) return KS_ERR_INVALID;
  return n_local(ctx->c.rank, ctx->c.world, total_limbs);
}

int ks_owner_of_limb(const ks_ctx *ctx, int limb) {
  if (!ctx || limb < 0) return KS_ERR_INVALID;
  return limb % ctx->c.world;
}

int ks_num_digits(const ks_ctx *ctx, int level_limbs) {
  if (!ctx || ctx->c.alpha == 0 || level_limbs < 1) return KS_ERR_INVALID;
  return (level_limbs + ctx->c.alpha - 1) / ctx->c.alpha;
}

int ks_galois_elt(const ks_ctx *ctx, int step, uint32_t *elt) {
  if (!ctx || !elt) return KS_ERR_INVALID;
  *elt = elt_of_step(ctx->c, step);
  return KS_OK;
}

size_t ks_key_words(const ks_ctx *ctx) { return ctx ? full_key_words(ctx->c) : 0; }

int ks_key_upload(ks_ctx *ctx, int kind, uint32_t elt, const uint64_t *host_key, size_t n) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] { key_upload(ctx->c, kind, elt, host_key, n, false, 0); });
}

int ks_key_distribute(ks_ctx *ctx, int kind, uint32_t elt, const uint64_t *full_dev, int root,
                      void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    key_distribute(ctx->c, kind, elt, full_dev, root, (cudaStream_t)stream);
  });
}

int ks_key_upload_wire(ks_ctx *ctx, const void *blob, size_t n) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    std::vector<uint64_t> q(c.primes.begin(), c.primes.begin() + c.L),
        p(c.primes.begin() + c.L, c.primes.end());
    const ks_params prm{(uint32_t)c.log_n, c.L, q.data(), c.alpha, p.data(), c.mode, 1};
    int object = 0;
    uint32_t elt = 0;
    if (ks_wire_unpack(&prm, blob, n, &object, &elt, nullptr, nullptr, nullptr, 0) != KS_OK)
      throw KsError{KS_ERR_INVALID, "not a key blob of this context's parameters (or corrupt)"};
    KS_REQUIRE(object == KS_WIRE_RELIN_KEY || object == KS_WIRE_GALOIS_KEY, "blob is not a key");
    const int kind = object == KS_WIRE_RELIN_KEY ? KS_KEY_RELIN : KS_KEY_GALOIS;
    key_upload(c, kind, object == KS_WIRE_RELIN_KEY ? 0u : elt,
               reinterpret_cast<const u64 *>(static_cast<const unsigned char *>(blob) + 64),
               full_key_words(c), false, 0);
  });
}

int ks_key_upload_device(ks_ctx *ctx, int kind, uint32_t elt, const uint64_t *dev_key, size_t n,
                         void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    key_upload(ctx->c, kind, elt, dev_key, n, true, (cudaStream_t)stream);
  });
}

int ks_key_generate(ks_ctx *ctx, int kind, uint32_t elt, const int8_t *secret, uint64_t seed,
                    void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] { key_generate(ctx->c, kind, elt, secret, seed, (cudaStream_t)stream); });
}

int ks_key_download(ks_ctx *ctx, int kind, uint32_t elt, uint64_t *host_key, size_t n) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    const KeyShard &k = key_get(c, kind, elt);
    const size_t words = (size_t)k.beta * 2 * k.limbs * c.N;
    KS_REQUIRE(host_key != nullptr && n >= words, "host buffer too small for the key shard");
    KS_CUDA(cudaSetDevice(c.device));
    KS_CUDA(cudaMemcpy(host_key, k.d, words * 8, cudaMemcpyDeviceToHost));
  });
}

int ks_key_drop(ks_ctx *ctx, int kind, uint32_t elt) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    auto it = ctx->c.keys.find(key_id(kind, elt));
    if (it == ctx->c.keys.end()) throw KsError{KS_ERR_NO_KEY, "no such key"};
    KS_CUDA(cudaSetDevice(ctx->c.device));
    KS_CUDA(cudaFree(it->second.d));
    ctx->c.keys.erase(it);
  });
}

int ks_relinearize(ks_ctx *ctx, uint64_t *ct, int level_limbs, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] { do_relin(ctx->c, lane0(ctx->c), ct, level_limbs, (cudaStream_t)stream); });
}

int ks_keyswitch_add(ks_ctx *ctx, const uint64_t *cin, uint64_t *ct, int level_limbs, int kind,
                     uint32_t elt, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    KS_REQUIRE(aligned16(cin) && aligned16(ct) &&
                   ((cin != nullptr && ct != nullptr) ||
                    n_local(c.rank, c.replicated() ? 1 : c.world, level_limbs) == 0),
               "pointers must be non-null and 16-byte aligned");
    KS_REQUIRE(kind == KS_KEY_RELIN || kind == KS_KEY_GALOIS, "unknown key kind");
    check_alive(c);
    const Level &lv = level_of(c, level_limbs);
    const KeyShard &key = key_get(c, kind, kind == KS_KEY_RELIN ? 0u : elt);
    const size_t nq = lv.n_q, N = c.N;
    KS_CUDA(cudaSetDevice(c.device));
    keyswitch_core(c, lane0(c), lv, key, cin, ct, ct + nq * N, nullptr, false,
                   (cudaStream_t)stream);
  });
}

int ks_apply_galois(ks_ctx *ctx, uint64_t *ct, int level_limbs, uint32_t elt, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    do_apply_galois(ctx->c, lane0(ctx->c), ct, level_limbs, elt, (cudaStream_t)stream);
  });
}

int ks_rotate(ks_ctx *ctx, uint64_t *ct, int level_limbs, int step, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    do_apply_galois(ctx->c, lane0(ctx->c), ct, level_limbs, elt_of_step(ctx->c, step),
                    (cudaStream_t)stream);
  });
}

int ks_rotate_batch(ks_ctx *ctx, uint64_t *const *cts, const int *steps, int n, int level_limbs,
                    void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    KS_REQUIRE(cts != nullptr && steps != nullptr && n >= 0, "bad batch arguments");
    Ctx &c = ctx->c;
    KS_REQUIRE(!c.lanes.empty(), "context has no special primes (NTT-only context)");
    const cudaStream_t s = (cudaStream_t)stream;
    // groups of up to c.group consecutive rotations, spread over the lanes
    const int g = c.group, n_groups = (n + g - 1) / g;
    const int nl = std::min<int>((int)c.lanes.size(), n_groups);
    std::vector<uint32_t> elts(n);
    for (int i = 0; i < n; ++i) elts[i] = elt_of_step(c, steps[i]);
    if (nl <= 1) {
      for (int i0 = 0; i0 < n; i0 += g)
        do_apply_galois_group(c, c.lanes[0], cts + i0, elts.data() + i0, std::min(g, n - i0),
                              level_limbs, s);
      return;
    }
    // fork: every lane waits for the work already queued on the caller's stream
    KS_CUDA(cudaSetDevice(c.device));
    KS_CUDA(cudaEventRecord(c.ev_fork, s));
    for (int li = 1; li < nl; ++li) KS_CUDA(cudaStreamWaitEvent(c.lanes[li].stream, c.ev_fork, 0));
    for (int gi = 0; gi < n_groups; ++gi) {
      const int li = gi % nl, i0 = gi * g;
      cudaStream_t ls = li == 0 ? s : c.lanes[li].stream;
      do_apply_galois_group(c, c.lanes[li], cts + i0, elts.data() + i0, std::min(g, n - i0),
                            level_limbs, ls);
    }
    // join: the caller's stream waits for every lane
    for (int li = 1; li < nl; ++li) {
      KS_CUDA(cudaEventRecord(c.lanes[li].done, c.lanes[li].stream));
      KS_CUDA(cudaStreamWaitEvent(s, c.lanes[li].done, 0));
    }
  });
}

int ks_rescale(ks_ctx *ctx, const uint64_t *ct, int level_limbs, uint64_t *out, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    do_rescale(ctx->c, lane0(ctx->c), ct, level_limbs, out, (cudaStream_t)stream);
  });
}

int ks_rotate_batch_host(ks_ctx *ctx, uint64_t *const *host_cts, const int *steps, int n,
                         int level_limbs, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    KS_REQUIRE(host_cts != nullptr && steps != nullptr && n >= 0, "bad batch arguments");
    Ctx &c = ctx->c;
    KS_REQUIRE(!c.lanes.empty(), "context has no special primes (NTT-only context)");
    const Level &lv = level_of(c, level_limbs);
    const size_t bytes = 2 * (size_t)lv.n_q * c.N * 8;
    const cudaStream_t s = (cudaStream_t)stream;
    // Double buffering: with group >= 2 each lane's staging buffer holds two
    // halves, and the copies in of a lane's next group (on the lane's copy
    // stream) overlap the rotation and copies out of its current one.
    const bool db = c.group >= 2;
    const int g = db ? c.group / 2 : c.group;
    // Group sizes: the copies are the bottleneck of this path, and the first
    // copy out waits for the first group's copies in and rotations, the last
    // rotations for the last copies in; groups of 1, 2, 4 .. at both ends of
    // the batch shorten that fill and drain (the engines stay busy in between).
    std::vector<int> sizes, ramp;
    int ramp_sum = 0;
    for (int r = 1; r < g; r *= 2) {
      ramp.push_back(r);
      ramp_sum += r;
    }
    if (n >= 2 * ramp_sum + g) {
      sizes = ramp;
      int rest = n - 2 * ramp_sum;
      for (; rest >= g; rest -= g) sizes.push_back(g);
      if (rest > 0) sizes.push_back(rest);
      sizes.insert(sizes.end(), ramp.rbegin(), ramp.rend());
    } else {
      for (int i0 = 0; i0 < n; i0 += g) sizes.push_back(std::min(g, n - i0));
    }
    const int n_groups = (int)sizes.size();
    const int nl = std::min<int>((int)c.lanes.size(), std::max(n_groups, 1));
    for (int i = 0; i < n; ++i) KS_REQUIRE(host_cts[i] != nullptr, "host ciphertext pointer is null");
    KS_CUDA(cudaSetDevice(c.device));
    // fork the lanes from the caller's stream; on each lane, per group: copy
    // the members in, rotate them in the lane's staging buffers, copy them
    // out -- the copies of one lane run on the copy engines while the other
    // lanes compute
    KS_CUDA(cudaEventRecord(c.ev_fork, s));
    for (int li = 1; li < nl; ++li) KS_CUDA(cudaStreamWaitEvent(c.lanes[li].stream, c.ev_fork, 0));
    // one in-order stream carries every copy in (lane 0's copy stream): the
    // groups' inputs arrive in batch order, so the last group's copies out
    // do not wait behind the inputs of every lane
    const cudaStream_t cs = db ? c.lanes[0].copy : nullptr;
    if (db) KS_CUDA(cudaStreamWaitEvent(cs, c.ev_fork, 0));
    for (int gi = 0, i0 = 0; gi < n_groups; i0 += sizes[gi], ++gi) {
      const int li = gi % nl, gs = sizes[gi];
      Ctx::Lane &L = c.lanes[li];
      const cudaStream_t ls = li == 0 ? s : L.stream;
      const int h = (gi / nl) & 1;  // staging half of this group (alternates per lane)
      u64 *dev[kMaxGroup];
      uint32_t elts[kMaxGroup];
      const cudaStream_t cin = db ? cs : ls;
      // the half is free once the copies out of the lane's group before last are done
      if (db) KS_CUDA(cudaStreamWaitEvent(cin, L.ev_out[h], 0));
      for (int b = 0; b < gs; ++b) {
        dev[b] = L.s_ct + ((db ? h * g : 0) + b) * c.st_ct;
        elts[b] = elt_of_step(c, steps[i0 + b]);
        KS_CUDA(cudaMemcpyAsync(dev[b], host_cts[i0 + b], bytes, cudaMemcpyHostToDevice, cin));
      }
      if (db) {
        KS_CUDA(cudaEventRecord(L.ev_in[h], cin));
        KS_CUDA(cudaStreamWaitEvent(ls, L.ev_in[h], 0));
      }
      do_apply_galois_group(c, L, dev, elts, gs, level_limbs, ls);
      for (int b = 0; b < gs; ++b)
        KS_CUDA(cudaMemcpyAsync(host_cts[i0 + b], dev[b], bytes, cudaMemcpyDeviceToHost, ls));
      if (db) KS_CUDA(cudaEventRecord(L.ev_out[h], ls));
    }
    for (int li = 1; li < nl; ++li) {
      KS_CUDA(cudaEventRecord(c.lanes[li].done, c.lanes[li].stream));
      KS_CUDA(cudaStreamWaitEvent(s, c.lanes[li].done, 0));
    }
  });
}

int ks_graph_capture_begin(ks_ctx *ctx, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    KS_REQUIRE(stream != nullptr, "graph capture needs a non-default stream");
    KS_REQUIRE(!c.profile, "profiling must be off during graph capture");
    KS_REQUIRE(!c.capturing, "a capture is already open on this context");
    KS_CUDA(cudaSetDevice(c.device));
    KS_CUDA(cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeThreadLocal));
    c.capturing = true;
    c.capture_stream = (cudaStream_t)stream;
  });
}

int ks_graph_capture_end(ks_ctx *ctx, void *stream, ks_graph **out) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    KS_REQUIRE(out != nullptr && stream != nullptr, "bad arguments");
    KS_REQUIRE(c.capturing, "no capture is open on this context");
    KS_REQUIRE((cudaStream_t)stream == c.capture_stream, "not the capturing stream");
    KS_CUDA(cudaSetDevice(c.device));
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture((cudaStream_t)stream, &g);
    c.capturing = false;
    KS_CUDA(e);
    cudaGraphExec_t x = nullptr;
    const cudaError_t e2 = cudaGraphInstantiate(&x, g, 0);
    if (e2 != cudaSuccess) cudaGraphDestroy(g);
    KS_CUDA(e2);
    *out = new ks_graph{g, x, c.device};
  });
}

int ks_graph_launch(ks_graph *graph, void *stream) {
  if (!graph || !graph->exec) return KS_ERR_INVALID;
  return guarded(nullptr, [&] {
    KS_CUDA(cudaSetDevice(graph->device));
    KS_CUDA(cudaGraphLaunch(graph->exec, (cudaStream_t)stream));
  });
}

int ks_graph_destroy(ks_graph *graph) {
  if (!graph) return KS_OK;
  cudaSetDevice(graph->device);
  if (graph->exec) cudaGraphExecDestroy(graph->exec);
  if (graph->graph) cudaGraphDestroy(graph->graph);
  delete graph;
  return KS_OK;
}

int ks_rotate_hoisted(ks_ctx *ctx, const uint64_t *ct, int level_limbs, const int *steps, int n,
                      uint64_t *const *outs, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    KS_REQUIRE(outs != nullptr, "outs is null");
    KS_REQUIRE(!ctx->c.lanes.empty(), "context has no special primes (NTT-only context)");
    do_hoisted(ctx->c, ct, level_limbs, steps, n, outs, nullptr, nullptr, (cudaStream_t)stream);
  });
}

int ks_linear_transform_hoisted(ks_ctx *ctx, const uint64_t *ct, int level_limbs,
                                const int *steps, int n, const uint64_t *const *diags,
                                uint64_t *out, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    KS_REQUIRE(out != nullptr && aligned16(out), "output pointer null or misaligned");
    KS_REQUIRE(out != ct, "out must not alias ct");
    KS_REQUIRE(!ctx->c.lanes.empty(), "context has no special primes (NTT-only context)");
    do_hoisted(ctx->c, ct, level_limbs, steps, n, nullptr, diags, out, (cudaStream_t)stream);
  });
}

size_t ks_bsgs_workspace_words(ks_ctx *ctx, int level_limbs, int n_in, int n_baby) {
  if (!ctx || n_in < 1 || n_baby < 1 || ctx->c.alpha == 0 || level_limbs < 1 ||
      level_limbs > ctx->c.L)
    return 0;
  return bsgs_workspace_words(ctx->c, level_limbs, n_in, n_baby);
}

int ks_bsgs_matmul(ks_ctx *ctx, const uint64_t *const *x, const uint64_t *const *baby,
                   int n_in, int level_limbs, int unit, int n_baby, int n_giant, int g_lo,
                   int g_hi, const uint64_t *const *pts, uint64_t *const *y, int n_out,
                   uint64_t *workspace, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    KS_REQUIRE(!ctx->c.lanes.empty(), "context has no special primes (NTT-only context)");
    do_bsgs_matmul(ctx->c, x, baby, n_in, level_limbs, unit, n_baby, n_giant, g_lo, g_hi, pts,
                   y, n_out, workspace, (cudaStream_t)stream);
  });
}

int ks_reduce_limbs(ks_ctx *ctx, uint64_t *x, int n_polys, int level_limbs, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    const Level &lv = level_of(c, level_limbs);
    KS_REQUIRE(n_polys >= 1, "n_polys must be positive");
    KS_REQUIRE(aligned16(x) && (x != nullptr || lv.n_q == 0), "pointer null or misaligned");
    KS_CUDA(cudaSetDevice(c.device));
    for (int p = 0; p < n_polys && lv.n_q > 0; ++p) {
      KS_CUDA(mod_reduce(x + (size_t)p * lv.n_q * c.N, lv.n_q, lv.q_index.d, c.d_primes,
                         c.log_n, (cudaStream_t)stream));
      c.launches += 1;
    }
  });
}

static int ntt_api(ks_ctx *ctx, uint64_t *data, int n_limbs, int first_prime, int batch,
                   void *stream, bool fwd) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    KS_REQUIRE(data != nullptr && aligned16(data), "data pointer null or not 16-byte aligned");
    KS_REQUIRE(n_limbs >= 1 && batch >= 1, "n_limbs and batch must be positive");
    KS_REQUIRE(first_prime >= 0 && first_prime + n_limbs <= c.K, "prime range out of the basis");
    KS_CUDA(cudaSetDevice(c.device));
    const long long total = (long long)n_limbs * batch;
    const NttTables T = c.tables();
    for (long long off = 0; off < total; off += 65535) {
      const int cnt = (int)std::min<long long>(65535, total - off);
      // keep the prime pattern aligned: chunks start at multiples of n_limbs
      LimbMap m{data + off * c.N, c.N, nullptr, nullptr, first_prime, n_limbs};
      if (off % n_limbs != 0) throw KsError{KS_ERR_UNSUPPORTED, "internal chunking error"};
      KS_CUDA(fwd ? ntt_forward(m, cnt, T, (cudaStream_t)stream)
                  : ntt_inverse(m, cnt, T, (cudaStream_t)stream));
      c.launches += 2;
    }
  });
}

int ks_ntt_forward(ks_ctx *ctx, uint64_t *data, int n_limbs, int first_prime, int batch,
                   void *stream) {
  return ntt_api(ctx, data, n_limbs, first_prime, batch, stream, true);
}
int ks_ntt_inverse(ks_ctx *ctx, uint64_t *data, int n_limbs, int first_prime, int batch,
                   void *stream) {
  return ntt_api(ctx, data, n_limbs, first_prime, batch, stream, false);
}

int ks_scatter_limbs(ks_ctx *ctx, const uint64_t *global_buf, uint64_t *local_buf, int n_polys,
                     int total_limbs, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    KS_REQUIRE(global_buf && local_buf && aligned16(global_buf) && aligned16(local_buf),
               "buffers must be non-null and 16-byte aligned");
    KS_REQUIRE(n_polys >= 0 && total_limbs >= 0, "bad sizes");
    KS_CUDA(cudaSetDevice(c.device));
    KS_CUDA(scatter_limbs(global_buf, local_buf, n_polys, total_limbs, c.log_n, c.rank, c.world,
                          (cudaStream_t)stream));
  });
}

int ks_gather_limbs(ks_ctx *ctx, const uint64_t *local_buf, uint64_t *global_buf, int n_polys,
                    int total_limbs, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    KS_REQUIRE(global_buf && local_buf && aligned16(global_buf) && aligned16(local_buf),
               "buffers must be non-null and 16-byte aligned");
    KS_REQUIRE(n_polys >= 0 && total_limbs >= 0, "bad sizes");
    KS_CUDA(cudaSetDevice(c.device));
    KS_CUDA(gather_limbs(local_buf, global_buf, n_polys, total_limbs, c.log_n, c.rank, c.world,
                         (cudaStream_t)stream));
  });
}

int ks_scatter_ciphertext_to_gpu(const uint64_t *global_buf, uint64_t *local_buf, size_t n_polys,
                                 size_t total_limbs, size_t degree, int gpu_id, int n_gpus,
                                 void *stream) {
  return guarded(nullptr, [&] {
    KS_REQUIRE(n_gpus >= 1 && gpu_id >= 0 && gpu_id < n_gpus, "gpu_id out of range");
    KS_REQUIRE(degree >= 1 && n_polys <= 65535 && total_limbs <= ((size_t)1 << 40),
               "bad sizes");
    if (n_local(gpu_id, n_gpus, (int)std::min<size_t>(total_limbs, 1u << 30)) == 0 || n_polys == 0)
      return;
    KS_REQUIRE(global_buf != nullptr && local_buf != nullptr, "null buffer");
    KS_CUDA(partition_copy(global_buf, local_buf, (long long)n_polys, (long long)total_limbs,
                           (long long)degree, gpu_id, n_gpus, true, (cudaStream_t)stream));
  });
}

int ks_gather_ciphertext_from_gpu(const uint64_t *local_buf, uint64_t *global_buf, size_t n_polys,
                                  size_t total_limbs, size_t degree, int gpu_id, int n_gpus,
                                  void *stream) {
  return guarded(nullptr, [&] {
    KS_REQUIRE(n_gpus >= 1 && gpu_id >= 0 && gpu_id < n_gpus, "gpu_id out of range");
    KS_REQUIRE(degree >= 1 && n_polys <= 65535 && total_limbs <= ((size_t)1 << 40),
               "bad sizes");
    if (n_local(gpu_id, n_gpus, (int)std::min<size_t>(total_limbs, 1u << 30)) == 0 || n_polys == 0)
      return;
    KS_REQUIRE(global_buf != nullptr && local_buf != nullptr, "null buffer");
    KS_CUDA(partition_copy(global_buf, const_cast<uint64_t *>(local_buf), (long long)n_polys,
                           (long long)total_limbs, (long long)degree, gpu_id, n_gpus, false,
                           (cudaStream_t)stream));
  });
}

int ks_allgather_limbs(ks_ctx *ctx, const uint64_t *local_buf, uint64_t *full_buf,
                       int total_limbs, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    KS_REQUIRE(local_buf && full_buf && aligned16(local_buf) && aligned16(full_buf),
               "buffers must be non-null and 16-byte aligned");
    KS_REQUIRE(total_limbs >= 1, "bad sizes");
    KS_CUDA(cudaSetDevice(c.device));
    cudaStream_t s = (cudaStream_t)stream;
    const size_t N = c.N, G = c.world, ml = (total_limbs + G - 1) / G;
    if (G == 1) {
      KS_CUDA(cudaMemcpyAsync(full_buf, local_buf, total_limbs * N * 8, cudaMemcpyDeviceToDevice, s));
      return;
    }
    // pad to ml limbs, gather rank-grouped, then reorder to limb order
    DevBuf<u64> send_buf(ml * N), recv_buf(G * ml * N);
    u64 *send = send_buf.p, *recv = recv_buf.p;
    const int nl = n_local(c.rank, c.world, total_limbs);
    KS_CUDA(cudaMemsetAsync(send, 0, ml * N * 8, s));
    if (nl > 0) KS_CUDA(cudaMemcpyAsync(send, local_buf, nl * N * 8, cudaMemcpyDeviceToDevice, s));
    allgather(c, c.comm, send, recv, ml * N, s);
    // rank-grouped [G][ml] -> sequential: limb j at (j % G, j / G)
    for (int j = 0; j < total_limbs; ++j)
      KS_CUDA(cudaMemcpyAsync(full_buf + (size_t)j * N, recv + ((j % G) * ml + j / G) * N, N * 8,
                              cudaMemcpyDeviceToDevice, s));
    KS_CUDA(cudaStreamSynchronize(s));  // before the staging buffers are freed
  });
}

int ks_last_launch_count(const ks_ctx *ctx) { return ctx ? ctx->c.launches.last : KS_ERR_INVALID; }
long long ks_total_launch_count(const ks_ctx *ctx) {
  return ctx ? ctx->c.launches.total : KS_ERR_INVALID;
}

int ks_profile_enable(ks_ctx *ctx, int on) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.profile = on != 0;
  return KS_OK;
}

int ks_profile_stage_count(void) { return ST_COUNT; }

const char *ks_profile_stage_name(int i) { return (i >= 0 && i < ST_COUNT) ? kStageNames[i] : ""; }

int ks_profile_read(ks_ctx *ctx, double *ms, int *calls, int n) {
  if (!ctx || !ms || !calls || n < ST_COUNT) return KS_ERR_INVALID;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    KS_CUDA(cudaSetDevice(c.device));
    for (int i = 0; i < ST_COUNT; ++i) {
      ms[i] = 0;
      calls[i] = 0;
    }
    for (auto &pe : c.prof_events) {
      KS_CUDA(cudaEventSynchronize(pe.second.second));
      float t = 0;
      KS_CUDA(cudaEventElapsedTime(&t, pe.second.first, pe.second.second));
      ms[pe.first] += t;
      calls[pe.first] += 1;
      c.event_pool.push_back(pe.second.first);
      c.event_pool.push_back(pe.second.second);
    }
    c.prof_events.clear();
  });
}

}  // extern "C"

// ===========================================================================
// Rotation without any allocation on the call
// ===========================================================================
// Some callers may not allocate device memory when they call in: code that
// runs under a fixed memory budget, or a service that reserves every byte of
// HBM up front and hands libraries only the buffers they work on.
// ks_apply_galois_noalloc serves them: the same automorphism + key switch as
// ks_apply_galois, but its scratch comes from the file-scope array below
// (kNoAllocWords words = 16 MiB, held by every GPU that loads the library
// until the process exits) instead of the context's lane arena, and the call
// itself allocates nothing.
namespace {

constexpr size_t kNoAllocWords = (size_t)2 << 20;  // 2 Mi words = 16 MiB
__device__ __align__(256) u64 g_noalloc_scratch[kNoAllocWords];

std::mutex g_noalloc_mu;
std::map<int, u64 *> g_noalloc_addr;  // device -> device address of g_noalloc_scratch

// Device address of the array on the current device (set-up once per device).
// In host code the array's name is only a host-side stand-in, so the address
// must come from cudaGetSymbolAddress with the device current.
u64 *noalloc_base(int device) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  auto it = g_noalloc_addr.find(device);
  if (it != g_noalloc_addr.end()) return it->second;
  void *p = nullptr;
  KS_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
  g_noalloc_addr[device] = static_cast<u64 *>(p);
  return static_cast<u64 *>(p);
}

}  // namespace

extern "C" int ks_apply_galois_noalloc(ks_ctx *ctx, uint64_t *ct, int level_limbs,
                                       uint32_t galois_elt, void *stream) {
  if (!ctx) return KS_ERR_INVALID;
  ctx->c.launches = 0;
  return guarded(ctx, [&] {
    Ctx &c = ctx->c;
    KS_REQUIRE(c.alpha > 0, "context has no special primes (NTT-only context)");
    KS_REQUIRE(c.world == 1, "the allocation-free rotation serves single-GPU contexts only");
    KS_REQUIRE(!c.profile, "disable per-stage profiling before the allocation-free rotation");
    // the lane layout of the context's own arena, laid over the static array:
    // automorphism output, coefficient input, extended digits, cx, z
    const size_t N = c.N, nq = n_local(0, 1, c.L), ml = c.L;
    const Level &top = c.levels[c.L];
    const size_t w_t = std::max((size_t)top.beta * top.n_out * N, 3 * c.own_key.size() * N);
    const size_t need = 2 * nq * N + ml * N + w_t + 2 * (size_t)top.n_out * N + 2 * nq * N;
    if (need > kNoAllocWords)
      throw KsError{KS_ERR_UNSUPPORTED,
                    "parameter set needs " + std::to_string(need * 8) +
                        " bytes of scratch; the allocation-free rotation holds at most " +
                        std::to_string(kNoAllocWords * 8)};
    KS_CUDA(cudaSetDevice(c.device));
    u64 *p = noalloc_base(c.device);
    Ctx::Lane ln;
    ln.comm = nullptr;
    ln.s_g = p; p += 2 * nq * N;
    ln.s_coef = p; p += ml * N;
    ln.s_coef_all = ln.s_coef;
    ln.s_t = p; p += w_t;
    ln.s_cx = p; p += 2 * (size_t)top.n_out * N;
    ln.s_ysend = ln.s_yall = p;
    ln.s_z = p;
    do_apply_galois(c, ln, ct, level_limbs, galois_elt, (cudaStream_t)stream);
  });
}
