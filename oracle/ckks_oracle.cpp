// ckks_oracle.cpp -- CPU restatement of CKKS hybrid key switching.
//
// TEST INFRASTRUCTURE ONLY (see ckks_oracle.h for the parity status and the
// conventions).  Plain C++17 with unsigned __int128; OpenMP over limbs.  The
// arithmetic is written for clarity: every value is kept canonical in
// [0, q) after every step, so the result of each function is a fixed
// mathematical quantity that any correct implementation reproduces bit for bit.
#include "ckks_oracle.h"

#include <algorithm>
#include <cmath>
#include <complex>
#include <cstdlib>
#include <cstring>
#include <map>
#include <stdexcept>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef unsigned __int128 u128;
typedef uint64_t u64;

namespace {

// ---------------------------------------------------------------------------
// Scalar modular arithmetic
// ---------------------------------------------------------------------------
inline u64 mulmod(u64 a, u64 b, u64 q) { return (u64)((u128)a * b % q); }
inline u64 addmod(u64 a, u64 b, u64 q) { u64 s = a + b; return s >= q ? s - q : s; }
inline u64 submod(u64 a, u64 b, u64 q) { return a >= b ? a - b : a + q - b; }
u64 powmod(u64 a, u64 e, u64 q) {
  u64 r = 1 % q;
  a %= q;
  while (e) {
    if (e & 1) r = mulmod(r, a, q);
    a = mulmod(a, a, q);
    e >>= 1;
  }
  return r;
}
u64 invmod(u64 a, u64 q) { return powmod(a, q - 2, q); }  // q prime
// Shoup companion floor(w * 2^64 / q).
inline u64 shoup_pre(u64 w, u64 q) { return (u64)(((u128)w << 64) / q); }
inline u64 shoup_mul(u64 x, u64 w, u64 wp, u64 q) {
  u64 hi = (u64)(((u128)x * wp) >> 64);
  u64 r = x * w - hi * q;
  return r >= q ? r - q : r;
}

bool is_prime_u64(u64 n) {
  if (n < 2) return false;
  static const u64 small[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
  for (u64 p : small) {
    if (n % p == 0) return n == p;
  }
  u64 d = n - 1;
  int s = 0;
  while ((d & 1) == 0) { d >>= 1; ++s; }
  for (u64 a : small) {  // deterministic for n < 3.3e24
    u64 x = powmod(a, d, n);
    if (x == 1 || x == n - 1) continue;
    bool comp = true;
    for (int r = 1; r < s; ++r) {
      x = mulmod(x, x, n);
      if (x == n - 1) { comp = false; break; }
    }
    if (comp) return false;
  }
  return true;
}

inline uint32_t brev(uint32_t x, int bits) {
  uint32_t r = 0;
  for (int i = 0; i < bits; ++i) { r = (r << 1) | (x & 1); x >>= 1; }
  return r;
}

// splitmix64 finaliser (Steele, Lea, Flood 2014) as a counter-based hash.
inline u64 mix64(u64 z) {
  z ^= z >> 30; z *= 0xBF58476D1CE4E5B9ULL;
  z ^= z >> 27; z *= 0x94D049BB133111EBULL;
  z ^= z >> 31;
  return z;
}
inline u64 umulhi(u64 a, u64 b) { return (u64)(((u128)a * b) >> 64); }

enum : u64 {
  DOM_SECRET = 1, DOM_SECRET_SIGN = 2, DOM_KEY_A = 3, DOM_KEY_E = 4,
  DOM_ENC_A = 5, DOM_ENC_E = 6
};

}  // namespace

// ---------------------------------------------------------------------------
// Context
// ---------------------------------------------------------------------------
struct ork_ctx {
  int logn = 0;
  size_t N = 0;
  int L = 0, alpha = 0;
  std::vector<u64> m;  // key basis: L Q primes then alpha P primes
  std::vector<u64> psi;
  std::vector<std::vector<u64>> fw, fwp, iv, ivp;  // psi^brev, psi^-brev (+Shoup)
  std::vector<u64> ninv;
  std::vector<int8_t> dummy;
};

namespace {

u64 minimal_psi(u64 q, size_t N) {
  // A primitive 2N-th root r satisfies r^N == -1.  The minimal one is the
  // smallest value among r^(odd) (SEAL/Phantom convention).
  u64 r = 0;
  for (u64 x = 2; x < q; ++x) {
    u64 c = powmod(x, (q - 1) / (2 * N), q);
    if (powmod(c, N, q) == q - 1) { r = c; break; }
  }
  if (!r) throw std::runtime_error("no 2N-th root");
  u64 r2 = mulmod(r, r, q), cur = r, best = r;
  for (size_t i = 0; i < N; ++i) {
    if (cur < best) best = cur;
    cur = mulmod(cur, r2, q);
  }
  return best;
}

void fwd_one(const ork_ctx *c, u64 *a, int k) {
  // Cooley-Tukey, natural order in, bit-reversed order out (Longa-Naehrig).
  const u64 q = c->m[k];
  const u64 *W = c->fw[k].data(), *Wp = c->fwp[k].data();
  size_t N = c->N, t = N;
  for (size_t mm = 1; mm < N; mm <<= 1) {
    t >>= 1;
    for (size_t i = 0; i < mm; ++i) {
      size_t j1 = 2 * i * t;
      u64 w = W[mm + i], wp = Wp[mm + i];
      for (size_t j = j1; j < j1 + t; ++j) {
        u64 U = a[j], V = shoup_mul(a[j + t], w, wp, q);
        a[j] = addmod(U, V, q);
        a[j + t] = submod(U, V, q);
      }
    }
  }
}

void inv_one(const ork_ctx *c, u64 *a, int k) {
  // Gentleman-Sande, bit-reversed in, natural out; then times N^-1.
  const u64 q = c->m[k];
  const u64 *W = c->iv[k].data(), *Wp = c->ivp[k].data();
  size_t N = c->N, t = 1;
  for (size_t mm = N >> 1; mm >= 1; mm >>= 1) {
    for (size_t i = 0; i < mm; ++i) {
      size_t j1 = 2 * i * t;
      u64 w = W[mm + i], wp = Wp[mm + i];
      for (size_t j = j1; j < j1 + t; ++j) {
        u64 U = a[j], V = a[j + t];
        a[j] = addmod(U, V, q);
        a[j + t] = shoup_mul(submod(U, V, q), w, wp, q);
      }
    }
    t <<= 1;
  }
  u64 ni = c->ninv[k], nip = shoup_pre(ni, q);
  for (size_t j = 0; j < N; ++j) a[j] = shoup_mul(a[j], ni, nip, q);
}

// Key-basis index of limb j of the QlP basis (Q limbs of the level, then P).
// Mirrors the `twr` mapping of output_aggregation.cu:95.
inline int qlp_key_index(const ork_ctx *c, int Ql, int j) {
  return j < Ql ? j : c->L + (j - Ql);
}

std::vector<uint32_t> galois_ntt_perm(const ork_ctx *c, uint32_t elt) {
  size_t N = c->N;
  u64 twoN = 2 * N;
  std::vector<uint32_t> perm(N);
  for (size_t i = 0; i < N; ++i) {
    u64 e = 2ull * brev((uint32_t)i, c->logn) + 1;
    u64 ge = (e * elt) % twoN;
    perm[i] = brev((uint32_t)((ge - 1) / 2), c->logn);
  }
  return perm;
}

// Base-conversion constants for source primes `src` (key indices).
struct BConv {
  std::vector<int> src;
  std::vector<u64> qhat_inv;  // [(B/b_i)^-1]_{b_i}
  // [(B/b_i)]_{c} for a destination prime c (computed on demand)
  u64 qhat_mod(const ork_ctx *c, int i, u64 dst) const {
    u64 r = 1 % dst;
    for (size_t t = 0; t < src.size(); ++t)
      if ((int)t != i) r = mulmod(r, c->m[src[t]] % dst, dst);
    return r;
  }
};

BConv make_bconv(const ork_ctx *c, const std::vector<int> &src) {
  BConv b;
  b.src = src;
  for (size_t i = 0; i < src.size(); ++i) {
    u64 qi = c->m[src[i]];
    u64 prod = 1;
    for (size_t t = 0; t < src.size(); ++t)
      if (t != i) prod = mulmod(prod, c->m[src[t]] % qi, qi);
    b.qhat_inv.push_back(invmod(prod, qi));
  }
  return b;
}

// y[j][k] = sum_i [x_i[k] * qhat_inv_i]_{b_i} * [qhat_i]_{c_j}  mod c_j.
void bconv_apply(const ork_ctx *c, const BConv &b, const u64 *const *x,
                 const std::vector<int> &dst, u64 *const *y) {
  size_t N = c->N, n_in = b.src.size();
#pragma omp parallel for schedule(static)
  for (long jj = 0; jj < (long)dst.size(); ++jj) {
    u64 cj = c->m[dst[jj]];
    std::vector<u64> w(n_in);
    for (size_t i = 0; i < n_in; ++i) w[i] = b.qhat_mod(c, (int)i, cj);
    std::vector<u64> v(n_in);
    for (size_t k = 0; k < N; ++k) {
      u128 acc = 0;
      for (size_t i = 0; i < n_in; ++i) {
        u64 qi = c->m[b.src[i]];
        u64 vi = mulmod(x[i][k], b.qhat_inv[i], qi);
        acc += (u128)vi * w[i];
      }
      y[jj][k] = (u64)(acc % cj);
    }
  }
}

void ntt_batch(const ork_ctx *c, u64 *data, int n, const int *idx, bool forward) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    if (forward) fwd_one(c, data + (size_t)i * c->N, idx[i]);
    else inv_one(c, data + (size_t)i * c->N, idx[i]);
  }
}

double gauss_cdf_scale() { return 9223372036854775808.0; }  // 2^63

}  // namespace

// ---------------------------------------------------------------------------
// C API
// ---------------------------------------------------------------------------
extern "C" {

int ork_is_prime(uint64_t v) { return is_prime_u64(v) ? 1 : 0; }

int ork_gen_primes(uint32_t log_n, const int *bits, int n, uint64_t *out) {
  // Phantom/SEAL CoeffModulus::Create: for each bit size b, the largest primes
  // q < 2^b with q ≡ 1 (mod 2N), found by stepping down from 2^b - 2N + 1;
  // within one bit size the smaller primes are assigned first (KAT:
  // ckks_bench.txt:11 gives (8192,{60,40,60}) -> 1152921504606748673,
  // 1099511480321, 1152921504606830593).
  u64 factor = 2ull << log_n;
  std::map<int, int> count;
  for (int i = 0; i < n; ++i) count[bits[i]]++;
  std::map<int, std::vector<u64>> found;  // descending
  for (auto &kv : count) {
    int b = kv.first;
    if (b < 2 || b > 61) return -1;
    u64 v = ((1ull << b) - 1) / factor * factor + 1;
    u64 lower = 1ull << (b - 1);
    std::vector<u64> ps;
    while ((int)ps.size() < kv.second && v > lower) {
      if (is_prime_u64(v)) ps.push_back(v);
      v -= factor;
    }
    if ((int)ps.size() < kv.second) return -1;
    found[b] = ps;
  }
  for (int i = 0; i < n; ++i) {
    auto &ps = found[bits[i]];
    out[i] = ps.back();
    ps.pop_back();
  }
  return 0;
}

ork_ctx *ork_create(uint32_t log_n, const uint64_t *q, int L, const uint64_t *p, int alpha) {
  ork_ctx *c = new ork_ctx();
  c->logn = (int)log_n;
  c->N = (size_t)1 << log_n;
  c->L = L;
  c->alpha = alpha;
  for (int i = 0; i < L; ++i) c->m.push_back(q[i]);
  for (int i = 0; i < alpha; ++i) c->m.push_back(p[i]);
  size_t K = c->m.size(), N = c->N;
  c->psi.resize(K);
  c->fw.resize(K); c->fwp.resize(K); c->iv.resize(K); c->ivp.resize(K);
  c->ninv.resize(K);
  for (size_t k = 0; k < K; ++k) {
    u64 qk = c->m[k];
    u64 psi = minimal_psi(qk, N), psii = invmod(psi, qk);
    c->psi[k] = psi;
    std::vector<u64> pw(N), pwi(N);
    pw[0] = 1; pwi[0] = 1;
    for (size_t i = 1; i < N; ++i) { pw[i] = mulmod(pw[i - 1], psi, qk); pwi[i] = mulmod(pwi[i - 1], psii, qk); }
    c->fw[k].resize(N); c->fwp[k].resize(N); c->iv[k].resize(N); c->ivp[k].resize(N);
    for (size_t i = 0; i < N; ++i) {
      uint32_t r = brev((uint32_t)i, c->logn);
      c->fw[k][i] = pw[r]; c->fwp[k][i] = shoup_pre(pw[r], qk);
      c->iv[k][i] = pwi[r]; c->ivp[k][i] = shoup_pre(pwi[r], qk);
    }
    c->ninv[k] = invmod(N % qk, qk);
  }
  return c;
}

void ork_destroy(ork_ctx *c) { delete c; }

void ork_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
int ork_get_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

int ork_num_digits(const ork_ctx *c, int Ql) { return (Ql + c->alpha - 1) / c->alpha; }
uint64_t ork_psi(const ork_ctx *c, int k) { return c->psi[k]; }

void ork_ntt_forward(const ork_ctx *c, uint64_t *d, int n, const int *idx) { ntt_batch(c, d, n, idx, true); }
void ork_ntt_inverse(const ork_ctx *c, uint64_t *d, int n, const int *idx) { ntt_batch(c, d, n, idx, false); }

uint32_t ork_galois_elt(const ork_ctx *c, int step) {
  // Left rotation by `step` slots: X -> X^(3^step mod 2N); the generator 3
  // has order N/2 modulo 2N, so negative steps wrap modulo N/2.
  long slots = (long)(c->N / 2);
  long s = ((step % slots) + slots) % slots;
  return (uint32_t)powmod(3, (u64)s, 2 * c->N);
}

void ork_galois_ntt(const ork_ctx *c, uint32_t elt, const uint64_t *in, uint64_t *out, int n) {
  auto perm = galois_ntt_perm(c, elt);
  size_t N = c->N;
  for (int l = 0; l < n; ++l)
    for (size_t i = 0; i < N; ++i) out[l * N + i] = in[l * N + perm[i]];
}

void ork_galois_coeff(const ork_ctx *c, uint32_t elt, const uint64_t *in, uint64_t *out,
                      int n, const int *idx) {
  size_t N = c->N;
  u64 twoN = 2 * N;
  for (int l = 0; l < n; ++l) {
    u64 q = c->m[idx[l]];
    for (size_t i = 0; i < N; ++i) {
      u64 e = ((u64)i * elt) % twoN;
      u64 v = in[l * N + i];
      if (e >= N) out[l * N + (e - N)] = v ? q - v : 0;
      else out[l * N + e] = v;
    }
  }
}

void ork_bconv(const ork_ctx *c, const uint64_t *in, const int *in_idx, int n_in,
               uint64_t *out, const int *out_idx, int n_out) {
  BConv b = make_bconv(c, std::vector<int>(in_idx, in_idx + n_in));
  std::vector<const u64 *> x(n_in);
  for (int i = 0; i < n_in; ++i) x[i] = in + (size_t)i * c->N;
  std::vector<u64 *> y(n_out);
  for (int j = 0; j < n_out; ++j) y[j] = out + (size_t)j * c->N;
  bconv_apply(c, b, x.data(), std::vector<int>(out_idx, out_idx + n_out), y.data());
}

// ModUp (Phantom DRNSTool::modup, called at output_aggregation.cu:240):
//   INTT the Ql limbs; for digit d with Q limbs D = [d*alpha, min((d+1)*alpha, Ql)):
//   t[d][j] = c[j] (NTT form) for j in D, else NTT_j(bconv_{D->j}(INTT(c)_D)).
void ork_modup(const ork_ctx *c, const uint64_t *in, int Ql, uint64_t *t) {
  size_t N = c->N;
  int QlP = Ql + c->alpha, beta = ork_num_digits(c, Ql);
  std::vector<u64> coef(in, in + (size_t)Ql * N);
  std::vector<int> idxQ(Ql);
  for (int j = 0; j < Ql; ++j) idxQ[j] = j;
  ntt_batch(c, coef.data(), Ql, idxQ.data(), false);
  for (int d = 0; d < beta; ++d) {
    int lo = d * c->alpha, hi = std::min(Ql, lo + c->alpha);
    std::vector<int> src;
    std::vector<const u64 *> x;
    for (int j = lo; j < hi; ++j) { src.push_back(j); x.push_back(coef.data() + (size_t)j * N); }
    BConv b = make_bconv(c, src);
    std::vector<int> dst, dst_local;
    std::vector<u64 *> y;
    u64 *td = t + (size_t)d * QlP * N;
    for (int j = 0; j < QlP; ++j) {
      if (j >= lo && j < hi) {
        std::memcpy(td + (size_t)j * N, in + (size_t)j * N, N * 8);
      } else {
        dst.push_back(qlp_key_index(c, Ql, j));
        dst_local.push_back(j);
        y.push_back(td + (size_t)j * N);
      }
    }
    bconv_apply(c, b, x.data(), dst, y.data());
#pragma omp parallel for schedule(static)
    for (long jj = 0; jj < (long)dst.size(); ++jj) fwd_one(c, y[jj], dst[jj]);
  }
}

// Inner product (output_aggregation.cu:73-126 with all digits on one device):
//   cx[p][j][k] = sum_d t[d][j][k] * key[d][p][twr(j)][k]  mod m_twr(j).
void ork_inner_product(const ork_ctx *c, const uint64_t *t, int Ql, const uint64_t *key,
                       uint64_t *cx) {
  size_t N = c->N;
  int QlP = Ql + c->alpha, beta = ork_num_digits(c, Ql), KP = c->L + c->alpha;
#pragma omp parallel for schedule(static)
  for (int j = 0; j < QlP; ++j) {
    int tw = qlp_key_index(c, Ql, j);
    u64 q = c->m[tw];
    for (int p = 0; p < 2; ++p) {
      for (size_t k = 0; k < N; ++k) {
        u128 acc = 0;
        for (int d = 0; d < beta; ++d) {
          u64 a = t[((size_t)d * QlP + j) * N + k];
          u64 e = key[(((size_t)d * 2 + p) * KP + tw) * N + k];
          acc += (u128)a * e;  // beta * q^2 < 2^128 for q < 2^61, beta < 64
        }
        cx[((size_t)p * QlP + j) * N + k] = (u64)(acc % q);
      }
    }
  }
}

// ModDown (Phantom moddown_from_NTT, output_aggregation.cu:278-282):
//   y = INTT(cx_P); z_j = NTT_j(bconv_{P->q_j}(y)); out_j = (cx_j - z_j) * P^-1 mod q_j.
void ork_moddown(const ork_ctx *c, const uint64_t *cx, int Ql, uint64_t *out) {
  size_t N = c->N;
  int a = c->alpha;
  std::vector<u64> y(cx + (size_t)Ql * N, cx + (size_t)(Ql + a) * N);
  std::vector<int> pidx(a);
  for (int i = 0; i < a; ++i) pidx[i] = c->L + i;
  ntt_batch(c, y.data(), a, pidx.data(), false);
  BConv b = make_bconv(c, pidx);
  std::vector<const u64 *> x(a);
  for (int i = 0; i < a; ++i) x[i] = y.data() + (size_t)i * N;
  std::vector<int> dst(Ql);
  std::vector<u64 *> z(Ql);
  for (int j = 0; j < Ql; ++j) { dst[j] = j; z[j] = out + (size_t)j * N; }
  bconv_apply(c, b, x.data(), dst, z.data());
#pragma omp parallel for schedule(static)
  for (int j = 0; j < Ql; ++j) {
    u64 q = c->m[j];
    fwd_one(c, z[j], j);
    u64 P = 1;
    for (int i = 0; i < a; ++i) P = mulmod(P, c->m[c->L + i] % q, q);
    u64 Pinv = invmod(P, q);
    for (size_t k = 0; k < N; ++k)
      z[j][k] = mulmod(submod(cx[(size_t)j * N + k], z[j][k], q), Pinv, q);
  }
}

void ork_keyswitch(const ork_ctx *c, const uint64_t *in, int Ql, const uint64_t *key, uint64_t *out) {
  size_t N = c->N;
  int QlP = Ql + c->alpha, beta = ork_num_digits(c, Ql);
  std::vector<u64> t((size_t)beta * QlP * N), cx((size_t)2 * QlP * N);
  ork_modup(c, in, Ql, t.data());
  ork_inner_product(c, t.data(), Ql, key, cx.data());
  for (int p = 0; p < 2; ++p)
    ork_moddown(c, cx.data() + (size_t)p * QlP * N, Ql, out + (size_t)p * Ql * N);
}

static void add_inplace(const ork_ctx *c, u64 *a, const u64 *b, int Ql) {
  size_t N = c->N;
  for (int j = 0; j < Ql; ++j)
    for (size_t k = 0; k < N; ++k) a[j * N + k] = addmod(a[j * N + k], b[j * N + k], c->m[j]);
}

// Rotation / apply_galois (Phantom apply_galois_inplace, input_broadcast.cu:200):
//   (c0, c1) -> (pi(c0) + ks0(pi(c1)), ks1(pi(c1))).
void ork_apply_galois(const ork_ctx *c, const uint64_t *ct, int Ql, uint32_t elt,
                      const uint64_t *key, uint64_t *out) {
  size_t N = c->N, QN = (size_t)Ql * N;
  std::vector<u64> g(2 * QN), ks(2 * QN);
  ork_galois_ntt(c, elt, ct, g.data(), 2 * Ql);
  ork_keyswitch(c, g.data() + QN, Ql, key, ks.data());
  std::memcpy(out, g.data(), QN * 8);
  add_inplace(c, out, ks.data(), Ql);
  std::memcpy(out + QN, ks.data() + QN, QN * 8);
}

// Relinearisation (Phantom keyswitch_inplace(is_relin=true), input_broadcast.cu:172):
//   (c0, c1, c2) -> (c0 + ks0(c2), c1 + ks1(c2)).
void ork_relinearize(const ork_ctx *c, const uint64_t *ct, int Ql, const uint64_t *key,
                     uint64_t *out) {
  size_t QN = (size_t)Ql * c->N;
  std::vector<u64> ks(2 * QN);
  ork_keyswitch(c, ct + 2 * QN, Ql, key, ks.data());
  std::memcpy(out, ct, 2 * QN * 8);
  add_inplace(c, out, ks.data(), Ql);
  add_inplace(c, out + QN, ks.data() + QN, Ql);
}

// Hoisted rotations: ModUp(c1) once; for each rotation permute the extended
// digits (the automorphism commutes with the base extension, being a
// per-limb index permutation in the NTT domain), then inner product + ModDown.
void ork_rotate_hoisted(const ork_ctx *c, const uint64_t *ct, int Ql, int n,
                        const uint32_t *elts, const uint64_t *const *keys, uint64_t *out) {
  size_t N = c->N, QN = (size_t)Ql * N;
  int QlP = Ql + c->alpha, beta = ork_num_digits(c, Ql);
  std::vector<u64> t((size_t)beta * QlP * N), tg(t.size()), cx((size_t)2 * QlP * N);
  ork_modup(c, ct + QN, Ql, t.data());
  for (int r = 0; r < n; ++r) {
    ork_galois_ntt(c, elts[r], t.data(), tg.data(), beta * QlP);
    ork_inner_product(c, tg.data(), Ql, keys[r], cx.data());
    u64 *o = out + (size_t)r * 2 * QN;
    std::vector<u64> ks(2 * QN);
    for (int p = 0; p < 2; ++p)
      ork_moddown(c, cx.data() + (size_t)p * QlP * N, Ql, ks.data() + (size_t)p * QN);
    ork_galois_ntt(c, elts[r], ct, o, Ql);
    add_inplace(c, o, ks.data(), Ql);
    std::memcpy(o + QN, ks.data() + QN, QN * 8);
  }
}

// Rescale by the last prime (Phantom rescale_to_next_inplace, called by the
// reference's dist_rescale_to_next_inplace, distributed_eval.cu:265-273; the
// SEAL/Phantom divide-and-round of the RNS literature):
//   c = INTT_{q_last}(ct_last) + floor(q_last / 2)  (mod q_last), per poly;
//   out_j = (ct_j - NTT_j([c]_{q_j} - [floor(q_last / 2)]_{q_j})) * q_last^-1  mod q_j,
// j < Ql - 1: out = round(ct / q_last) at level Ql - 1.
void ork_rescale(const ork_ctx *c, const uint64_t *ct, int Ql, uint64_t *out) {
  size_t N = c->N;
  const int last = Ql - 1;
  const u64 ql = c->m[last], half = ql >> 1;
  for (int p = 0; p < 2; ++p) {
    std::vector<u64> v(ct + ((size_t)p * Ql + last) * N, ct + ((size_t)p * Ql + last + 1) * N);
    int li = last;
    ntt_batch(c, v.data(), 1, &li, false);
    for (size_t k = 0; k < N; ++k) v[k] = addmod(v[k], half, ql);
#pragma omp parallel for schedule(static)
    for (int j = 0; j < last; ++j) {
      const u64 q = c->m[j], hj = half % q, inv = invmod(ql % q, q);
      std::vector<u64> t(N);
      for (size_t k = 0; k < N; ++k) t[k] = submod(v[k] % q, hj, q);
      int jj = j;
      ntt_batch(c, t.data(), 1, &jj, true);
      const u64 *src = ct + ((size_t)p * Ql + j) * N;
      u64 *dst = out + ((size_t)p * last + j) * N;
      for (size_t k = 0; k < N; ++k) dst[k] = mulmod(submod(src[k], t[k], q), inv, q);
    }
  }
}

// Hoisted linear transform with one ModDown ("double hoisting", Bossuat,
// Mouchet, Troncoso-Pastoriza, Hubaux, Eurocrypt 2021; the reference has no
// counterpart -- its bootstrapping lives in the absent NEXUS Bootstrapper):
//   t = ModUp(c1) once; for each rotation r (element g_r):
//     acc_0 += d_r * (IP_0(g_r(t), key_r) + [P]_{q_j} g_r(c0))   (Q limbs; P limbs: no c0)
//     acc_1 += d_r * IP_1(g_r(t), key_r)
//   out_p = ModDown(acc_p).
// d_r: the plaintext diagonal in the extended basis, [Ql + alpha][N] NTT form
// (Q limbs, then the alpha P limbs).  P * x has zero residues mod every p_i,
// so ModDown(P * x + y) = x + ModDown(y) exactly: out = sum_r d_r * rot_r(ct)
// up to the rounding of one ModDown instead of one per rotation.
void ork_linear_transform_hoisted(const ork_ctx *c, const uint64_t *ct, int Ql, int n,
                                  const uint32_t *elts, const uint64_t *const *keys,
                                  const uint64_t *const *diags, uint64_t *out) {
  size_t N = c->N, QN = (size_t)Ql * N;
  int QlP = Ql + c->alpha, beta = ork_num_digits(c, Ql);
  std::vector<u64> t((size_t)beta * QlP * N), tg(t.size()), cx((size_t)2 * QlP * N);
  std::vector<u64> acc((size_t)2 * QlP * N, 0), g0(QN);
  std::vector<u64> Pq(Ql);
  for (int j = 0; j < Ql; ++j) {
    u64 P = 1;
    for (int i = 0; i < c->alpha; ++i) P = mulmod(P, c->m[c->L + i] % c->m[j], c->m[j]);
    Pq[j] = P;
  }
  ork_modup(c, ct + QN, Ql, t.data());
  for (int r = 0; r < n; ++r) {
    ork_galois_ntt(c, elts[r], t.data(), tg.data(), beta * QlP);
    ork_inner_product(c, tg.data(), Ql, keys[r], cx.data());
    ork_galois_ntt(c, elts[r], ct, g0.data(), Ql);
#pragma omp parallel for schedule(static)
    for (int j = 0; j < QlP; ++j) {
      u64 q = c->m[qlp_key_index(c, Ql, j)];
      for (int p = 0; p < 2; ++p)
        for (size_t k = 0; k < N; ++k) {
          u64 v = cx[((size_t)p * QlP + j) * N + k];
          if (p == 0 && j < Ql) v = addmod(v, mulmod(Pq[j], g0[(size_t)j * N + k], q), q);
          u64 &a = acc[((size_t)p * QlP + j) * N + k];
          a = addmod(a, mulmod(diags[r][(size_t)j * N + k], v, q), q);
        }
    }
  }
  for (int p = 0; p < 2; ++p) ork_moddown(c, acc.data() + (size_t)p * QlP * N, Ql, out + (size_t)p * QN);
}

// Ciphertext x plaintext block matrix product by the diagonal method with baby
// and giant steps (Halevi-Shoup).  The reference has no counterpart: NEXUS's
// matmul is absent, and the reference describes it as multiply_plain +
// add_many + rescale per output column (src/benchmarks/bert_matmul_pipeline.cu:7-15).
//   y[o] = sum_{g in [g_lo, g_hi)} rot_g( sum_{i < n_in} sum_{b < B}
//            pts[((o n_in + i) G + g) B + b] * rot_b(x[i]) )
// rot_b (0 < b < B): baby_elts[b - 1] by ork_rotate_hoisted (one ModUp per
// input); plaintext products and sums limb by limb mod q_j.  The giant steps
// g > 0 of one output share one ModDown, as the hoisted linear transform's
// rotations do: each partial sum s_g gets its own ModUp and inner product
// with the key of giant_elts[g], read through the automorphism, and
//   acc_0 += IP_0 + [P]_{q_j} g(s_g.c0) (Q limbs),  acc_1 += IP_1,
// then y[o] += ModDown(acc).  ModDown(P x + v) = x + ModDown(v) exactly, so
// this is sum_g rot_g(s_g) up to the rounding of one ModDown per output
// instead of one per giant step (the rounding depends on which giant steps
// one call covers: a split over [g_lo, g_hi) ranges rounds per range).
void ork_bsgs_matmul(const ork_ctx *c, const uint64_t *const *x, int n_in, int Ql, int B,
                     int G, int g_lo, int g_hi, const uint32_t *baby_elts,
                     const uint64_t *const *baby_keys, const uint32_t *giant_elts,
                     const uint64_t *const *giant_keys, const uint64_t *const *pts, int n_out,
                     uint64_t *const *y) {
  const size_t N = c->N, QN = (size_t)Ql * N, CT = 2 * QN;
  std::vector<u64> rots((size_t)n_in * B * CT);
  for (int i = 0; i < n_in; ++i) {
    std::memcpy(rots.data() + (size_t)i * B * CT, x[i], CT * 8);
    if (B > 1)
      ork_rotate_hoisted(c, x[i], Ql, B - 1, baby_elts, baby_keys,
                         rots.data() + ((size_t)i * B + 1) * CT);
  }
  const int QlP = Ql + c->alpha, beta = ork_num_digits(c, Ql);
  std::vector<u64> inner(CT), t((size_t)beta * QlP * N), tg(t.size()), cx((size_t)2 * QlP * N);
  std::vector<u64> acc((size_t)2 * QlP * N), g0(QN), ks(CT), Pq(Ql);
  for (int j = 0; j < Ql; ++j) {
    u64 P = 1;
    for (int i = 0; i < c->alpha; ++i) P = mulmod(P, c->m[c->L + i] % c->m[j], c->m[j]);
    Pq[j] = P;
  }
  for (int o = 0; o < n_out; ++o) {
    std::memset(y[o], 0, CT * 8);
    std::fill(acc.begin(), acc.end(), 0);
    bool any_giant = false;
    for (int g = g_lo; g < g_hi; ++g) {
      std::fill(inner.begin(), inner.end(), 0);
      for (int i = 0; i < n_in; ++i)
        for (int b = 0; b < B; ++b) {
          const u64 *pt = pts[(((size_t)o * n_in + i) * G + g) * B + b];
          const u64 *r = rots.data() + ((size_t)i * B + b) * CT;
#pragma omp parallel for schedule(static)
          for (int j = 0; j < Ql; ++j) {
            const u64 q = c->m[j];
            for (int p = 0; p < 2; ++p)
              for (size_t k = 0; k < N; ++k) {
                u64 &a = inner[(size_t)p * QN + (size_t)j * N + k];
                a = addmod(a, mulmod(pt[(size_t)j * N + k], r[(size_t)p * QN + (size_t)j * N + k], q), q);
              }
          }
        }
      if (g == 0) {
        add_inplace(c, y[o], inner.data(), Ql);
        add_inplace(c, y[o] + QN, inner.data() + QN, Ql);
        continue;
      }
      any_giant = true;
      ork_modup(c, inner.data() + QN, Ql, t.data());
      ork_galois_ntt(c, giant_elts[g], t.data(), tg.data(), beta * QlP);
      ork_inner_product(c, tg.data(), Ql, giant_keys[g], cx.data());
      ork_galois_ntt(c, giant_elts[g], inner.data(), g0.data(), Ql);
#pragma omp parallel for schedule(static)
      for (int j = 0; j < QlP; ++j) {
        const u64 q = c->m[qlp_key_index(c, Ql, j)];
        for (int p = 0; p < 2; ++p)
          for (size_t k = 0; k < N; ++k) {
            u64 v = cx[((size_t)p * QlP + j) * N + k];
            if (p == 0 && j < Ql) v = addmod(v, mulmod(Pq[j], g0[(size_t)j * N + k], q), q);
            u64 &a = acc[((size_t)p * QlP + j) * N + k];
            a = addmod(a, v, q);
          }
      }
    }
    if (any_giant) {
      for (int p = 0; p < 2; ++p)
        ork_moddown(c, acc.data() + (size_t)p * QlP * N, Ql, ks.data() + (size_t)p * QN);
      add_inplace(c, y[o], ks.data(), Ql);
      add_inplace(c, y[o] + QN, ks.data() + QN, Ql);
    }
  }
}

// ---------------------------------------------------------------------------
// Deterministic sampling (synthetic keys and ciphertexts; NOT a secure RNG)
// ---------------------------------------------------------------------------
uint64_t ork_prng(uint64_t seed, uint64_t domain, uint64_t idx) {
  u64 key = mix64(seed ^ mix64(domain + 0x9E3779B97F4A7C15ULL));
  return mix64(key + (idx + 1) * 0x9E3779B97F4A7C15ULL);
}

void ork_gauss_table(uint64_t *T) {
  // Cumulative distribution of |e| for the discrete Gaussian with sigma 3.2,
  // support |e| <= 19, as thresholds on a 63-bit uniform value.
  const double sigma = 3.2;
  double rho[20], Z = 0;
  for (int x = 0; x < 20; ++x) {
    rho[x] = std::exp(-(double)x * x / (2 * sigma * sigma));
    Z += (x == 0 ? 1.0 : 2.0) * rho[x];
  }
  double cum = 0;
  for (int x = 0; x < 20; ++x) {
    cum += (x == 0 ? 1.0 : 2.0) * rho[x];
    T[x] = (x == 19) ? (1ull << 63) : (u64)(cum / Z * gauss_cdf_scale());
  }
}

namespace {
struct GaussTable {
  u64 T[20];
  GaussTable() { ork_gauss_table(T); }
};
}  // namespace

int ork_gauss(uint64_t r) {
  static const GaussTable tbl;  // thread-safe one-time initialisation
  const u64 *T = tbl.T;
  u64 u = r >> 1;
  int k = 0;
  while (k < 19 && u >= T[k]) ++k;
  return (r & 1) ? -k : k;
}

void ork_secret(const ork_ctx *c, uint64_t seed, int h, int8_t *s) {
  size_t N = c->N;
  if (h <= 0) {
    for (size_t k = 0; k < N; ++k) s[k] = (int8_t)((int)umulhi(ork_prng(seed, DOM_SECRET, k), 3) - 1);
    return;
  }
  std::vector<uint32_t> pos(N);
  for (size_t k = 0; k < N; ++k) pos[k] = (uint32_t)k;
  std::memset(s, 0, N);
  for (int i = 0; i < h; ++i) {
    size_t j = i + (size_t)umulhi(ork_prng(seed, DOM_SECRET, (u64)i), N - i);
    std::swap(pos[i], pos[j]);
    s[pos[i]] = (ork_prng(seed, DOM_SECRET_SIGN, (u64)i) & 1) ? -1 : 1;
  }
}

void ork_secret_ntt(const ork_ctx *c, const int8_t *s, int n, uint64_t *out) {
  size_t N = c->N;
  std::vector<int> idx(n);
  for (int j = 0; j < n; ++j) {
    idx[j] = j;
    u64 q = c->m[j];
    for (size_t k = 0; k < N; ++k) out[j * N + k] = s[k] >= 0 ? (u64)s[k] : q - (u64)(-s[k]);
  }
  ntt_batch(c, out, n, idx.data(), true);
}

static void keygen_common(const ork_ctx *c, const int8_t *s, const u64 *snew, uint64_t seed,
                          uint64_t *key) {
  // key[d][0][j] = -a_d s + e_d + [j in digit d] * [P]_{q_j} * s'   (mod m_j)
  // key[d][1][j] = a_d                     (all values in NTT form)
  size_t N = c->N;
  int K = c->L + c->alpha, beta = ork_num_digits(c, c->L);
  std::vector<u64> sn((size_t)K * N);
  ork_secret_ntt(c, s, K, sn.data());
  std::vector<int> idx(K);
  for (int j = 0; j < K; ++j) idx[j] = j;
  for (int d = 0; d < beta; ++d) {
    std::vector<u64> e((size_t)K * N);
    for (size_t k = 0; k < N; ++k) {
      int ev = ork_gauss(ork_prng(seed, DOM_KEY_E, (u64)d * N + k));
      for (int j = 0; j < K; ++j) e[j * N + k] = ev >= 0 ? (u64)ev : c->m[j] - (u64)(-ev);
    }
    ntt_batch(c, e.data(), K, idx.data(), true);
#pragma omp parallel for schedule(static)
    for (int j = 0; j < K; ++j) {
      u64 q = c->m[j];
      u64 Pq = 1;
      for (int i = 0; i < c->alpha; ++i) Pq = mulmod(Pq, c->m[c->L + i] % q, q);
      bool in_digit = j < c->L && j / c->alpha == d;
      u64 *b = key + (((size_t)d * 2 + 0) * K + j) * N;
      u64 *a = key + (((size_t)d * 2 + 1) * K + j) * N;
      for (size_t k = 0; k < N; ++k) {
        u64 av = umulhi(ork_prng(seed, DOM_KEY_A, ((u64)d * K + j) * N + k), q);
        a[k] = av;
        u64 v = submod(e[j * N + k], mulmod(av, sn[j * N + k], q), q);
        if (in_digit) v = addmod(v, mulmod(Pq, snew[j * N + k], q), q);
        b[k] = v;
      }
    }
  }
}

void ork_keygen_galois(const ork_ctx *c, const int8_t *s, uint32_t elt, uint64_t seed, uint64_t *key) {
  size_t N = c->N;
  int L = c->L;
  std::vector<u64> sn((size_t)L * N), sg((size_t)L * N);
  ork_secret_ntt(c, s, L, sn.data());
  ork_galois_ntt(c, elt, sn.data(), sg.data(), L);
  keygen_common(c, s, sg.data(), seed, key);
}

void ork_keygen_relin(const ork_ctx *c, const int8_t *s, uint64_t seed, uint64_t *key) {
  size_t N = c->N;
  int L = c->L;
  std::vector<u64> sn((size_t)L * N);
  ork_secret_ntt(c, s, L, sn.data());
  for (int j = 0; j < L; ++j)
    for (size_t k = 0; k < N; ++k) sn[j * N + k] = mulmod(sn[j * N + k], sn[j * N + k], c->m[j]);
  keygen_common(c, s, sn.data(), seed, key);
}

// ---------------------------------------------------------------------------
// CKKS encode / decode (host doubles, libm) and symmetric encryption
// ---------------------------------------------------------------------------
namespace {
typedef std::complex<double> cd;

// X_k = sum_n x_n exp(sign * 2 pi i n k / N), radix-2 iterative.
void fft(std::vector<cd> &a, int sign) {
  size_t n = a.size();
  int lg = 0;
  while ((1ull << lg) < n) ++lg;
  for (size_t i = 0; i < n; ++i) {
    size_t r = brev((uint32_t)i, lg);
    if (i < r) std::swap(a[i], a[r]);
  }
  for (size_t len = 2; len <= n; len <<= 1) {
    double ang = sign * 2 * M_PI / (double)len;
    for (size_t i = 0; i < n; i += len) {
      for (size_t j = 0; j < len / 2; ++j) {
        cd w = std::polar(1.0, ang * (double)j);
        cd u = a[i + j], v = a[i + j + len / 2] * w;
        a[i + j] = u + v;
        a[i + j + len / 2] = u - v;
      }
    }
  }
}
}  // namespace

void ork_encode(const ork_ctx *c, const double *re, const double *im, int n_slots, double scale,
                int Ql, uint64_t *pt) {
  std::vector<int> idx(Ql);
  for (int j = 0; j < Ql; ++j) idx[j] = j;
  ork_encode_basis(c, re, im, n_slots, scale, idx.data(), Ql, pt);
}

// Same encoding into the primes idx[0..n_idx) of the key basis (Q primes,
// then P primes): pt [n_idx][N], NTT form.
void ork_encode_basis(const ork_ctx *c, const double *re, const double *im, int n_slots,
                      double scale, const int *key_idx, int n_idx, uint64_t *pt) {
  size_t N = c->N, slots = N / 2;
  std::vector<cd> V(N, cd(0, 0));
  u64 e = 1, twoN = 2 * N;
  for (size_t j = 0; j < slots; ++j) {
    cd z = (int)j < n_slots ? cd(re[j], im ? im[j] : 0.0) : cd(0, 0);
    V[(e - 1) / 2] = z;
    V[(twoN - e - 1) / 2] = std::conj(z);
    e = (e * 3) % twoN;
  }
  fft(V, -1);
  std::vector<long long> coef(N);
  for (size_t n = 0; n < N; ++n) {
    cd x = V[n] / (double)N * std::polar(1.0, -M_PI * (double)n / (double)N);
    coef[n] = std::llround(x.real() * scale);
  }
  std::vector<int> idx(key_idx, key_idx + n_idx);
  for (int j = 0; j < n_idx; ++j) {
    u64 q = c->m[idx[j]];
    for (size_t n = 0; n < N; ++n) {
      long long v = coef[n];
      pt[j * N + n] = v >= 0 ? (u64)v % q : (q - ((u64)(-v) % q)) % q;
    }
  }
  ntt_batch(c, pt, n_idx, idx.data(), true);
}

void ork_decode(const ork_ctx *c, const uint64_t *pt, int Ql, double scale, double *re, double *im,
                int n_slots) {
  size_t N = c->N;
  int use = Ql >= 2 ? 2 : 1;
  std::vector<u64> x(pt, pt + (size_t)use * N);
  std::vector<int> idx = {0, 1};
  ntt_batch(c, x.data(), use, idx.data(), false);
  std::vector<cd> V(N);
  u64 q0 = c->m[0];
  for (size_t n = 0; n < N; ++n) {
    double val;
    if (use == 1) {
      u64 v = x[n];
      val = v > q0 / 2 ? -(double)(q0 - v) : (double)v;
    } else {
      u64 q1 = c->m[1];
      u64 x0 = x[n], x1 = x[N + n];
      u64 t = mulmod(submod(x1 % q1, x0 % q1, q1), invmod(q0 % q1, q1), q1);
      u128 X = (u128)x0 + (u128)q0 * t, Q = (u128)q0 * q1;
      val = X > Q / 2 ? -(double)(Q - X) : (double)X;
    }
    V[n] = cd(val / scale, 0) * std::polar(1.0, M_PI * (double)n / (double)N);
  }
  fft(V, +1);
  u64 e = 1, twoN = 2 * N;
  for (int j = 0; j < n_slots && (size_t)j < N / 2; ++j) {
    cd z = V[(e - 1) / 2];
    re[j] = z.real();
    if (im) im[j] = z.imag();
    e = (e * 3) % twoN;
  }
}

void ork_encrypt(const ork_ctx *c, const int8_t *s, const uint64_t *pt, int Ql, uint64_t seed,
                 uint64_t *ct) {
  // c1 = a (uniform, NTT form), c0 = -a*s + e + pt.
  size_t N = c->N, QN = (size_t)Ql * N;
  std::vector<u64> sn(QN), e(QN);
  ork_secret_ntt(c, s, Ql, sn.data());
  std::vector<int> idx(Ql);
  for (size_t k = 0; k < N; ++k) {
    int ev = ork_gauss(ork_prng(seed, DOM_ENC_E, k));
    for (int j = 0; j < Ql; ++j) e[j * N + k] = ev >= 0 ? (u64)ev : c->m[j] - (u64)(-ev);
  }
  for (int j = 0; j < Ql; ++j) idx[j] = j;
  ntt_batch(c, e.data(), Ql, idx.data(), true);
  for (int j = 0; j < Ql; ++j) {
    u64 q = c->m[j];
    for (size_t k = 0; k < N; ++k) {
      u64 a = umulhi(ork_prng(seed, DOM_ENC_A, (u64)j * N + k), q);
      ct[QN + j * N + k] = a;
      u64 v = submod(e[j * N + k], mulmod(a, sn[j * N + k], q), q);
      ct[j * N + k] = addmod(v, pt[j * N + k], q);
    }
  }
}

void ork_decrypt(const ork_ctx *c, const int8_t *s, const uint64_t *ct, int n_polys, int Ql,
                 uint64_t *pt) {
  size_t N = c->N, QN = (size_t)Ql * N;
  std::vector<u64> sn(QN);
  ork_secret_ntt(c, s, Ql, sn.data());
  for (int j = 0; j < Ql; ++j) {
    u64 q = c->m[j];
    for (size_t k = 0; k < N; ++k) {
      size_t i = j * N + k;
      u64 spow = sn[i], acc = ct[i];
      for (int p = 1; p < n_polys; ++p) {
        acc = addmod(acc, mulmod(ct[p * QN + i], spow, q), q);
        spow = mulmod(spow, sn[i], q);
      }
      pt[i] = acc;
    }
  }
}

void ork_multiply(const ork_ctx *c, const uint64_t *a, const uint64_t *b, int Ql, uint64_t *out) {
  size_t N = c->N, QN = (size_t)Ql * N;
  for (int j = 0; j < Ql; ++j) {
    u64 q = c->m[j];
    for (size_t k = 0; k < N; ++k) {
      size_t i = j * N + k;
      out[i] = mulmod(a[i], b[i], q);
      out[QN + i] = addmod(mulmod(a[i], b[QN + i], q), mulmod(a[QN + i], b[i], q), q);
      out[2 * QN + i] = mulmod(a[QN + i], b[QN + i], q);
    }
  }
}

double ork_ks_noise_log2(const ork_ctx *c, const int8_t *s, const uint64_t *in,
                         const uint64_t *snew, const uint64_t *ks, int Ql) {
  // d = ks0 + ks1*s - in*s'  on limb 0, back to coefficients, max |centered|.
  size_t N = c->N, QN = (size_t)Ql * N;
  std::vector<u64> sn(N);
  ork_secret_ntt(c, s, 1, sn.data());
  u64 q = c->m[0];
  std::vector<u64> d(N);
  for (size_t k = 0; k < N; ++k) {
    u64 v = addmod(ks[k], mulmod(ks[QN + k], sn[k], q), q);
    d[k] = submod(v, mulmod(in[k], snew[k], q), q);
  }
  int idx0 = 0;
  ntt_batch(c, d.data(), 1, &idx0, false);
  double mx = 0;
  for (size_t k = 0; k < N; ++k) {
    double v = d[k] > q / 2 ? (double)(q - d[k]) : (double)d[k];
    mx = std::max(mx, v);
  }
  return mx > 0 ? std::log2(mx) : 0.0;
}

}  // extern "C"
