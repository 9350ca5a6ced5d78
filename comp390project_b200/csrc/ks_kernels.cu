// ks_kernels.cu -- automorphism, the standalone inner products of the
// hoisted path, the post-all-reduce reduction, partition copies and the
// synthetic-key samplers (sm_100a).  The fused ModUp / ModDown kernels live
// in ks_fused.cu.
//
// All kernels stream 128-bit words (two coefficients per thread per access)
// and keep per-limb constants in registers; the limb index of a CTA is
// blockIdx.y so every constant load is warp-uniform.
#include "ks_kernels.cuh"
#include "ks_galois.cuh"

namespace ksb {
namespace {

constexpr int kBlk = 256;

__device__ __forceinline__ u64 mix64(u64 z) {
  z ^= z >> 30;
  z *= 0xBF58476D1CE4E5B9ull;
  z ^= z >> 27;
  z *= 0x94D049BB133111EBull;
  z ^= z >> 31;
  return z;
}

// One thread: the output pair (2m, 2m + 1) from the aligned source pair.
// Member b of a group (grid z) reads mi.in[b] through mi.elt[b] and writes
// out + b out_bstride (mi.in[0] null: in, elt).
__global__ void k_galois_ntt(const u64 *__restrict__ in, u64 *__restrict__ out, int log_n,
                             uint32_t elt, const __grid_constant__ MemberIn mi,
                             long long out_bstride) {
  const int N = 1 << log_n;
  const long long limb = blockIdx.y;
  if (mi.in[0]) {
    in = mi.in[blockIdx.z];
    elt = mi.elt[blockIdx.z];
  }
  out += blockIdx.z * out_bstride;
  const uint32_t i = (blockIdx.x * kBlk + threadIdx.x) * 2;
  if (i >= (uint32_t)N) return;
  const uint32_t src = galois_src(i, elt, log_n);
  ulonglong2 v = __ldg(reinterpret_cast<const ulonglong2 *>(in + limb * N + (src & ~1u)));
  if (src & 1u) {
    const u64 t = v.x;
    v.x = v.y;
    v.y = t;
  }
  *reinterpret_cast<ulonglong2 *>(out + limb * N + i) = v;
}

// Inner product of the automorphism X -> X^elt of the extended digits for
// the two adjacent output slots (k, k+1) of output limb s, both polys
// (canonical).  The pair reads the aligned source pair galois_src(k) & ~1 (the
// two sources are galois_src(k) and its neighbour galois_src(k) ^ 1), so every
// warp still reads whole 256-byte segments.  Keys are streamed (__ldcs) so the
// extended digits stay in L2 across calls.
struct IpPair {
  ulonglong2 r0, r1;
};
__device__ __forceinline__ IpPair ip_pair(const u64 *__restrict__ t, const u64 *__restrict__ c_ntt,
                                          const u64 *__restrict__ key, int key_limbs,
                                          const ModUpDev &mu, const KsLayout &lay,
                                          const PrimeDev &P, int N, int s, int k, uint32_t sbase,
                                          bool swap) {
  const int j = lay.out_j[s];
  const long long ks = lay.key_slot[s];
  const int dj = j < mu.Ql ? j / mu.alpha : -1;  // digit holding limb j
  u128v a00 = {0, 0}, a01 = {0, 0}, a10 = {0, 0}, a11 = {0, 0};
  const long long kstride = (long long)key_limbs * N;
  for (int di = 0; di < lay.n_digits; ++di) {
    const int d = lay.digits[di];
    const u64 *T = (d == dj) ? c_ntt + (long long)lay.c_slot[s] * N
                             : t + ((long long)d * lay.n_out + s) * N;
    ulonglong2 x = *reinterpret_cast<const ulonglong2 *>(T + sbase);
    if (swap) {
      const u64 tmp = x.x;
      x.x = x.y;
      x.y = tmp;
    }
    const u64 *kb = key + (long long)(2 * di) * kstride + ks * N + k;
    const ulonglong2 b = __ldcs(reinterpret_cast<const ulonglong2 *>(kb));
    const ulonglong2 a = __ldcs(reinterpret_cast<const ulonglong2 *>(kb + kstride));
    mac(a00, x.x, b.x);
    mac(a01, x.y, b.y);
    mac(a10, x.x, a.x);
    mac(a11, x.y, a.y);
  }
  IpPair r;
  r.r0.x = barrett128(a00, P.q, P.br_hi, P.br_lo);
  r.r0.y = barrett128(a01, P.q, P.br_hi, P.br_lo);
  r.r1.x = barrett128(a10, P.q, P.br_hi, P.br_lo);
  r.r1.y = barrett128(a11, P.q, P.br_hi, P.br_lo);
  return r;
}

// One thread: two adjacent output slots of one output limb, both polys.
__global__ void __launch_bounds__(kBlk) k_inner_product(const u64 *__restrict__ t,
                                                       const u64 *__restrict__ c_ntt,
                                                       const u64 *__restrict__ key,
                                                       int key_limbs, u64 *__restrict__ cx,
                                                       ModUpDev mu, KsLayout lay,
                                                       const PrimeDev *primes, int log_n,
                                                       uint32_t elt) {
  const int N = 1 << log_n;
  const int s = blockIdx.y;
  const int k = (blockIdx.x * kBlk + threadIdx.x) * 2;
  if (k >= N) return;
  const PrimeDev P = primes[mu.prime_of[lay.out_j[s]]];
  const uint32_t src = galois_src((uint32_t)k, elt, log_n);
  const IpPair r = ip_pair(t, c_ntt, key, key_limbs, mu, lay, P, N, s, k, src & ~1u, src & 1u);
  *reinterpret_cast<ulonglong2 *>(cx + (long long)s * N + k) = r.r0;
  *reinterpret_cast<ulonglong2 *>(cx + ((long long)lay.n_out + s) * N + k) = r.r1;
}

// Linear-transform accumulation in the extended basis (double hoisting):
//   acc[0][s] (+)= diag[s] * (ip0 + [P]_{q_j} * c0[galois_src])   (Q limbs; c0 term if add_c0)
//   acc[1][s] (+)= diag[s] * ip1
// first: acc starts at zero instead of being read.
__global__ void __launch_bounds__(kBlk) k_inner_product_acc(
    const u64 *__restrict__ t, const u64 *__restrict__ c_ntt, const u64 *__restrict__ key,
    int key_limbs, u64 *__restrict__ acc, const u64 *__restrict__ diag,
    const u64 *__restrict__ c0, const ulonglong2 *__restrict__ pmodq, int add_c0, int first,
    ModUpDev mu, KsLayout lay, const PrimeDev *primes, int log_n, uint32_t elt) {
  const int N = 1 << log_n;
  const int s = blockIdx.y;
  const int k = (blockIdx.x * kBlk + threadIdx.x) * 2;
  if (k >= N) return;
  const int j = lay.out_j[s];
  const PrimeDev P = primes[mu.prime_of[j]];
  const uint32_t src = galois_src((uint32_t)k, elt, log_n);
  const uint32_t sbase = src & ~1u;
  const bool swap = (src & 1u) != 0;
  IpPair r = ip_pair(t, c_ntt, key, key_limbs, mu, lay, P, N, s, k, sbase, swap);
  if (add_c0 && j < mu.Ql) {
    ulonglong2 x = *reinterpret_cast<const ulonglong2 *>(c0 + (long long)lay.c_slot[s] * N + sbase);
    if (swap) {
      const u64 tmp = x.x;
      x.x = x.y;
      x.y = tmp;
    }
    const ulonglong2 pq = pmodq[j];
    r.r0.x = add_mod(r.r0.x, mul_shoup(x.x, pq.x, pq.y, P.q), P.q);
    r.r0.y = add_mod(r.r0.y, mul_shoup(x.y, pq.x, pq.y, P.q), P.q);
  }
  u64 *a0 = acc + (long long)s * N + k;
  u64 *a1 = acc + ((long long)lay.n_out + s) * N + k;
  ulonglong2 v0 = first ? make_ulonglong2(0, 0) : *reinterpret_cast<const ulonglong2 *>(a0);
  ulonglong2 v1 = first ? make_ulonglong2(0, 0) : *reinterpret_cast<const ulonglong2 *>(a1);
  if (diag) {
    const ulonglong2 dg = *reinterpret_cast<const ulonglong2 *>(diag + (long long)s * N + k);
    v0.x = mac_reduce(v0.x, r.r0.x, dg.x, P.q, P.br_hi, P.br_lo);
    v0.y = mac_reduce(v0.y, r.r0.y, dg.y, P.q, P.br_hi, P.br_lo);
    v1.x = mac_reduce(v1.x, r.r1.x, dg.x, P.q, P.br_hi, P.br_lo);
    v1.y = mac_reduce(v1.y, r.r1.y, dg.y, P.q, P.br_hi, P.br_lo);
  } else {  // no plaintext factor: a plain sum of rotations
    v0.x = add_mod(v0.x, r.r0.x, P.q);
    v0.y = add_mod(v0.y, r.r0.y, P.q);
    v1.x = add_mod(v1.x, r.r1.x, P.q);
    v1.y = add_mod(v1.y, r.r1.y, P.q);
  }
  *reinterpret_cast<ulonglong2 *>(a0) = v0;
  *reinterpret_cast<ulonglong2 *>(a1) = v1;
}

__global__ void k_mod_reduce(u64 *x, const int *prime_of_slot, const PrimeDev *primes,
                             int log_n) {
  const int N = 1 << log_n;
  const int l = blockIdx.y;
  const int k = blockIdx.x * kBlk + threadIdx.x;
  if (k >= N) return;
  const PrimeDev &P = primes[prime_of_slot[l]];
  u64 &v = x[(long long)l * N + k];
  v = reduce_full(v, P.q, P.mu);
}

// One thread: two adjacent coefficients of one limb slot l, both polys, every
// output j < NG (the outputs share the ciphertext terms, which are read once):
//   out_j[p][l] (+)= sum_m pt_j,m[l] * ct_m[p][l]  mod q   (p = 0, 1).
// 128-bit accumulation, Barrett-reduced every 8 terms: 8 products of words
// below 2^62 plus one residue stay below 2^128.
template <int NG>
__global__ void __launch_bounds__(kBlk, NG >= 3 ? 2 : 3) k_mac_plain(const MacTerms a, int n_limbs,
                                                   const int *__restrict__ prime_of_slot,
                                                   const PrimeDev *primes, int log_n) {
  const int N = 1 << log_n;
  const int l = blockIdx.y;
  const int k = (blockIdx.x * kBlk + threadIdx.x) * 2;
  if (k >= N) return;
  const PrimeDev &P = primes[prime_of_slot[l]];
  const u64 q = P.q, rh = P.br_hi, rl = P.br_lo;
  const long long lo = (long long)l * N + k, stride = (long long)n_limbs * N;
  u128v acc[NG][4];  // [output][poly 0 even, poly 0 odd, poly 1 even, poly 1 odd]
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    if (a.accumulate) {
      const ulonglong2 y0 = *reinterpret_cast<const ulonglong2 *>(a.out[j] + lo);
      const ulonglong2 y1 = *reinterpret_cast<const ulonglong2 *>(a.out[j] + stride + lo);
      acc[j][0] = {y0.x, 0};
      acc[j][1] = {y0.y, 0};
      acc[j][2] = {y1.x, 0};
      acc[j][3] = {y1.y, 0};
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[j][i] = {0, 0};
    }
  }
  for (int m = 0; m < a.n_terms; ++m) {
    const ulonglong2 x0 = *reinterpret_cast<const ulonglong2 *>(a.ct[m] + lo);
    const ulonglong2 x1 = *reinterpret_cast<const ulonglong2 *>(a.ct[m] + stride + lo);
#pragma unroll
    for (int j = 0; j < NG; ++j) {
      const ulonglong2 w = *reinterpret_cast<const ulonglong2 *>(a.pt[j][m] + lo);
      mac(acc[j][0], x0.x, w.x);
      mac(acc[j][1], x0.y, w.y);
      mac(acc[j][2], x1.x, w.x);
      mac(acc[j][3], x1.y, w.y);
    }
    if ((m & 7) == 7) {
#pragma unroll
      for (int j = 0; j < NG; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = {barrett128(acc[j][i], q, rh, rl), 0};
    }
  }
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    *reinterpret_cast<ulonglong2 *>(a.out[j] + lo) =
        make_ulonglong2(barrett128(acc[j][0], q, rh, rl), barrett128(acc[j][1], q, rh, rl));
    *reinterpret_cast<ulonglong2 *>(a.out[j] + stride + lo) =
        make_ulonglong2(barrett128(acc[j][2], q, rh, rl), barrett128(acc[j][3], q, rh, rl));
  }
}

// Cyclic-partition copy between the global layout [poly][total][degree]
// and rank g's local layout [poly][n_local][degree] (global limb loc*G + g at
// local slot loc, loc < n_local); to_local picks the direction.  VEC: the
// degree is even and both bases are 16-byte aligned, so every limb starts on
// a 16-byte boundary and each thread moves one ulonglong2.
template <bool VEC>
__global__ void k_scatter(const u64 *__restrict__ gbuf, u64 *__restrict__ lbuf, long long total,
                          long long n_local, long long degree, int g, int G, int to_local) {
  const long long poly = blockIdx.z, loc = blockIdx.y;
  const long long k = ((long long)blockIdx.x * kBlk + threadIdx.x) * (VEC ? 2 : 1);
  if (k >= degree) return;
  const long long glimb = loc * G + g;
  u64 *gp = const_cast<u64 *>(gbuf) + (poly * total + glimb) * degree + k;
  u64 *lp = lbuf + (poly * n_local + loc) * degree + k;
  if (VEC) {
    ulonglong2 *a = reinterpret_cast<ulonglong2 *>(gp), *b = reinterpret_cast<ulonglong2 *>(lp);
    if (to_local) *b = *a;
    else *a = *b;
  } else {
    if (to_local) *lp = *gp;
    else *gp = *lp;
  }
}

__global__ void k_keygen(u64 *key_b, u64 *key_a, const u64 *__restrict__ s_ntt,
                         const u64 *__restrict__ snew_ntt, const u64 *__restrict__ e_ntt,
                         const int *key_index, const int *prime_of_slot, const int *in_digit,
                         const u64 *p_mod_q, u64 key_a_stream, int d, int K,
                         const PrimeDev *primes, int log_n) {
  const int N = 1 << log_n;
  const int l = blockIdx.y;
  const int k = blockIdx.x * kBlk + threadIdx.x;
  if (k >= N) return;
  const PrimeDev P = primes[prime_of_slot[l]];
  const long long o = (long long)l * N + k;
  const u64 idx = ((u64)d * K + (u64)key_index[l]) * N + k;
  const u64 r = mix64(key_a_stream + (idx + 1) * 0x9E3779B97F4A7C15ull);
  const u64 a = __umul64hi(r, P.q);
  u128v prod = {0, 0};
  mac(prod, a, s_ntt[o]);
  const u64 as = barrett128(prod, P.q, P.br_hi, P.br_lo);
  u64 v = sub_mod(e_ntt[o], as, P.q);
  if (in_digit[l]) {
    u128v g = {0, 0};
    mac(g, p_mod_q[l], snew_ntt[o]);
    v = add_mod(v, barrett128(g, P.q, P.br_hi, P.br_lo), P.q);
  }
  key_a[o] = a;
  key_b[o] = v;
}

__global__ void k_gauss(u64 *e, const int *prime_of_slot, const PrimeDev *primes,
                        const u64 *__restrict__ table, u64 stream, u64 idx0, int log_n) {
  const int N = 1 << log_n;
  const int l = blockIdx.y;
  const int k = blockIdx.x * kBlk + threadIdx.x;
  if (k >= N) return;
  const u64 r = mix64(stream + (idx0 + k + 1) * 0x9E3779B97F4A7C15ull);
  const u64 u = r >> 1;
  int mag = 0;
  while (mag < 19 && u >= table[mag]) ++mag;
  const u64 q = primes[prime_of_slot[l]].q;
  u64 v = (u64)mag;
  if ((r & 1) && mag) v = q - v;
  e[(long long)l * N + k] = v;
}

__global__ void k_ternary(const int8_t *s, u64 *out, const int *prime_of_slot,
                          const PrimeDev *primes, int log_n) {
  const int N = 1 << log_n;
  const int l = blockIdx.y;
  const int k = blockIdx.x * kBlk + threadIdx.x;
  if (k >= N) return;
  const u64 q = primes[prime_of_slot[l]].q;
  const int v = s[k];
  out[(long long)l * N + k] = v >= 0 ? (u64)v : q - (u64)(-v);
}

__global__ void k_mul(const u64 *a, const u64 *b, u64 *out, const int *prime_of_slot,
                      const PrimeDev *primes, int log_n) {
  const int N = 1 << log_n;
  const int l = blockIdx.y;
  const int k = blockIdx.x * kBlk + threadIdx.x;
  if (k >= N) return;
  const PrimeDev P = primes[prime_of_slot[l]];
  const long long o = (long long)l * N + k;
  u128v p = {0, 0};
  mac(p, a[o], b[o]);
  out[o] = barrett128(p, P.q, P.br_hi, P.br_lo);
}

inline dim3 grid2(int log_n, int y, int per_thread) {
  const int N = 1 << log_n;
  return dim3((N / per_thread + kBlk - 1) / kBlk, y);
}

}  // namespace

cudaError_t galois_ntt(const u64 *in, u64 *out, int n_limbs, int log_n, uint32_t elt,
                       cudaStream_t s) {
  if (n_limbs <= 0) return cudaSuccess;
  const MemberIn none{};
  k_galois_ntt<<<grid2(log_n, n_limbs, 2), kBlk, 0, s>>>(in, out, log_n, elt, none, 0);
  return cudaGetLastError();
}

cudaError_t galois_ntt_group(const MemberIn &mi, int group, u64 *out, long long out_bstride,
                             int n_limbs, int log_n, cudaStream_t s) {
  if (group < 1 || group > kMaxGroup) return cudaErrorInvalidValue;
  for (int b = 0; b < group; ++b)
    if (!mi.in[b] || !(mi.elt[b] & 1u) || mi.elt[b] >= (2u << log_n)) return cudaErrorInvalidValue;
  if (n_limbs <= 0) return cudaSuccess;
  dim3 g = grid2(log_n, n_limbs, 2);
  g.z = group;
  k_galois_ntt<<<g, kBlk, 0, s>>>(nullptr, out, log_n, 1, mi, out_bstride);
  return cudaGetLastError();
}

cudaError_t inner_product_acc(const u64 *t, const u64 *c_ntt, const u64 *key, int key_limbs,
                              u64 *acc, const u64 *diag, const u64 *c0, const ulonglong2 *pmodq,
                              bool add_c0, bool first, const ModUpDev &mu, const KsLayout &lay,
                              const PrimeDev *primes, int log_n, uint32_t elt, cudaStream_t s) {
  if (lay.n_out <= 0) return cudaSuccess;
  if (!(elt & 1u) || elt >= (2u << log_n)) return cudaErrorInvalidValue;
  k_inner_product_acc<<<grid2(log_n, lay.n_out, 2), kBlk, 0, s>>>(
      t, c_ntt, key, key_limbs, acc, diag, c0, pmodq, add_c0 ? 1 : 0, first ? 1 : 0, mu, lay,
      primes, log_n, elt);
  return cudaGetLastError();
}

cudaError_t inner_product(const u64 *t, const u64 *c_ntt, const u64 *key, int key_limbs,
                          u64 *cx, const ModUpDev &mu, const KsLayout &lay,
                          const PrimeDev *primes, int log_n, uint32_t elt, cudaStream_t s) {
  if (lay.n_out <= 0) return cudaSuccess;
  if (!(elt & 1u) || elt >= (2u << log_n)) return cudaErrorInvalidValue;
  k_inner_product<<<grid2(log_n, lay.n_out, 2), kBlk, 0, s>>>(t, c_ntt, key, key_limbs, cx, mu,
                                                              lay, primes, log_n, elt);
  return cudaGetLastError();
}

cudaError_t mod_reduce(u64 *x, int n_limbs, const int *prime_of_slot, const PrimeDev *primes,
                       int log_n, cudaStream_t s) {
  if (n_limbs <= 0) return cudaSuccess;
  k_mod_reduce<<<grid2(log_n, n_limbs, 1), kBlk, 0, s>>>(x, prime_of_slot, primes, log_n);
  return cudaGetLastError();
}

cudaError_t mac_plain(const MacTerms &a, int n_limbs, const int *prime_of_slot,
                      const PrimeDev *primes, int log_n, cudaStream_t s) {
  if (n_limbs <= 0) return cudaSuccess;
  if (a.n_terms < 1 || a.n_terms > kMacMaxTerms || a.n_out < 1 || a.n_out > kMacMaxOut)
    return cudaErrorInvalidValue;
  const dim3 g = grid2(log_n, n_limbs, 2);
  switch (a.n_out) {
    case 1: k_mac_plain<1><<<g, kBlk, 0, s>>>(a, n_limbs, prime_of_slot, primes, log_n); break;
    case 2: k_mac_plain<2><<<g, kBlk, 0, s>>>(a, n_limbs, prime_of_slot, primes, log_n); break;
    case 3: k_mac_plain<3><<<g, kBlk, 0, s>>>(a, n_limbs, prime_of_slot, primes, log_n); break;
    default: k_mac_plain<4><<<g, kBlk, 0, s>>>(a, n_limbs, prime_of_slot, primes, log_n); break;
  }
  return cudaGetLastError();
}

cudaError_t partition_copy(const u64 *global_buf, u64 *local_buf, long long n_polys,
                           long long total_limbs, long long degree, int g, int G, bool to_local,
                           cudaStream_t s) {
  if (G < 1 || g < 0 || g >= G || n_polys < 0 || total_limbs < 0 || degree < 1)
    return cudaErrorInvalidValue;
  const long long n_local = g < total_limbs ? (total_limbs - g - 1) / G + 1 : 0;
  if (n_local == 0 || n_polys == 0) return cudaSuccess;
  if (n_local > 65535 || n_polys > 65535) return cudaErrorInvalidValue;
  const bool vec = degree % 2 == 0 && ((uintptr_t)global_buf & 15) == 0 &&
                   ((uintptr_t)local_buf & 15) == 0;
  const long long per_thread = vec ? 2 : 1;
  const long long bx = (degree / per_thread + kBlk - 1) / kBlk;
  if (bx > 0x7fffffffLL) return cudaErrorInvalidValue;
  dim3 grid((unsigned)bx, (unsigned)n_local, (unsigned)n_polys);
  if (vec)
    k_scatter<true><<<grid, kBlk, 0, s>>>(global_buf, local_buf, total_limbs, n_local, degree, g,
                                          G, to_local ? 1 : 0);
  else
    k_scatter<false><<<grid, kBlk, 0, s>>>(global_buf, local_buf, total_limbs, n_local, degree, g,
                                           G, to_local ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t scatter_limbs(const u64 *global_buf, u64 *local_buf, int n_polys, int total_limbs,
                          int log_n, int g, int G, cudaStream_t s) {
  return partition_copy(global_buf, local_buf, n_polys, total_limbs, 1ll << log_n, g, G, true, s);
}

cudaError_t gather_limbs(const u64 *local_buf, u64 *global_buf, int n_polys, int total_limbs,
                         int log_n, int g, int G, cudaStream_t s) {
  return partition_copy(global_buf, const_cast<u64 *>(local_buf), n_polys, total_limbs,
                        1ll << log_n, g, G, false, s);
}

cudaError_t keygen_digit(u64 *key_b, u64 *key_a, const u64 *s_ntt, const u64 *snew_ntt,
                         const u64 *e_ntt, int n_limbs, const int *key_index,
                         const int *prime_of_slot, const int *in_digit, const u64 *p_mod_q,
                         uint64_t key_a_stream, int d, int K, const PrimeDev *primes, int log_n,
                         cudaStream_t s) {
  if (n_limbs <= 0) return cudaSuccess;
  k_keygen<<<grid2(log_n, n_limbs, 1), kBlk, 0, s>>>(key_b, key_a, s_ntt, snew_ntt, e_ntt,
                                                     key_index, prime_of_slot, in_digit, p_mod_q,
                                                     key_a_stream, d, K, primes, log_n);
  return cudaGetLastError();
}

cudaError_t sample_gauss(u64 *e, int n_limbs, const int *prime_of_slot, const PrimeDev *primes,
                         const u64 *table, uint64_t stream, uint64_t idx0, int log_n,
                         cudaStream_t s) {
  if (n_limbs <= 0) return cudaSuccess;
  k_gauss<<<grid2(log_n, n_limbs, 1), kBlk, 0, s>>>(e, prime_of_slot, primes, table, stream, idx0,
                                                    log_n);
  return cudaGetLastError();
}

cudaError_t expand_ternary(const int8_t *sk, u64 *out, int n_limbs, const int *prime_of_slot,
                           const PrimeDev *primes, int log_n, cudaStream_t s) {
  if (n_limbs <= 0) return cudaSuccess;
  k_ternary<<<grid2(log_n, n_limbs, 1), kBlk, 0, s>>>(sk, out, prime_of_slot, primes, log_n);
  return cudaGetLastError();
}

cudaError_t mul_pointwise(const u64 *a, const u64 *b, u64 *out, int n_limbs,
                          const int *prime_of_slot, const PrimeDev *primes, int log_n,
                          cudaStream_t s) {
  if (n_limbs <= 0) return cudaSuccess;
  k_mul<<<grid2(log_n, n_limbs, 1), kBlk, 0, s>>>(a, b, out, prime_of_slot, primes, log_n);
  return cudaGetLastError();
}

}  // namespace ksb
