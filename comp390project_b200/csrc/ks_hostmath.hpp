// ks_hostmath.hpp -- host-side number theory for the key-switching context:
// primality, the prime-selection rule, primitive roots, Shoup/Barrett
// constants and base-conversion tables.  Runs once at context creation.
#pragma once
#include <cstdint>
#include <map>
#include <stdexcept>
#include <vector>

namespace ksb {

typedef unsigned __int128 u128;
typedef uint64_t u64;

inline u64 h_mulmod(u64 a, u64 b, u64 q) { return (u64)((u128)a * b % q); }
inline u64 h_powmod(u64 a, u64 e, u64 q) {
  u64 r = 1 % q;
  a %= q;
  for (; e; e >>= 1) {
    if (e & 1) r = h_mulmod(r, a, q);
    a = h_mulmod(a, a, q);
  }
  return r;
}
inline u64 h_invmod(u64 a, u64 q) { return h_powmod(a, q - 2, q); }
inline u64 h_shoup(u64 w, u64 q) { return (u64)(((u128)w << 64) / q); }

inline bool h_is_prime(u64 n) {
  if (n < 2) return false;
  static const u64 bases[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
  for (u64 p : bases)
    if (n % p == 0) return n == p;
  u64 d = n - 1;
  int s = 0;
  while (!(d & 1)) { d >>= 1; ++s; }
  for (u64 a : bases) {
    u64 x = h_powmod(a, d, n);
    if (x == 1 || x == n - 1) continue;
    bool witness = true;
    for (int r = 1; r < s && witness; ++r) {
      x = h_mulmod(x, x, n);
      if (x == n - 1) witness = false;
    }
    if (witness) return false;
  }
  return true;
}

// Phantom / SEAL CoeffModulus::Create(N, bit_sizes): for every bit size b the
// largest primes below 2^b that are 1 mod 2N; within one size the smaller
// primes take the earlier positions.
inline int h_gen_primes(int log_n, const int *bits, int n, u64 *out) {
  const u64 f = 2ull << log_n;
  std::map<int, int> need;
  for (int i = 0; i < n; ++i) need[bits[i]]++;
  std::map<int, std::vector<u64>> pool;
  for (auto &kv : need) {
    int b = kv.first;
    if (b < 2 || b > 61) return -1;
    std::vector<u64> got;
    for (u64 v = ((1ull << b) - 1) / f * f + 1; (int)got.size() < kv.second && v > (1ull << (b - 1)); v -= f)
      if (h_is_prime(v)) got.push_back(v);
    if ((int)got.size() < kv.second) return -1;
    pool[b] = got;
  }
  for (int i = 0; i < n; ++i) {
    out[i] = pool[bits[i]].back();
    pool[bits[i]].pop_back();
  }
  return 0;
}

inline uint32_t h_brev(uint32_t x, int bits) {
  uint32_t r = 0;
  for (int i = 0; i < bits; ++i) { r = (r << 1) | (x & 1u); x >>= 1; }
  return r;
}

// Minimal primitive 2N-th root of unity mod q.
inline u64 h_min_psi(u64 q, u64 N) {
  u64 g = 0;
  for (u64 x = 2; x < q && !g; ++x) {
    u64 c = h_powmod(x, (q - 1) / (2 * N), q);
    if (h_powmod(c, N, q) == q - 1) g = c;
  }
  if (!g) throw std::runtime_error("modulus has no primitive 2N-th root");
  u64 g2 = h_mulmod(g, g, q), cur = g, best = g;
  for (u64 i = 0; i < N; ++i) {
    if (cur < best) best = cur;
    cur = h_mulmod(cur, g2, q);
  }
  return best;
}

// floor(2^128 / q) as (hi, lo).
inline void h_barrett_ratio(u64 q, u64 &hi, u64 &lo) {
  u128 top = ~(u128)0;  // 2^128 - 1; q is not a power of two, so floor matches
  u128 r = top / q;
  hi = (u64)(r >> 64);
  lo = (u64)r;
}

}  // namespace ksb
