// ks_kernels.cuh -- element-wise and base-conversion kernels of the hybrid
// key switch (ModUp base extension, evaluation-key inner product, ModDown
// finish, NTT-domain automorphism), the limb scatter/gather of the cyclic
// partition, and the synthetic-key samplers.
#pragma once
#include <cuda_runtime.h>

#include "ks_arith.cuh"
#include "ks_ntt.cuh"

namespace ksb {

constexpr int KS_MAX_ALPHA = 8;

// Per-level constants of the base extension Q_d -> (Ql+alpha) basis, in
// device memory.  Digit d covers the Q limbs [d*alpha, min((d+1)*alpha, Ql)).
struct ModUpDev {
  int Ql, QlP, beta, alpha;
  const int *prime_of;        // [QlP] prime index of QlP limb j (Q limbs, then P)
  const ulonglong2 *qhatinv;  // [beta][alpha] {[(Q_d/q_i)^-1]_{q_i}, Shoup}
  const u64 *w;               // [beta][QlP][alpha] [Q_d/q_i]_{m_j}
  const u64 *wsh;             // same layout: Shoup companions of w w.r.t. m_j
  const double *wq;           // same layout: fl(w / m_j) for FP64 primes m_j
};

// Constants of the conversion P -> Q (ModDown), indexed by Q limb j.
struct ModDownDev {
  int alpha;
  int first_p;                // prime index of p_0
  const ulonglong2 *phatinv;  // [alpha] {[(P/p_i)^-1]_{p_i}, Shoup}
  const u64 *w;               // [L][alpha] [P/p_i]_{q_j}
  const ulonglong2 *pinv;     // [L] {[P^-1]_{q_j}, Shoup}
  const u64 *wsh;             // [L][alpha] Shoup companions of w w.r.t. q_j
  const double *wq;           // [L][alpha] fl(w / q_j) for FP64 primes q_j
};

// Which QlP limbs this device produces and where its inputs live.
struct KsLayout {
  int n_out;                  // number of output limbs (owned QlP limbs)
  const int *out_j;           // [n_out] QlP index of output slot s
  const int *key_slot;        // [n_out] limb slot of that limb in the key shard
  const int *c_slot;          // [n_out] local slot of Q limb j in the NTT-form input, or -1
  int coef_G, coef_ml;        // coefficient-form Q limb j at slot (j % G) * ml + j / G
  const int *digits;          // [n_digits] digits summed by the inner product, ascending;
  int n_digits;               // digit digits[i] is digit i of the key shard
  // the output slots whose prime takes the FP64 path and the others, each
  // served by its own launch of the fused row pass (kernels of one arithmetic
  // kind keep the instruction cache warm)
  const int *slots_fp, *slots_int;
  int n_slots_fp, n_slots_int;
  // [2 n_out] or null: for a P slot s, where the integer launch writes poly
  // p's tile after the inverse row pass (word offset fold_off[2 s + p] from
  // the fold base of the member) instead of writing cx; -1 for Q slots
  const long long *fold_off;
};

// out[l][i] = in[l][perm_elt(i)] for the NTT-domain automorphism X -> X^elt.
cudaError_t galois_ntt(const u64 *in, u64 *out, int n_limbs, int log_n, uint32_t elt,
                       cudaStream_t s);
// The same for a group: member b permutes mi.in[b] by mi.elt[b] into
// out + b out_bstride.
cudaError_t galois_ntt_group(const MemberIn &mi, int group, u64 *out, long long out_bstride,
                             int n_limbs, int log_n, cudaStream_t s);

// Inner product of the automorphism X -> X^elt of the extended digits
// (elt = 1: no automorphism), all in NTT form:
//   cx[p][s][k] = sum_i src_{d_i}[s][galois_src(k)] * key[i][p][key_slot[s]][k]  mod m_j,
// d_i = lay.digits[i], src_d = c_ntt[c_slot[s]] when limb j lies in digit d,
// else t[d][s] (t: [beta][n_out][N]); key: [n_digits][2][key_limbs][N].
cudaError_t inner_product(const u64 *t, const u64 *c_ntt, const u64 *key, int key_limbs,
                          u64 *cx, const ModUpDev &mu, const KsLayout &lay,
                          const PrimeDev *primes, int log_n, uint32_t elt, cudaStream_t s);
// The same inner product accumulated into a linear transform in the extended
// basis (double hoisting): with ip_p the inner product above,
//   acc[0][s] = (first ? 0 : acc[0][s]) + diag[s] * (ip_0 + [P]_{q_j} c0[c_slot[s]] o elt)
//   acc[1][s] = (first ? 0 : acc[1][s]) + diag[s] * ip_1
// (the c0 term only for Q limbs and when add_c0; pmodq[j] = {[P]_{q_j}, Shoup};
// diag null: no plaintext factor).
cudaError_t inner_product_acc(const u64 *t, const u64 *c_ntt, const u64 *key, int key_limbs,
                              u64 *acc, const u64 *diag, const u64 *c0, const ulonglong2 *pmodq,
                              bool add_c0, bool first, const ModUpDev &mu, const KsLayout &lay,
                              const PrimeDev *primes, int log_n, uint32_t elt, cudaStream_t s);

// Plaintext multiply-accumulate over a term list, for up to kMacMaxOut outputs
// that share the ciphertext terms (passed by value as kernel parameters):
//   out_j[p][l] (+)= sum_m pt[j][m][l] * ct[m][p][l]  mod q_{prime_of_slot[l]},  p = 0, 1,
// ct[m] and out_j: [2][n_limbs][N], pt[j][m]: [n_limbs][N], all NTT form with
// canonical residues; accumulate != 0 adds to out_j's contents.  Every
// pointer 16-byte aligned.
constexpr int kMacMaxTerms = 64;
constexpr int kMacMaxOut = 4;
struct MacTerms {
  const u64 *ct[kMacMaxTerms];
  const u64 *pt[kMacMaxOut][kMacMaxTerms];
  u64 *out[kMacMaxOut];
  int n_terms, n_out, accumulate;
};
cudaError_t mac_plain(const MacTerms &a, int n_limbs, const int *prime_of_slot,
                      const PrimeDev *primes, int log_n, cudaStream_t s);

// x %= q for each limb (after an integer all-reduce / reduce-scatter of partial sums).
cudaError_t mod_reduce(u64 *x, int n_limbs, const int *prime_of_slot, const PrimeDev *primes,
                       int log_n, cudaStream_t s);

// Cyclic partition copies: global [poly][total][N] <-> local [poly][n_local][N]
// for the limbs j = local*G + g (reference rns_partition.cu:26-80).
// Cyclic-partition copy for rank g of G with an arbitrary degree (words per
// limb): global [n_polys][total][degree] <-> local [n_polys][n_local][degree].
cudaError_t partition_copy(const u64 *global_buf, u64 *local_buf, long long n_polys,
                           long long total_limbs, long long degree, int g, int G, bool to_local,
                           cudaStream_t s);
cudaError_t scatter_limbs(const u64 *global_buf, u64 *local_buf, int n_polys, int total_limbs,
                          int log_n, int g, int G, cudaStream_t s);
cudaError_t gather_limbs(const u64 *local_buf, u64 *global_buf, int n_polys, int total_limbs,
                         int log_n, int g, int G, cudaStream_t s);

// Synthetic evaluation-key generation for one digit d over n_limbs key limbs
// (not a secure generator; the sampler is the counter-based hash shared with
// the CPU oracle).  key_a_stream = the per-(seed, domain) hash key.
cudaError_t keygen_digit(u64 *key_b, u64 *key_a, const u64 *s_ntt, const u64 *snew_ntt,
                         const u64 *e_ntt, int n_limbs, const int *key_index,
                         const int *prime_of_slot, const int *in_digit, const u64 *p_mod_q,
                         uint64_t key_a_stream, int d, int K, const PrimeDev *primes, int log_n,
                         cudaStream_t s);
cudaError_t sample_gauss(u64 *e, int n_limbs, const int *prime_of_slot, const PrimeDev *primes,
                         const u64 *table, uint64_t stream, uint64_t idx0, int log_n,
                         cudaStream_t s);
cudaError_t expand_ternary(const int8_t *sk, u64 *out, int n_limbs, const int *prime_of_slot,
                           const PrimeDev *primes, int log_n, cudaStream_t s);
cudaError_t mul_pointwise(const u64 *a, const u64 *b, u64 *out, int n_limbs,
                          const int *prime_of_slot, const PrimeDev *primes, int log_n,
                          cudaStream_t s);

}  // namespace ksb
