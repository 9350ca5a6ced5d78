/*
 * ckks_oracle.h -- CPU restatement of the CKKS hybrid key-switching path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code; it is the checker that the CUDA path is compared against
 * (tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py).
 *
 * Parity status.  The reference (hkanpak21/Comp390Project) delegates all
 * arithmetic to the Phantom FHE library (git submodule encryptorion-lab/
 * phantom-fhe @ 1f4a198), which is not vendored in the reference tree, so
 * no limb-level golden vector of the reference exists.  Bit-level parity
 * with Phantom is therefore UNPINNED.  What IS pinned:
 *   - prime selection, against every modulus the reference logged
 *     (experiments/results/2026-03-29_l4_baseline-ops/raw/ckks_bench.txt:11,35,59,...),
 *   - the partition/index math, against the reference's own header
 *     src/multi_gpu/partition/rns_partition.cuh compiled under oracle/_ref,
 *   - semantics, by the reference's own acceptance criterion: decrypt+decode
 *     MAE < 1e-3 against the plaintext result
 *     (src/benchmarks/multi_gpu_keyswitch_test.cu:292-298),
 *   - the NTT against a naive O(N^2) negacyclic evaluation, and base
 *     conversion against Python big-integer CRT (tests/).
 *
 * Conventions (fixed here because Phantom's source is absent):
 *   - ring Z_q[X]/(X^N+1); NTT output in bit-reversed order: slot i holds
 *     a(psi^(2*brev(i)+1)); psi = the minimal primitive 2N-th root mod q.
 *   - ciphertext layout [poly][limb][coeff] (paper/code_study.tex:371-372).
 *   - key-switching key layout [digit][2][L+alpha][N], P limbs after the
 *     L Q limbs (src/multi_gpu/keyswitching/output_aggregation.cu:94-118).
 *   - digits are consecutive groups of alpha Q limbs; at a level with Ql
 *     limbs there are ceil(Ql/alpha) digits, the last possibly short.
 *   - Galois element of a left rotation by r slots is 3^r mod 2N.
 *
 * All arrays are uint64 words in little-endian host order.
 */
#ifndef CKKS_ORACLE_H
#define CKKS_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ork_ctx ork_ctx;

/* Primes ≡ 1 (mod 2N) by the rule of Phantom/SEAL CoeffModulus::Create.
 * Returns 0 on success, -1 if a bit size has too few primes. */
int ork_gen_primes(uint32_t log_n, const int *bit_sizes, int n, uint64_t *out);
int ork_is_prime(uint64_t v);

ork_ctx *ork_create(uint32_t log_n, const uint64_t *q, int L,
                    const uint64_t *p, int alpha);
void ork_destroy(ork_ctx *c);
void ork_set_threads(int n);
int ork_get_threads(void);
int ork_num_digits(const ork_ctx *c, int Ql);
uint64_t ork_psi(const ork_ctx *c, int key_idx);

/* Transforms on [n_limbs][N] in place; limb i uses key-basis prime key_idx[i]
 * (0..L-1 are Q primes, L..L+alpha-1 are P primes). */
void ork_ntt_forward(const ork_ctx *c, uint64_t *data, int n_limbs, const int *key_idx);
void ork_ntt_inverse(const ork_ctx *c, uint64_t *data, int n_limbs, const int *key_idx);

uint32_t ork_galois_elt(const ork_ctx *c, int step);
/* NTT-domain automorphism X -> X^elt on [n_limbs][N]. */
void ork_galois_ntt(const ork_ctx *c, uint32_t elt, const uint64_t *in,
                    uint64_t *out, int n_limbs);
/* Coefficient-domain automorphism. */
void ork_galois_coeff(const ork_ctx *c, uint32_t elt, const uint64_t *in,
                      uint64_t *out, int n_limbs, const int *key_idx);

/* Fast base conversion (coefficient domain) from the primes in_idx to the
 * primes out_idx: y_j = sum_i [x_i * (B/b_i)^-1]_{b_i} * [B/b_i]_{c_j} mod c_j. */
void ork_bconv(const ork_ctx *c, const uint64_t *in, const int *in_idx, int n_in,
               uint64_t *out, const int *out_idx, int n_out);

/* Key-switching stages.  c: [Ql][N] NTT form.  t: [beta][Ql+alpha][N].
 * cx: [2][Ql+alpha][N].  moddown: one poly [Ql+alpha][N] -> [Ql][N]. */
void ork_modup(const ork_ctx *c, const uint64_t *in, int Ql, uint64_t *t);
void ork_inner_product(const ork_ctx *c, const uint64_t *t, int Ql,
                       const uint64_t *key, uint64_t *cx);
void ork_moddown(const ork_ctx *c, const uint64_t *cx_poly, int Ql, uint64_t *out);
/* Whole key switch: out [2][Ql][N] = (ks0, ks1). */
void ork_keyswitch(const ork_ctx *c, const uint64_t *in, int Ql,
                   const uint64_t *key, uint64_t *out);
/* ct [2][Ql][N] -> out [2][Ql][N] (galois + key switch). */
void ork_apply_galois(const ork_ctx *c, const uint64_t *ct, int Ql, uint32_t elt,
                      const uint64_t *key, uint64_t *out);
/* ct [3][Ql][N] -> out [2][Ql][N]. */
void ork_relinearize(const ork_ctx *c, const uint64_t *ct, int Ql,
                     const uint64_t *key, uint64_t *out);
/* Hoisted rotations: one ModUp of c1 shared by n rotations.  out [n][2][Ql][N]. */
void ork_rotate_hoisted(const ork_ctx *c, const uint64_t *ct, int Ql, int n,
                        const uint32_t *elts, const uint64_t *const *keys,
                        uint64_t *out);
/* out = sum_r diags[r] * rotate(ct, elts[r]) with one ModUp and one ModDown
 * (double hoisting); diags[r] [Ql + alpha][N] NTT form in the extended basis. */
/* ct [2][Ql][N] -> out [2][Ql-1][N]: divide by the last prime and round. */
void ork_rescale(const ork_ctx *c, const uint64_t *ct, int Ql, uint64_t *out);
void ork_linear_transform_hoisted(const ork_ctx *c, const uint64_t *ct, int Ql, int n,
                                  const uint32_t *elts, const uint64_t *const *keys,
                                  const uint64_t *const *diags, uint64_t *out);
/* Block BSGS matrix product: y[o] [2][Ql][N] =
 *   sum_{g_lo <= g < g_hi} rot_g( sum_i sum_{b < B} pts[((o n_in + i) G + g) B + b] * rot_b(x[i]) ),
 * rot_b by baby_elts[b - 1] (hoisted), rot_g by giant_elts[g] (g > 0). */
void ork_bsgs_matmul(const ork_ctx *c, const uint64_t *const *x, int n_in, int Ql, int B,
                     int G, int g_lo, int g_hi, const uint32_t *baby_elts,
                     const uint64_t *const *baby_keys, const uint32_t *giant_elts,
                     const uint64_t *const *giant_keys, const uint64_t *const *pts, int n_out,
                     uint64_t *const *y);

/* Deterministic sampling shared with the product's synthetic-key generator. */
uint64_t ork_prng(uint64_t seed, uint64_t domain, uint64_t idx);
int ork_gauss(uint64_t r);
void ork_gauss_table(uint64_t *t20);
void ork_secret(const ork_ctx *c, uint64_t seed, int hamming_weight, int8_t *s);
/* key: [ceil(L/alpha)][2][L+alpha][N] */
void ork_keygen_galois(const ork_ctx *c, const int8_t *s, uint32_t elt,
                       uint64_t seed, uint64_t *key);
void ork_keygen_relin(const ork_ctx *c, const int8_t *s, uint64_t seed, uint64_t *key);

/* CKKS encoding with N/2 slots, slot j <-> root zeta^(3^j). pt: [Ql][N] NTT. */
void ork_encode(const ork_ctx *c, const double *re, const double *im, int n_slots,
                double scale, int Ql, uint64_t *pt);
void ork_encode_basis(const ork_ctx *c, const double *re, const double *im, int n_slots,
                      double scale, const int *key_idx, int n_idx, uint64_t *pt);
void ork_decode(const ork_ctx *c, const uint64_t *pt, int Ql, double scale,
                double *re, double *im, int n_slots);
void ork_encrypt(const ork_ctx *c, const int8_t *s, const uint64_t *pt, int Ql,
                 uint64_t seed, uint64_t *ct);
void ork_decrypt(const ork_ctx *c, const int8_t *s, const uint64_t *ct, int n_polys,
                 int Ql, uint64_t *pt);
void ork_multiply(const ork_ctx *c, const uint64_t *a, const uint64_t *b, int Ql,
                  uint64_t *out);
/* max |centered coefficient| over limb 0 of  (k0 + k1*s - in*s')  where the
 * key-switch target s' is given in NTT form over the Q primes; used by the
 * size-independent noise check.  Returns log2 of the bound (or 64 if huge). */
double ork_ks_noise_log2(const ork_ctx *c, const int8_t *s, const uint64_t *in,
                         const uint64_t *snew_ntt, const uint64_t *ks, int Ql);
/* s' helpers, NTT form over the first n_limbs key primes. */
void ork_secret_ntt(const ork_ctx *c, const int8_t *s, int n_limbs, uint64_t *out);

#ifdef __cplusplus
}
#endif
#endif
