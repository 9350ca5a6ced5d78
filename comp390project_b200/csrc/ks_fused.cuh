// ks_fused.cuh -- key-switch kernels that fuse a base conversion into the
// NTT column pass and the ModDown finish into the NTT row pass.
#pragma once
#include <cuda_runtime.h>

#include "ks_kernels.cuh"
#include "ks_ntt.cuh"

namespace ksb {

// Inverse NTT whose last stage multiplies by a per-limb constant c (on top
// of N^-1): scale[i] = {N^-1 c, Shoup}, {psi^-brev(1) N^-1 c, Shoup}.
// Reads src, writes dst (which may alias src when elt == 1).  elt != 1
// transforms the automorphism X -> X^elt of src (read by gathering).
// Outputs of primes below kFpBound are the bits of the canonical value as a
// double, the others canonical uint64 (the form the base conversions read).
cudaError_t ntt_inverse_scaled(const LimbMap &src, const LimbMap &dst, int n_limbs,
                               const ulonglong2 *scale, const NttTables &T, cudaStream_t s,
                               uint32_t elt = 1, const MemberIn *mi = nullptr, int group = 1);
// ntt_inverse_scaled (with a member's input read as is) through a scratch
// map: the row pass writes tmp, the column pass reads tmp and writes dst,
// limbs li >= pack_from in the 42-bit packed form of pack42 (their primes
// must be below 2^42).
cudaError_t ntt_inverse_scaled_pack(const LimbMap &src, const LimbMap &tmp, const LimbMap &dst,
                                    int n_limbs, const ulonglong2 *scale, const NttTables &T,
                                    cudaStream_t s, const MemberIn *mi, int group, int pack_from);
// The column pass of ntt_inverse_scaled alone, in place on dst (the inverse
// row pass already done).
cudaError_t ntt_inverse_cols_scaled(const LimbMap &dst, int n_limbs, const ulonglong2 *scale,
                                    const NttTables &T, cudaStream_t s, int group);

// A group of key switches pushed through each launch together (grid z =
// member): the member strides (words) of the scratch buffers, and the
// buffers of each member that the caller owns.
struct GroupArgs {
  int n;                                 // members, 1..kMaxGroup
  long long t, cx, z, g0;                // member strides of t, cx, z, g0
  MemberIn in;                           // NTT-form input (read through elt) of each member
  const u64 *key[kMaxGroup];             // key shard of each member
  u64 *ct0[kMaxGroup], *ct1[kMaxGroup];  // output polys of each member
  const u64 *g0p[kMaxGroup];             // rotated c0 of each member (null: none)
  u64 *fold = nullptr;                   // base of the folded P-slot row passes ...
  long long fold_b = 0;                  // ... and its member stride (KsLayout::fold_off)
};

// ModUp: for each job (digit d, output slot s) the column pass of the
// forward NTT of  y[k] = sum_i v_i[k] * w[d][j][i] mod m_j  (j = out_j[s]),
// where v_i are the digit's scaled coefficient limbs (v_all +
// (src_ref[d*alpha + i] >> 1) words, in the 42-bit packed form of pack42
// when bit 0 of src_ref is set).  Result (column pass done) -> t[d][s].
// n_fp of the jobs have targets below kFpBound (FP64 path); the path is
// chosen per CTA from the target prime, so the job order is free (the
// context spreads the integer jobs evenly over the list).
// group > 1: member b reads v_all + b v_bstride and writes t + b t_bstride.
cudaError_t modup_fused_cols(const u64 *v_all, const long long *src_ref, u64 *t, const ModUpDev &mu,
                             const KsLayout &lay, const int *job_d, const int *job_s, int n_jobs,
                             int n_fp, const NttTables &T, cudaStream_t s, int group = 1,
                             long long v_bstride = 0, long long t_bstride = 0,
                             bool packed = false);

// ModUp row pass (t[d][s] from modup_fused_cols, d outside the digit of
// out_j[s]; that digit reads c_ntt slot c_slot[s]) fused with the inner
// product against the key shard ([n_digits][2][key_limbs][N], limb key_slot[s]):
//   cx[p][s] = sum_i NTT_rows(t[d_i][s]) * key[i][p][key_slot[s]]  (p = 0, 1,
// d_i = lay.digits[i], lay.n_digits >= 1).  Two launches: one over the
// integer output slots lay.slots_int, one over the FP64 slots lay.slots_fp.
// elt != 1: the NTT-form input c_ntt is read through X -> X^elt.
cudaError_t modup_rows_inner_product(const u64 *t, const u64 *c_ntt, const u64 *key,
                                     int key_limbs, u64 *cx, const ModUpDev &mu,
                                     const KsLayout &lay, const NttTables &T, cudaStream_t s,
                                     uint32_t elt = 1);
// The same for a group: member b uses t + b G.t, G.in.in[b] read through
// G.in.elt[b], G.key[b], and writes cx + b G.cx.
// side (optional, with two events): the integer launch runs on it, forked
// from and joined back into s, so that it overlaps the FP64 launch.
cudaError_t modup_rows_inner_product_group(const GroupArgs &G, const u64 *t, int key_limbs,
                                           u64 *cx, const ModUpDev &mu, const KsLayout &lay,
                                           const NttTables &T, cudaStream_t s,
                                           cudaStream_t side = nullptr,
                                           cudaEvent_t ev_fork = nullptr,
                                           cudaEvent_t ev_join = nullptr);

// ModDown: for each job (poly p, Q slot s) the column pass of the forward
// NTT of  z[k] = sum_i v_i[k] * w[j][i] mod q_j  (j = q_index[s]), v_i the
// scaled P limbs of poly p at y_base + y_off[p*alpha + i].  -> z[p][s].
// job_ps[2*n_q] lists p*n_q + s in launch order; n_fp of them have q_j
// below kFpBound.
// group > 1: member b reads y_base + b y_bstride and writes z + b z_bstride.
cudaError_t moddown_fused_cols(const u64 *y_base, const long long *y_off, u64 *z, int n_q,
                               const int *q_index, const ModDownDev &md, const int *job_ps,
                               int n_fp, const NttTables &T, cudaStream_t s, int group = 1,
                               long long y_bstride = 0, long long z_bstride = 0);

// Rescale, first part: for every job (poly p, Q slot s), j = q_index[s], the
// column pass of the forward NTT of ([c_p + h]_{q_last} mod q_j) - [h]_{q_j},
// h = floor(q_last / 2), c_p = last[p * N ..] the coefficient-form last limb
// (the bits of a double when last_fp) -> z[p][s].  The second part is
// moddown_fused_rows with q_last^-1 in place of P^-1.
cudaError_t rescale_fused_cols(const u64 *last, u64 q_last, bool last_fp, u64 *z, int n_q,
                               const int *q_index, const NttTables &T, cudaStream_t s);

// Row pass of z[p][s] with the ModDown finish in the epilogue:
//   o = (cx[p][cx_slot[s]] - z) * P^-1 mod q_j;
//   p = 0: v = (rotate ? g0 : ct0) + o (rotate with g0 null: v = o);
//   p = 1: v = rotate ? o : ct1 + o;
//   ct_p = v, or with diag ([n_q][N], NTT form): ct_p += diag * v (a plaintext
//   product accumulated into ct_p).
cudaError_t moddown_fused_rows(const u64 *z, int n_q, const int *q_index, const int *cx_slot,
                               const u64 *cx, long long cx_stride_poly, u64 *ct0, u64 *ct1,
                               const u64 *g0, bool rotate, const u64 *diag,
                               const ModDownDev &md, const NttTables &T, cudaStream_t s);
// The same for a group (no diag): member b reads z + b G.z, cx + b G.cx,
// G.g0p[b] and writes G.ct0[b], G.ct1[b].
cudaError_t moddown_fused_rows_group(const GroupArgs &G, const u64 *z, int n_q,
                                     const int *q_index, const int *cx_slot, const u64 *cx,
                                     long long cx_stride_poly, bool rotate, const ModDownDev &md,
                                     const NttTables &T, cudaStream_t s);

}  // namespace ksb
