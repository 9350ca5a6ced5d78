/*
 * ks_capi.h -- C ABI of the B200-native CKKS hybrid key-switching library
 * (libks_b200.so).
 *
 * This is the drop-in boundary for the reference's key-switching layer
 * (hkanpak21/Comp390Project, namespace nexus_multi_gpu):
 *   src/multi_gpu/keyswitching/input_broadcast.cuh:68-114
 *   src/multi_gpu/keyswitching/output_aggregation.cuh:69-92
 *   src/multi_gpu/comm/nccl_comm.cuh:42-195
 *   src/multi_gpu/partition/rns_partition.cuh:29-191
 * and of the Phantom entry points those files call (keyswitch_inplace,
 * apply_galois_inplace, rotate_vector, relinearize, nwt_2d_radix8_*).
 *
 * Conventions
 *  - C linkage, no exceptions cross the boundary.  Every function returns an
 *    int status: KS_OK (0) or a negative KS_ERR_* code; ks_last_error()
 *    describes the last failure on that context.
 *  - Ciphertexts are caller-owned device arrays of uint64 words in the
 *    PhantomCiphertext layout [poly][limb][N] (reference
 *    paper/code_study.tex:371-372).  With world > 1 each rank holds only the
 *    limbs it owns under the cyclic partition (limb j on rank j % world, at
 *    local slot j / world; rns_partition.cuh:29-60), i.e. [poly][n_local][N].
 *  - NTT values are canonical residues in [0, q); NTT order is bit-reversed.
 *  - `level_limbs` is the number of Q limbs of the ciphertext (Phantom's
 *    coeff_modulus_size; chain_index c corresponds to L - c + 1 limbs).
 *  - Streams are passed as `void *` holding a cudaStream_t (NULL = legacy
 *    default stream).  Calls are asynchronous on that stream.
 *  - One host thread drives one context; contexts are independent.
 *  - Calls on one context must be stream-ordered: every call shares the
 *    context's scratch (lane 0's arena is used by every call, and batched
 *    calls fork their lanes from, and join them back into, the caller's
 *    stream only).  Use one stream per context, or order calls made on
 *    different streams with events; calls that overlap on the GPU race.
 *  - All device pointers must be 16-byte aligned.
 */
#ifndef KS_CAPI_H
#define KS_CAPI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KS_OK 0
#define KS_ERR_INVALID (-1)     /* bad argument: null/misaligned pointer, size, level */
#define KS_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define KS_ERR_NCCL (-3)        /* an NCCL call failed */
#define KS_ERR_NO_KEY (-4)      /* no evaluation key for the requested element */
#define KS_ERR_UNSUPPORTED (-5) /* parameter set outside what the kernels support */
#define KS_ERR_ALLOC (-6)       /* device allocation failed */
#define KS_ERR_TIMEOUT (-7)     /* a collective did not complete within the deadline */

#define KS_KEY_RELIN 0
#define KS_KEY_GALOIS 1

#define KS_MODE_INPUT_BROADCAST 0   /* all-gather c2 limbs, limb-local extension */
#define KS_MODE_OUTPUT_AGGREGATION 1 /* whole ciphertext per rank, digit-split inner product,
                                        all-reduce of the partial sums */

typedef struct ks_ctx ks_ctx;

typedef struct ks_params {
  uint32_t log_n;       /* ring degree N = 2^log_n (12..16) */
  int n_q;              /* L: number of ciphertext (Q) primes */
  const uint64_t *q;    /* Q primes, q_0 first */
  int n_p;              /* alpha: number of special (P) primes = digit size (0..8) */
  const uint64_t *p;    /* P primes */
  int mode;             /* KS_MODE_* (ignored when world == 1) */
  int max_batch;        /* execution lanes (streams with their own scratch) of batched calls, 1..8 */
  int group;            /* key switches each lane pushes through every launch together
                           (0 or 1: one; up to 8); scratch holds max_batch x group key
                           switches.  Zero-initialised callers get one. */
} ks_params;

/* Phantom/SEAL CoeffModulus::Create: the largest primes below 2^bits that are
 * 1 mod 2N, smaller ones first within one bit size. */
int ks_gen_primes(uint32_t log_n, const int *bit_sizes, int n, uint64_t *out);

/* Synthetic ternary secret [N] from a seed: uniform ternary (hamming_weight
 * <= 0) or exactly hamming_weight entries of +-1.  Host function; the
 * sampler is a counter hash, NOT a secure RNG. */
int ks_secret_generate(uint32_t log_n, uint64_t seed, int hamming_weight, int8_t *out);

/* NCCL bootstrap: rank 0 calls ks_nccl_unique_id and shares the bytes
 * (KS_NCCL_ID_BYTES) with the other ranks by any means (e.g. a torch store). */
#define KS_NCCL_ID_BYTES 128
int ks_nccl_unique_id(void *out, size_t n);

/* One context per (device, rank).  world == 1 needs no NCCL id.
 * Replaces MultiGpuContext::create (reference nccl_comm.cu:41-58). */
int ks_ctx_create(const ks_params *prm, int device, int rank, int world,
                  const void *nccl_id, ks_ctx **out);
/* Single-process, all devices (ncclCommInitAll); outs[i] drives devices[i]. */
int ks_ctx_create_all(const ks_params *prm, const int *devices, int n, ks_ctx **outs);
int ks_ctx_destroy(ks_ctx *ctx);
/* Copies the last error message of ctx (or the global one if ctx is NULL). */
int ks_last_error(const ks_ctx *ctx, char *buf, size_t n);
/* Collective deadline in milliseconds (0 = wait forever); default 60000. */
int ks_set_timeout_ms(ks_ctx *ctx, int ms);

/* Partition queries (reference rns_partition.cuh:29-60). */
int ks_n_local_limbs(const ks_ctx *ctx, int total_limbs);
int ks_owner_of_limb(const ks_ctx *ctx, int limb);
int ks_num_digits(const ks_ctx *ctx, int level_limbs);
int ks_galois_elt(const ks_ctx *ctx, int step, uint32_t *elt);
/* Words of one full (unsharded) key: ceil(L/alpha) * 2 * (L+alpha) * N. */
size_t ks_key_words(const ks_ctx *ctx);

/* Evaluation keys, full layout [ceil(L/alpha)][2][L+alpha][N] (NTT form,
 * key[d][0] = b_d, key[d][1] = a_d; reference output_aggregation.cu:115-118).
 * The context keeps the shard its partition needs. */
int ks_key_upload(ks_ctx *ctx, int kind, uint32_t galois_elt, const uint64_t *host_key,
                  size_t n_words);
/* Same, from a device array of the same full layout. */
int ks_key_upload_device(ks_ctx *ctx, int kind, uint32_t galois_elt,
                         const uint64_t *dev_key, size_t n_words, void *stream);
/* Key distribution (collective over the context's ranks; synchronous): the
 * root passes the full key in ITS device memory, the other ranks pass null;
 * every rank ends with its shard, sent from the root over NCCL point-to-point
 * (the reference's distribute_relin_keys / distribute_galois_keys,
 * distributed_context.cu:112-134, are stubs).  With one rank it is
 * ks_key_upload_device. */
int ks_key_distribute(ks_ctx *ctx, int kind, uint32_t galois_elt, const uint64_t *full_dev,
                      int root, void *stream);
/* Generates a synthetic key on the device from an int8 ternary secret [N]
 * (host array) and a seed.  The sampler is a counter hash, NOT a secure RNG. */
int ks_key_generate(ks_ctx *ctx, int kind, uint32_t galois_elt, const int8_t *secret,
                    uint64_t seed, void *stream);
/* Copies the (local shard of the) key back to host memory (for tests). */
int ks_key_download(ks_ctx *ctx, int kind, uint32_t galois_elt, uint64_t *host_key,
                    size_t n_words);
int ks_key_drop(ks_ctx *ctx, int kind, uint32_t galois_elt);

/* Wire format (host functions, no device needed): a self-describing
 * little-endian blob of a full key [digits][2][L+alpha][N] or a ciphertext
 * [polys][level_limbs][N] -- 64-byte header (magic "KSB2WIRE", version,
 * object, Galois element, log_n, n_q, n_p, dimensions, FNV-1a digests of the
 * parameters and of the header + payload) then the words.  The reference has no
 * serialised form (its key distribution, distributed_context.cu:112-134,
 * regenerates keys on every GPU).  Unpack checks parameters, sizes, digests
 * and that every word is a canonical residue; words may be null to only
 * validate. */
#define KS_WIRE_RELIN_KEY 1
#define KS_WIRE_GALOIS_KEY 2
#define KS_WIRE_CIPHERTEXT 3
size_t ks_wire_size(const ks_params *prm, int object, int level_limbs, int n_polys);
int ks_wire_pack(const ks_params *prm, int object, uint32_t galois_elt, int level_limbs,
                 int n_polys, const uint64_t *words, void *out, size_t cap);
int ks_wire_unpack(const ks_params *prm, const void *blob, size_t n, int *object,
                   uint32_t *galois_elt, int *level_limbs, int *n_polys, uint64_t *words,
                   size_t cap_words);
/* Validates a key blob against the context's parameters and uploads it
 * (the context keeps its shard, as ks_key_upload). */
int ks_key_upload_wire(ks_ctx *ctx, const void *blob, size_t n);

/* Relinearisation of ct [3][n_local][N] in place: polys 0, 1 receive the
 * result.  Replaces keyswitching_input_broadcast / keyswitching_output_
 * aggregation (input_broadcast.cu:117-176, output_aggregation.cu:197-294). */
int ks_relinearize(ks_ctx *ctx, uint64_t *ct, int level_limbs, void *stream);
/* Generic key switch of one polynomial c [n_local][N] (NTT form) with the key
 * (kind, galois_elt), added into ct [2][n_local][N]: ct0 += ks0(c),
 * ct1 += ks1(c).  With the relinearisation key this is the reference's
 * keyswitching_input_broadcast(encrypted, local_c2, relin_keys)
 * (input_broadcast.cuh:68-78), c and ct in separate buffers. */
int ks_keyswitch_add(ks_ctx *ctx, const uint64_t *c, uint64_t *ct, int level_limbs, int kind,
                     uint32_t galois_elt, void *stream);
/* X -> X^galois_elt on ct [2][n_local][N] in place plus key switch with the
 * Galois key of that element (Phantom apply_galois_inplace;
 * rotation_input_broadcast, input_broadcast.cu:182-202). */
int ks_apply_galois(ks_ctx *ctx, uint64_t *ct, int level_limbs, uint32_t galois_elt,
                    void *stream);
/* ks_apply_galois for callers that may not allocate device memory when they
 * call in (a fixed memory budget, or HBM reserved up front by the host
 * application).  No counterpart in the reference.  Same result as
 * ks_apply_galois; its scratch is a file-scope device array of 16 MiB (held
 * by every GPU that loads the library until the process exits) and the call
 * makes no cudaMalloc/cudaFree.  Parameter sets whose key switch needs more
 * scratch than that (e.g. N = 2^16 with 35 + 5 primes) are rejected with
 * KS_ERR_UNSUPPORTED; world must be 1 and profiling off.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress), so make
 * that first call before any stream capture.  All calls share the one array:
 * calls that overlap on the GPU (other streams, other contexts on the same
 * device) race; serialise them.  No word of the array needs to start at zero. */
int ks_apply_galois_noalloc(ks_ctx *ctx, uint64_t *ct, int level_limbs, uint32_t galois_elt,
                            void *stream);
/* Left rotation of the slots by `step` (galois element 3^step mod 2N). */
int ks_rotate(ks_ctx *ctx, uint64_t *ct, int level_limbs, int step, void *stream);
/* n rotations of n independent ciphertexts (cts[i] rotated by steps[i]). */
int ks_rotate_batch(ks_ctx *ctx, uint64_t *const *cts, const int *steps, int n,
                    int level_limbs, void *stream);
/* Rescale by the last prime of the level (divide by q_{Ql-1} and round;
 * Phantom rescale_to_next_inplace as called by the reference's
 * dist_rescale_to_next_inplace, distributed_eval.cu:265-273): ct
 * [2][n_local(Ql)][N] -> out [2][n_local(Ql-1)][N], out must not alias ct.
 * With input broadcast only the owner's last limb crosses NVLink (one
 * broadcast of 2N words); the reference gathers the whole ciphertext on
 * GPU 0 instead. */
int ks_rescale(ks_ctx *ctx, const uint64_t *ct, int level_limbs, uint64_t *out, void *stream);
/* ks_rotate_batch on ciphertexts in HOST memory (pinned memory lets the
 * copies overlap the compute): host_cts[i] [2][n_local][N] is copied to the
 * device, rotated by steps[i] and copied back in place.  The ciphertexts are
 * spread over the lanes, each with its own device staging buffer, so the
 * copies of one lane overlap the key switches of the others; with
 * ks_params.group >= 2 the staging buffer is split in two halves and a
 * lane's next group is copied in (on one copy stream shared by the lanes,
 * in batch order) while its current group rotates and is copied out.  Asynchronous on `stream`: the
 * host buffers may be read only after it completes. */
int ks_rotate_batch_host(ks_ctx *ctx, uint64_t *const *host_cts, const int *steps, int n,
                         int level_limbs, void *stream);
/* Hoisted rotations: one ModUp of ct's c1 shared by n rotations (the
 * extended digits are permuted per rotation inside the inner product); outs[i]
 * [2][n_local][N] receives ct rotated by steps[i].  ct is not modified.  Keys
 * for every step must be uploaded. */
int ks_rotate_hoisted(ks_ctx *ctx, const uint64_t *ct, int level_limbs, const int *steps,
                      int n, uint64_t *const *outs, void *stream);
/* Hoisted linear transform (BSGS / CoeffToSlot style):
 *   out = sum_i diags[i] * rotate(ct, steps[i])
 * with one ModUp of c1 and one ModDown for all rotations (double hoisting:
 * the products are accumulated in the extended basis Q_l * P).  diags[i]
 * is the plaintext diagonal in NTT form in the extended basis, one word per
 * output limb of this rank: [Ql + alpha][N] (Q limbs then P limbs) on one
 * GPU or in output aggregation, the owned Q limbs then the owned P limbs in
 * input broadcast.  No rescale.  out [2][n_local][N] is overwritten and must
 * not alias ct. */
int ks_linear_transform_hoisted(ks_ctx *ctx, const uint64_t *ct, int level_limbs,
                                const int *steps, int n, const uint64_t *const *diags,
                                uint64_t *out, void *stream);

/* Ciphertext x plaintext block matrix product by the diagonal method with
 * baby and giant steps (B = n_baby, G = n_giant, u = unit):
 *   y[o] = sum_{g_lo <= g < g_hi} rotate( sum_{i < n_in} sum_{b < B}
 *            pts[((o n_in + i) G + g) B + b] (.) rotate(x[i], b u),  g B u )
 * x[i], y[o]: [2][n_local][N] at level_limbs; pts[...]: NTT-form plaintexts
 * [n_local][N] over the Q limbs (the diagonals, already rotated by -g B u).
 * baby == NULL: the B - 1 baby-step rotations of each input are computed
 * here, sharing one ModUp per input; otherwise baby[i (B-1) + b - 1] holds
 * rotate(x[i], b u) (e.g. computed by several GPUs and all-gathered).  Up to
 * four giant steps share one pass over the baby-step ciphertexts.  No
 * rescale.  Galois keys are needed for steps b u (0 < b < B, baby == NULL)
 * and g B u (g > 0 in range).  [g_lo, g_hi) = [0, G) gives the whole
 * product; a sub-range gives the partial sum over those giant steps (callers
 * that split the giant steps over GPUs add the partial sums and call
 * ks_reduce_limbs).  workspace holds ks_bsgs_workspace_words(ctx,
 * level_limbs, n_in, baby ? 1 : n_baby) words; y[o] must alias neither an
 * input nor the workspace. */
size_t ks_bsgs_workspace_words(ks_ctx *ctx, int level_limbs, int n_in, int n_baby);
int ks_bsgs_matmul(ks_ctx *ctx, const uint64_t *const *x, const uint64_t *const *baby,
                   int n_in, int level_limbs, int unit, int n_baby, int n_giant, int g_lo,
                   int g_hi, const uint64_t *const *pts, uint64_t *const *y, int n_out,
                   uint64_t *workspace, void *stream);
/* x [n_polys][n_local][N] in place: every word (any 64-bit value, e.g. a sum
 * of residues from an integer all-reduce) reduced mod its limb's prime. */
int ks_reduce_limbs(ks_ctx *ctx, uint64_t *x, int n_polys, int level_limbs, void *stream);

/* Batched negacyclic NTT in place over data [batch][n_limbs][N]; limb i uses
 * prime first_prime + i of the context's basis (Q primes then P primes).
 * Replaces nwt_2d_radix8_forward_inplace / backward_inplace. */
int ks_ntt_forward(ks_ctx *ctx, uint64_t *data, int n_limbs, int first_prime, int batch,
                   void *stream);
int ks_ntt_inverse(ks_ctx *ctx, uint64_t *data, int n_limbs, int first_prime, int batch,
                   void *stream);

/* Cyclic partition copies global [n_polys][total][N] <-> local
 * [n_polys][n_local][N] for this context's rank (rns_partition.cu:86-128). */
int ks_scatter_limbs(ks_ctx *ctx, const uint64_t *global_buf, uint64_t *local_buf,
                     int n_polys, int total_limbs, void *stream);
int ks_gather_limbs(ks_ctx *ctx, const uint64_t *local_buf, uint64_t *global_buf,
                    int n_polys, int total_limbs, void *stream);
/* The same copies without a context, with the reference's own signature
 * (scatter_ciphertext_to_gpu / gather_ciphertext_from_gpu,
 * rns_partition.cuh:165-190): rank gpu_id of n_gpus, any degree (words per
 * limb), both buffers on the current device.  A rank that owns no limb copies
 * nothing (the reference returns early too). */
int ks_scatter_ciphertext_to_gpu(const uint64_t *global_buf, uint64_t *local_buf, size_t n_polys,
                                 size_t total_limbs, size_t degree, int gpu_id, int n_gpus,
                                 void *stream);
int ks_gather_ciphertext_from_gpu(const uint64_t *local_buf, uint64_t *global_buf, size_t n_polys,
                                  size_t total_limbs, size_t degree, int gpu_id, int n_gpus,
                                  void *stream);
/* All-gather of local limbs [n_local][N] into sequential order [total][N]
 * on every rank (allgather_c2_limbs + reorder, input_broadcast.cu:45-111). */
int ks_allgather_limbs(ks_ctx *ctx, const uint64_t *local_buf, uint64_t *full_buf,
                       int total_limbs, void *stream);

/* Number of kernels the last hot-path call launched (for bench accounting). */
int ks_last_launch_count(const ks_ctx *ctx);
/* Kernel launches of every call since the context was created. */
long long ks_total_launch_count(const ks_ctx *ctx);

/* CUDA graph capture and replay of hot-path calls (the capture/replay half
 * of the reference's StreamManager, overlap/stream_manager.cu:25-159).
 * ks_graph_capture_begin starts a thread-local capture on `stream` (not the
 * legacy default stream); every hot-path call made on that stream until
 * ks_graph_capture_end is recorded instead of run (batched calls fork their
 * lanes from the capturing stream, NCCL collectives are captured too); end
 * instantiates the graph.  Replay with ks_graph_launch on any stream of the
 * context's device.  The graph keeps the pointers and keys of the captured
 * calls: the ciphertext buffers must stay allocated and the keys uploaded
 * while it is used; a call that fails during capture ends the capture.
 * Make each kind of call once outside capture first (kernel attributes are
 * set on first use); profiling must be off. */
typedef struct ks_graph ks_graph;
int ks_graph_capture_begin(ks_ctx *ctx, void *stream);
int ks_graph_capture_end(ks_ctx *ctx, void *stream, ks_graph **out);
int ks_graph_launch(ks_graph *graph, void *stream);
int ks_graph_destroy(ks_graph *graph);

/* Optional per-stage timing of the key switch with CUDA events recorded on
 * the launch stream (bench accounting; off by default).  ks_profile_read
 * waits for the recorded events, returns the summed milliseconds and the
 * number of timed calls per stage, and clears the record. */
int ks_profile_enable(ks_ctx *ctx, int on);
int ks_profile_stage_count(void);
const char *ks_profile_stage_name(int i);
int ks_profile_read(ks_ctx *ctx, double *ms, int *calls, int n);

#ifdef __cplusplus
}
#endif
#endif /* KS_CAPI_H */
