// ks_context.hpp -- the per-device key-switching context behind the C ABI.
//
// One context drives one GPU (one rank).  It owns the NTT/base-conversion
// tables, the evaluation-key shards, the scratch arena (sized once at
// creation for the top level, never grown on the hot path) and, for
// world > 1, an NCCL communicator.  The reference keeps the same state in
// PhantomContext + MultiGpuContext and grows thread_local scratch per call
// (input_broadcast.cu:133-152); here every buffer exists before the first call.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/ks_capi.h"
#include "ks_kernels.cuh"
#include "ks_ntt.cuh"

namespace ksb {

// Host copy + device copy of an int table.
struct DevInts {
  std::vector<int> h;
  int *d = nullptr;
};
struct DevI64 {
  std::vector<long long> h;
  long long *d = nullptr;
};

// Everything the key switch needs at one level (Ql Q limbs) on this rank.
struct Level {
  int Ql = 0, QlP = 0, beta = 0;
  int n_out = 0;      // owned output limbs (Q first, then P)
  int n_q = 0;        // owned Q limbs
  int n_p = 0;        // owned P limbs
  int coef_ml = 0;    // ceil(Ql / G): all-gather slot count per rank
  DevInts prime_of;   // [QlP]
  DevInts out_j, key_slot, c_slot;  // [n_out]
  DevInts t_jobs;     // [beta * n_out] prime of t slot or -1
  DevInts q_index;    // [n_q] global Q limb of local Q slot
  DevInts z_jobs;     // [2 * n_q] prime of z slot
  DevInts cx_slot_q;  // [n_q]
  DevInts p_jobs;     // [2 * n_p] primes of the owned P slots being inverse-transformed
  DevI64 p_offsets;   // [2 * n_p] word offsets of those slots (in cx for G=1, in ysend otherwise)
  DevI64 p_cx_offsets;  // [2 * n_p] word offsets of the same slots in cx
  // [2 * n_out]: the fused row pass runs the inverse row pass of the P slots
  // and writes them at these offsets (p_offsets), -1 for Q slots; empty when
  // the level does not fold (output aggregation, FP64-sized P primes)
  DevI64 fold_off;
  DevI64 y_off;       // [2 * alpha] offsets of P limb i of poly p in the y buffer
  ulonglong2 *qhatinv = nullptr;  // [beta][alpha]
  u64 *w = nullptr;               // [beta][QlP][alpha]
  u64 *wsh = nullptr;             // Shoup companions of w
  double *wq = nullptr;           // fl(w / m_j) for FP64 primes
  // fused ModUp: one job per (digit d, output slot s) with limb j outside digit d
  int n_jobs = 0, n_jobs_fp = 0;  // jobs with FP64 targets come first
  DevInts md_job_ps;              // [2 * n_q] ModDown jobs p*n_q + s, FP64 targets first
  int n_md_fp = 0;
  // [beta * alpha] (word offset << 1) | packed of Q limb d*alpha+i in the
  // gathered input (packed: the 42-bit form of pack42)
  DevI64 src_ref;
  // input broadcast with packing: word offsets of the INTT'd owned limbs in
  // the all-gather send buffer (slot 0 whole, then packed limbs)
  DevI64 coef_off;
  long long coef_words = 0;       // words per rank of the input all-gather
  DevInts job_d, job_s, job_prime;  // [n_jobs]
  DevI64 job_off;                 // [n_jobs] word offset of t[d][s]
  // input INTT: the Q limbs this rank extends (owned limbs; in output-aggregation
  // mode the limbs of its digits), at word offset intt_off of the input and
  // of the coefficient buffer, prime intt_prime
  int n_intt = 0;
  DevI64 intt_off;
  DevInts intt_prime;
  DevInts digits;                 // digits of the inner product (all, or this rank's)
  DevInts rip_fp, rip_int;        // output slots of the FP64 / integer row-pass launches
  DevInts cx_prime;               // [2 * n_out] prime of cx slot (post-all-reduce reduction)
  ulonglong2 *scale_in = nullptr; // [2 * n_intt] last-stage INTT scales with (Q_d/q_j)^-1 folded in
  ulonglong2 *scale_p = nullptr;  // [2 * 2 * n_p] same with (P/p_i)^-1 for the owned P limbs
  ModUpDev mu{};
  KsLayout lay{};
  // rescale by q_{Ql-1} (Ql >= 2): unit-scale INTT pairs of the last limb (both
  // polys), its word offsets in the input and prime, and q_{Ql-1}^-1 mod q_j
  ulonglong2 *rs_scale = nullptr;  // [4]
  DevI64 rs_off;                   // [2]
  DevInts rs_prime;                // [2]
  ulonglong2 *rs_pinv = nullptr;   // [L] (j < Ql - 1)
  ModDownDev rs_md{};
};

struct KeyShard {
  u64 *d = nullptr;
  int limbs = 0;  // key limbs held (owned key-basis limbs)
  int beta = 0;   // digits held (Ctx::key_digits)
};

struct Ctx {
  // parameters
  int device = 0, rank = 0, world = 1, mode = 0, max_batch = 1;
  bool capturing = false;  // a graph capture is open (ks_graph_capture_begin)
  cudaStream_t capture_stream = nullptr;
  int log_n = 0, N = 0, L = 0, alpha = 0, K = 0;
  std::vector<u64> primes;  // K = L + alpha
  // device tables (and the host copy of the per-prime constants)
  std::vector<PrimeDev> h_primes;
  PrimeDev *d_primes = nullptr;
  ulonglong2 *d_tw_fwd = nullptr, *d_tw_inv = nullptr;
  double *d_tw_fwd_fp = nullptr, *d_tw_inv_fp = nullptr;
  double2 *d_tw_fwd_col = nullptr, *d_tw_inv_col = nullptr;
  u64 *d_gauss = nullptr;
  ModDownDev md{};
  ulonglong2 *d_phatinv = nullptr, *d_pinv = nullptr;
  ulonglong2 *d_pmodq = nullptr;  // [L] {[P]_{q_j}, Shoup}
  u64 *d_mdw = nullptr, *d_mdwsh = nullptr;
  double *d_mdwq = nullptr;
  std::vector<Level> levels;  // index Ql (1..L)
  // key-basis ownership
  std::vector<int> own_key;   // owned key-basis limbs, increasing
  DevInts own_key_prime;      // same, device copy (prime index == key index)
  std::vector<int> key_digits;  // digits of the key held (all; output aggregation: d % G == g)
  // Input broadcast (G > 1): every rank holds its cyclic limbs of the
  // ciphertext and of the key.  Output aggregation: every rank holds the whole
  // ciphertext and the key digits d % G == g, all limbs.
  bool oa() const { return world > 1 && mode == KS_MODE_OUTPUT_AGGREGATION; }
  // all limbs of the ciphertext on this rank (G = 1 or output aggregation)
  bool replicated() const { return world == 1 || oa(); }
  // keys
  std::map<unsigned long long, KeyShard> keys;  // (kind << 32) | elt
  // Execution lanes: lane 0 runs single calls on the caller's stream; a batch
  // of independent key switches is spread over all lanes, each with its own
  // stream, scratch arena and (world > 1) communicator, so memory-bound and
  // compute-bound stages of different key switches overlap.
  struct Lane {
    cudaStream_t stream = nullptr;  // null for lane 0 (uses the caller's stream)
    cudaEvent_t done = nullptr;
    // side stream of the lane with its fork / join events: the integer launch
    // of the fused row pass overlaps the FP64 launch on it
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    // host-ciphertext path: copies in (on lane 0's `copy` stream, for every
    // lane) fill one half of the staging buffer while the other half's group
    // computes; ev_in[h] / ev_out[h] mark half h filled / emptied
    cudaStream_t copy = nullptr;
    cudaEvent_t ev_in[2] = {nullptr, nullptr}, ev_out[2] = {nullptr, nullptr};
    u64 *arena = nullptr;
    u64 *s_g = nullptr, *s_coef = nullptr, *s_coef_all = nullptr, *s_t = nullptr,
        *s_cx = nullptr, *s_ysend = nullptr, *s_yall = nullptr, *s_z = nullptr,
        *s_ct = nullptr;  // staging of a host ciphertext
    ncclComm_t comm = nullptr;
  };
  std::vector<Lane> lanes;
  cudaEvent_t ev_fork = nullptr;
  size_t arena_words = 0;
  // Groups: a lane pushes up to `group` key switches through every launch
  // together; member b of a lane's scratch buffer X sits b * st_X words on.
  int group = 1;
  long long st_g = 0, st_coef = 0, st_coef_all = 0, st_t = 0, st_cx = 0, st_ys = 0, st_ya = 0,
            st_z = 0, st_ct = 0;
  int max_p_own = 0;
  // 42-bit packing of the input all-gather (input broadcast, world > 1, every
  // Q prime after q_0 below 2^42): a packed limb is pk_words = 11 N / 16 words
  bool pack = false;
  long long pk_words = 0;
  // comm (lane 0's communicator)
  ncclComm_t comm = nullptr;
  bool own_comm = false;
  int timeout_ms = 60000;
  // Collective deadline (see watch_collective): events recorded after the
  // collectives, polled by a watchdog thread that aborts the communicators
  // when one is late.  nccl_mu serialises NCCL enqueues with the abort.
  struct Watch {
    cudaEvent_t ev;
    std::chrono::steady_clock::time_point deadline;
  };
  std::mutex wd_mu, nccl_mu;
  std::vector<Watch> wd_pending;
  std::vector<cudaEvent_t> wd_free;
  std::thread wd_thread;
  std::atomic<bool> wd_stop{false}, aborted{false};
  // written once by the watchdog, before `aborted` is set
  std::string abort_msg;
  // diagnostics
  std::string err;
  // kernel launches of the last API call (reset by each call) and since the
  // context was created
  struct LaunchCount {
    int last = 0;
    long long total = 0;
    LaunchCount &operator+=(int n) {
      last += n;
      total += n;
      return *this;
    }
    LaunchCount &operator=(int v) {
      last = v;
      return *this;
    }
    operator int() const { return last; }
  } launches;
  // optional per-stage timing: event pairs recorded on the launch stream
  bool profile = false;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> prof_events;
  std::vector<cudaEvent_t> event_pool;

  NttTables tables() const {
    return NttTables{d_tw_fwd,    d_tw_inv,    d_primes,     log_n,
                     d_tw_fwd_fp, d_tw_inv_fp, d_tw_fwd_col, d_tw_inv_col};
  }
};

}  // namespace ksb
