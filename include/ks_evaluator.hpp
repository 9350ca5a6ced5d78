// ks_evaluator.hpp -- C++ host-side shim over the C ABI (header only).
//
// Gives existing C++ callers of the reference (hkanpak21/Comp390Project,
// namespace nexus_multi_gpu) the same entry points with the same argument
// meaning:
//   keyswitching_input_broadcast   input_broadcast.cuh:68-78
//   rotation_input_broadcast       input_broadcast.cuh:86-97
//   keyswitching_output_aggregation output_aggregation.cuh:69-77
//   allgather_c2_limbs             input_broadcast.cuh:106-114
// and a Phantom-style Evaluator (rotate_vector / relinearize / apply_galois).
// Errors throw std::runtime_error carrying ks_last_error(), as the
// reference's CUDA_CHECK/NCCL_CHECK do; calls synchronise the stream before
// returning, as the reference's do.
#pragma once
#include <cuda_runtime_api.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "ks_capi.h"

namespace ks_b200 {

inline void check(int rc, const ks_ctx *ctx) {
  if (rc < 0) {
    char buf[512];
    ks_last_error(ctx, buf, sizeof(buf));
    throw std::runtime_error(std::string("ks_b200: ") + buf);
  }
}

// Device view of a PhantomCiphertext: data [size][local limbs][N].
struct CiphertextView {
  uint64_t *data;
  size_t size;                // number of polynomials (2, or 3 after a multiply)
  size_t coeff_modulus_size;  // Ql over all ranks
  size_t poly_modulus_degree;
};

// One context per GPU (reference MultiGpuContext, nccl_comm.cuh:42-54).
class MultiGpuContext {
 public:
  MultiGpuContext(const ks_params &prm, const std::vector<int> &dev_ids) {
    ctxs_.assign(dev_ids.size(), nullptr);
    check(ks_ctx_create_all(&prm, dev_ids.data(), (int)dev_ids.size(), ctxs_.data()), nullptr);
    streams_.assign(dev_ids.size(), nullptr);
    for (size_t i = 0; i < dev_ids.size(); ++i) {
      cudaSetDevice(dev_ids[i]);
      cudaStreamCreateWithFlags(&streams_[i], cudaStreamNonBlocking);
    }
    n_gpus = (int)dev_ids.size();
  }
  // One rank of a multi-process job; nccl_id from ks_nccl_unique_id on rank 0.
  MultiGpuContext(const ks_params &prm, int device, int rank, int world, const void *nccl_id) {
    ctxs_.assign(1, nullptr);
    check(ks_ctx_create(&prm, device, rank, world, nccl_id, &ctxs_[0]), nullptr);
    cudaSetDevice(device);
    streams_.assign(1, nullptr);
    cudaStreamCreateWithFlags(&streams_[0], cudaStreamNonBlocking);
    n_gpus = world;
  }
  ~MultiGpuContext() { destroy(); }
  MultiGpuContext(const MultiGpuContext &) = delete;
  MultiGpuContext &operator=(const MultiGpuContext &) = delete;

  void destroy() {
    for (auto s : streams_)
      if (s) cudaStreamDestroy(s);
    streams_.clear();
    for (auto c : ctxs_)
      if (c) ks_ctx_destroy(c);
    ctxs_.clear();
  }
  ks_ctx *ctx(int gpu_id) const { return ctxs_.size() == 1 ? ctxs_[0] : ctxs_[gpu_id]; }
  cudaStream_t stream(int gpu_id) const {
    return streams_.size() == 1 ? streams_[0] : streams_[gpu_id];
  }
  void sync(int gpu_id) const {
    if (cudaStreamSynchronize(stream(gpu_id)) != cudaSuccess)
      throw std::runtime_error("ks_b200: stream synchronisation failed");
  }

  int n_gpus = 0;

 private:
  std::vector<ks_ctx *> ctxs_;
  std::vector<cudaStream_t> streams_;
};

// encrypted (c0, c1) += KS(local_c2) with the relinearisation key.
inline void keyswitching_input_broadcast(MultiGpuContext &mc, int gpu_id,
                                         CiphertextView &encrypted, const uint64_t *local_c2,
                                         size_t total_limbs) {
  check(ks_keyswitch_add(mc.ctx(gpu_id), local_c2, encrypted.data, (int)total_limbs, KS_KEY_RELIN,
                         0, mc.stream(gpu_id)),
        mc.ctx(gpu_id));
  mc.sync(gpu_id);
}

inline void rotation_input_broadcast(MultiGpuContext &mc, int gpu_id, CiphertextView &encrypted,
                                     uint32_t galois_elt, size_t total_limbs) {
  check(ks_apply_galois(mc.ctx(gpu_id), encrypted.data, (int)total_limbs, galois_elt,
                        mc.stream(gpu_id)),
        mc.ctx(gpu_id));
  mc.sync(gpu_id);
}

inline void keyswitching_output_aggregation(MultiGpuContext &mc, int gpu_id,
                                            CiphertextView &encrypted, const uint64_t *c2) {
  keyswitching_input_broadcast(mc, gpu_id, encrypted, c2, encrypted.coeff_modulus_size);
}

inline void allgather_c2_limbs(MultiGpuContext &mc, int gpu_id, const uint64_t *local_c2,
                               uint64_t *full_c2, size_t total_limbs) {
  check(ks_allgather_limbs(mc.ctx(gpu_id), local_c2, full_c2, (int)total_limbs,
                           mc.stream(gpu_id)),
        mc.ctx(gpu_id));
  mc.sync(gpu_id);
}

// Phantom-style evaluator for one GPU / rank.
class Evaluator {
 public:
  Evaluator(MultiGpuContext &mc, int gpu_id) : mc_(mc), g_(gpu_id) {}
  void rotate_vector_inplace(CiphertextView &ct, int step) {
    check(ks_rotate(mc_.ctx(g_), ct.data, (int)ct.coeff_modulus_size, step, mc_.stream(g_)),
          mc_.ctx(g_));
    mc_.sync(g_);
  }
  void relinearize_inplace(CiphertextView &ct) {
    if (ct.size != 3) throw std::runtime_error("ks_b200: relinearize expects size 3");
    check(ks_relinearize(mc_.ctx(g_), ct.data, (int)ct.coeff_modulus_size, mc_.stream(g_)),
          mc_.ctx(g_));
    mc_.sync(g_);
    ct.size = 2;
  }
  void apply_galois_inplace(CiphertextView &ct, uint32_t galois_elt) {
    check(ks_apply_galois(mc_.ctx(g_), ct.data, (int)ct.coeff_modulus_size, galois_elt,
                          mc_.stream(g_)),
          mc_.ctx(g_));
    mc_.sync(g_);
  }
  // Phantom rescale_to_next (reference dist_rescale_to_next_inplace,
  // distributed_eval.cu:265-273): out receives ct / q_last at one level down
  // (out.coeff_modulus_size = ct.coeff_modulus_size - 1, separate buffer).
  void rescale_to_next(const CiphertextView &ct, CiphertextView &out) {
    check(ks_rescale(mc_.ctx(g_), ct.data, (int)ct.coeff_modulus_size, out.data, mc_.stream(g_)),
          mc_.ctx(g_));
    mc_.sync(g_);
  }
  // Hoisted rotations: outs[i] = ct rotated by steps[i], one ModUp shared.
  void rotate_hoisted(const CiphertextView &ct, const int *steps, int n, uint64_t *const *outs) {
    check(ks_rotate_hoisted(mc_.ctx(g_), ct.data, (int)ct.coeff_modulus_size, steps, n, outs,
                            mc_.stream(g_)),
          mc_.ctx(g_));
    mc_.sync(g_);
  }
  // Ciphertext x plaintext matmul by BSGS diagonals (ks_bsgs_matmul), the
  // product NEXUS's BERT layers run (reference bert_matmul_pipeline.cu:7-15):
  // y[o] = sum_g rot_{g B unit}(sum_i sum_b pts[((o n_in + i) G + g) B + b] * rot_{b unit}(x[i]))
  // with B = n_baby, G = n_giant; pts are NTT-form diagonals [n_local][N].
  // The workspace is allocated and freed around the call.
  void matmul_bsgs(const std::vector<CiphertextView> &x, int unit, int n_baby, int n_giant,
                   const std::vector<const uint64_t *> &pts, std::vector<CiphertextView> &y) {
    if (x.empty() || y.empty()) throw std::runtime_error("ks_b200: empty matmul operand list");
    std::vector<const uint64_t *> xp;
    for (const CiphertextView &v : x) xp.push_back(v.data);
    std::vector<uint64_t *> yp;
    for (CiphertextView &v : y) yp.push_back(v.data);
    const int Ql = (int)x[0].coeff_modulus_size;
    ks_ctx *ctx = mc_.ctx(g_);
    const size_t words = ks_bsgs_workspace_words(ctx, Ql, (int)x.size(), n_baby);
    uint64_t *work = nullptr;
    if (words > 0 && cudaMalloc(reinterpret_cast<void **>(&work), words * sizeof(uint64_t)) !=
                         cudaSuccess)
      throw std::runtime_error("ks_b200: cannot allocate the matmul workspace");
    const int rc = ks_bsgs_matmul(ctx, xp.data(), nullptr, (int)x.size(), Ql, unit, n_baby,
                                  n_giant, 0, n_giant, pts.data(), yp.data(), (int)y.size(),
                                  work, mc_.stream(g_));
    const cudaError_t se = cudaStreamSynchronize(mc_.stream(g_));
    cudaFree(work);
    check(rc, ctx);
    if (se != cudaSuccess) throw std::runtime_error("ks_b200: stream synchronisation failed");
  }

 private:
  MultiGpuContext &mc_;
  int g_;
};

}  // namespace ks_b200
