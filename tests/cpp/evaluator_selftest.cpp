// C++ caller of the library through include/ks_evaluator.hpp: the reference-
// named entry points must give the same words as the direct C ABI calls.
// Built and run by tests/test_gpu_cpp_shim.py on a GPU.
#include <cuda_runtime_api.h>

#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "ks_evaluator.hpp"

int main() {
  const int log_n = 13, N = 1 << log_n;
  const int bits[4] = {60, 40, 40, 60};
  uint64_t pr[4];
  ks_b200::check(ks_gen_primes(log_n, bits, 4, pr), nullptr);
  ks_params prm{(uint32_t)log_n, 3, pr, 1, pr + 3, KS_MODE_INPUT_BROADCAST, 1};
  ks_b200::MultiGpuContext mc(prm, std::vector<int>{0});
  ks_ctx *ctx = mc.ctx(0);
  std::vector<int8_t> sk(N);
  ks_b200::check(ks_secret_generate(log_n, 5, 0, sk.data()), nullptr);
  uint32_t elt = 0;
  ks_b200::check(ks_galois_elt(ctx, 3, &elt), ctx);
  ks_b200::check(ks_key_generate(ctx, KS_KEY_GALOIS, elt, sk.data(), 7, mc.stream(0)), ctx);
  ks_b200::check(ks_key_generate(ctx, KS_KEY_RELIN, 0, sk.data(), 8, mc.stream(0)), ctx);
  mc.sync(0);
  // random 3-poly ciphertext, canonical residues
  const size_t words = 3 * 3 * (size_t)N;
  std::vector<uint64_t> h(words);
  std::mt19937_64 rng(1);
  for (int p = 0; p < 3; ++p)
    for (int j = 0; j < 3; ++j)
      for (int k = 0; k < N; ++k) h[((size_t)p * 3 + j) * N + k] = rng() % pr[j];
  uint64_t *a = nullptr, *b = nullptr;
  cudaMalloc(reinterpret_cast<void **>(&a), words * 8);
  cudaMalloc(reinterpret_cast<void **>(&b), words * 8);
  // rotation: shim vs direct
  cudaMemcpy(a, h.data(), words * 8, cudaMemcpyHostToDevice);
  cudaMemcpy(b, h.data(), words * 8, cudaMemcpyHostToDevice);
  ks_b200::CiphertextView ct{a, 2, 3, (size_t)N};
  ks_b200::Evaluator ev(mc, 0);
  ev.rotate_vector_inplace(ct, 3);
  ks_b200::check(ks_apply_galois(ctx, b, 3, elt, nullptr), ctx);
  cudaDeviceSynchronize();
  std::vector<uint64_t> ra(words), rb(words);
  cudaMemcpy(ra.data(), a, 2 * 3 * (size_t)N * 8, cudaMemcpyDeviceToHost);
  cudaMemcpy(rb.data(), b, 2 * 3 * (size_t)N * 8, cudaMemcpyDeviceToHost);
  if (std::memcmp(ra.data(), rb.data(), 2 * 3 * (size_t)N * 8) != 0) {
    std::printf("rotation mismatch\n");
    return 1;
  }
  // relinearisation: reference-named input broadcast vs ks_relinearize
  cudaMemcpy(a, h.data(), words * 8, cudaMemcpyHostToDevice);
  cudaMemcpy(b, h.data(), words * 8, cudaMemcpyHostToDevice);
  ks_b200::CiphertextView ct3{a, 3, 3, (size_t)N};
  ks_b200::keyswitching_input_broadcast(mc, 0, ct3, a + 2 * 3 * (size_t)N, 3);
  ks_b200::check(ks_relinearize(ctx, b, 3, nullptr), ctx);
  cudaDeviceSynchronize();
  cudaMemcpy(ra.data(), a, 2 * 3 * (size_t)N * 8, cudaMemcpyDeviceToHost);
  cudaMemcpy(rb.data(), b, 2 * 3 * (size_t)N * 8, cudaMemcpyDeviceToHost);
  if (std::memcmp(ra.data(), rb.data(), 2 * 3 * (size_t)N * 8) != 0) {
    std::printf("relinearisation mismatch\n");
    return 1;
  }
  // rescale: Evaluator::rescale_to_next vs ks_rescale into separate buffers
  cudaMemcpy(a, h.data(), words * 8, cudaMemcpyHostToDevice);
  uint64_t *r1 = nullptr, *r2 = nullptr;
  cudaMalloc(reinterpret_cast<void **>(&r1), 2 * 2 * (size_t)N * 8);
  cudaMalloc(reinterpret_cast<void **>(&r2), 2 * 2 * (size_t)N * 8);
  ks_b200::CiphertextView cin{a, 2, 3, (size_t)N}, cout{r1, 2, 2, (size_t)N};
  ev.rescale_to_next(cin, cout);
  ks_b200::check(ks_rescale(ctx, a, 3, r2, nullptr), ctx);
  cudaDeviceSynchronize();
  cudaMemcpy(ra.data(), r1, 2 * 2 * (size_t)N * 8, cudaMemcpyDeviceToHost);
  cudaMemcpy(rb.data(), r2, 2 * 2 * (size_t)N * 8, cudaMemcpyDeviceToHost);
  if (std::memcmp(ra.data(), rb.data(), 2 * 2 * (size_t)N * 8) != 0) {
    std::printf("rescale mismatch\n");
    return 1;
  }
  cudaFree(r1);
  cudaFree(r2);
  // error path: unknown galois element
  bool threw = false;
  try {
    ks_b200::CiphertextView c2{a, 2, 3, (size_t)N};
    ev.apply_galois_inplace(c2, 11);
  } catch (const std::runtime_error &e) {
    threw = std::strstr(e.what(), "no galois key") != nullptr;
  }
  if (!threw) {
    std::printf("missing-key error not reported\n");
    return 1;
  }
  cudaFree(a);
  cudaFree(b);
  std::printf("evaluator shim ok\n");
  return 0;
}
