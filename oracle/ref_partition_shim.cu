// ref_partition_shim.cu -- C wrappers around the reference's OWN partition
// code, compiled from the reference tree (not copied) by `make ref`:
//   src/multi_gpu/partition/rns_partition.cuh:29-107 (index math)
//   src/multi_gpu/partition/rns_partition.cu:26-128  (scatter/gather kernels)
// TEST INFRASTRUCTURE ONLY: tests use it to pin the product's partition
// math and copy kernels against the reference itself.
#include <cstdint>
#include <stdexcept>
#include <string>

#include "rns_partition.cuh"

using namespace nexus_multi_gpu;

extern "C" {
int ref_owner_of_limb(size_t j, int n) { return owner_of_limb(j, n); }
size_t ref_local_index_of_limb(size_t j, int n) { return local_index_of_limb(j, n); }
size_t ref_global_limb_index(int g, size_t loc, int n) { return global_limb_index(g, loc, n); }
size_t ref_n_local_limbs(int g, int n, size_t total) { return n_local_limbs(g, n, total); }
size_t ref_local_buf_offset(size_t poly, size_t loc, size_t nloc, size_t deg) {
  return local_buf_offset(poly, loc, nloc, deg);
}
size_t ref_global_buf_offset(size_t poly, size_t j, size_t total, size_t deg) {
  return global_buf_offset(poly, j, total, deg);
}
int ref_limbs_for_gpu(int g, int n, size_t total, size_t *out, int cap) {
  auto v = limbs_for_gpu(g, n, total);
  int k = 0;
  for (size_t x : v) {
    if (k < cap) out[k] = x;
    ++k;
  }
  return k;
}
// Device buffers; runs the reference kernels on the current device.
int ref_scatter(const uint64_t *global_buf, uint64_t *local_buf, size_t n_polys,
                size_t total, size_t degree, int g, int n) {
  try {
    scatter_ciphertext_to_gpu(global_buf, local_buf, n_polys, total, degree, g, n, 0);
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : -2;
  } catch (...) {
    return -1;
  }
}
int ref_gather(const uint64_t *local_buf, uint64_t *global_buf, size_t n_polys, size_t total,
               size_t degree, int g, int n) {
  try {
    gather_ciphertext_from_gpu(local_buf, global_buf, n_polys, total, degree, g, n, 0);
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : -2;
  } catch (...) {
    return -1;
  }
}
}
