// TEST INFRASTRUCTURE ONLY -- host-memory stand-ins for the CUDA runtime
// calls the reference's PagedKVCache / BlockAllocator make, so the
// UNMODIFIED reference page-table code (compiled from its sources into
// oracle/_ref/) runs on a CPU-only machine.  Device memory becomes host
// memory; copies become memcpy.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

extern "C" {
cudaError_t cudaMemGetInfo(size_t *free_b, size_t *total_b) {
  *free_b = (size_t)1 << 40;
  *total_b = (size_t)1 << 40;
  return cudaSuccess;
}
cudaError_t cudaMallocAsync(void **p, size_t n, cudaStream_t) {
  *p = std::calloc(1, n ? n : 1);
  return *p ? cudaSuccess : cudaErrorMemoryAllocation;
}
cudaError_t cudaFreeAsync(void *p, cudaStream_t) {
  std::free(p);
  return cudaSuccess;
}
cudaError_t cudaMalloc(void **p, size_t n) { return cudaMallocAsync(p, n, nullptr); }
cudaError_t cudaFree(void *p) { return cudaFreeAsync(p, nullptr); }
cudaError_t cudaHostAlloc(void **p, size_t n, unsigned int) { return cudaMallocAsync(p, n, nullptr); }
cudaError_t cudaFreeHost(void *p) { return cudaFreeAsync(p, nullptr); }
cudaError_t cudaMemcpyAsync(void *d, const void *s, size_t n, cudaMemcpyKind, cudaStream_t) {
  std::memcpy(d, s, n);
  return cudaSuccess;
}
const char *cudaGetErrorString(cudaError_t) { return "fake cudart"; }
}
