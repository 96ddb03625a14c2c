// Stream-ordered workspace of the library: one memory pool per device, created on first
// use, that keeps its memory between calls (release threshold = unlimited) so that the
// per-call workspace of the GEMMs (their tf32-split weights, when the caller passes no
// split of its own) is re-used instead of re-mapped. Under stream capture the
// allocations become graph allocation nodes.
#include "fc_base.cuh"

#ifndef FC_HOST_EMU

#include <mutex>

namespace fc {

static std::mutex g_pool_mu;
static cudaMemPool_t g_pools[64] = {};

static cudaMemPool_t device_pool() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_pool_mu);
  if (!g_pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t p = nullptr;
    if (cudaMemPoolCreate(&p, &props) != cudaSuccess) return nullptr;
    uint64_t keep = ~uint64_t(0);
    cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
    g_pools[dev] = p;
  }
  return g_pools[dev];
}

int fc_pool_alloc(void** ptr, size_t bytes, cudaStream_t s) {
  *ptr = nullptr;
  if (bytes == 0) return 0;
  cudaMemPool_t p = device_pool();
  if (!p) return FC_ERR_LAUNCH;
  return cudaMallocFromPoolAsync(ptr, bytes, p, s) == cudaSuccess ? 0 : FC_ERR_LAUNCH;
}

int fc_pool_free(void* ptr, cudaStream_t s) {
  if (!ptr) return 0;
  return cudaFreeAsync(ptr, s) == cudaSuccess ? 0 : FC_ERR_LAUNCH;
}

}  // namespace fc

#endif  // FC_HOST_EMU
