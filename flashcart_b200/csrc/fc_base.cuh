// Shared definitions of the flashcart_b200 kernels.
//
// Two builds use these headers:
//  * the CUDA build (nvcc, sm_100a): FC_HD = __host__ __device__, real kernels;
//  * the host-emulation build (g++ -DFC_HOST_EMU): the same per-thread bodies are
//    executed by plain host loops so that the CPU test suite checks the generated
//    arithmetic and the C-ABI layer without a GPU. The emulation library is a test
//    artefact only; the Python package never loads it.
#pragma once

#include <stdint.h>
#include <stddef.h>

#ifdef FC_HOST_EMU
#include <cstring>
#include <cmath>
#include <algorithm>
typedef void* cudaStream_t;
#define FC_HD
#define FC_DEV
#define FC_INLINE inline
#define __restrict__
#else
#include <cuda_runtime.h>
#define FC_HD __host__ __device__
#define FC_DEV __device__
#define FC_INLINE __forceinline__
#endif

#include "../../include/flashcart_b200.h"

namespace fc {

#ifndef FC_HOST_EMU
// The CUDA error behind the last failed launch of this thread, kept for the message of
// the entry point (cudaGetLastError clears it when the launcher checks it).
inline cudaError_t& fc_noted_error() {
  static thread_local cudaError_t e = cudaSuccess;
  return e;
}
// Stream-ordered device workspace from the library's per-device pool (pool.cu).
int fc_pool_alloc(void** ptr, size_t bytes, cudaStream_t s);
int fc_pool_free(void* ptr, cudaStream_t s);
// Launcher epilogue: FC_OK, or FC_ERR_LAUNCH with the CUDA error noted.
inline int fc_check_launch() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return 0;
  fc_noted_error() = e;
  return FC_ERR_LAUNCH;
}
#endif

// Device-side data errors, OR-ed into the caller's status word (if any).
FC_HD FC_INLINE void fc_flag(int* status, int code) {
  if (status == nullptr) return;
#if defined(__CUDA_ARCH__)
  atomicOr(status, code);
#else
  *status |= code;
#endif
}

template <typename T>
FC_HD FC_INLINE T fc_ldg(const T* p) {
#if defined(__CUDA_ARCH__)
  return __ldg(p);
#else
  return *p;
#endif
}

template <typename T>
FC_HD FC_INLINE void fc_atomic_add(T* p, T v) {
#if defined(__CUDA_ARCH__)
  atomicAdd(p, v);
#else
  *p += v;
#endif
}

template <typename T>
FC_HD FC_INLINE T fc_warp_sum(T v) {
#if defined(__CUDA_ARCH__)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
#endif
  return v;
}

FC_HD FC_INLINE bool fc_lane0() {
#if defined(__CUDA_ARCH__)
  return (threadIdx.x & 31) == 0;
#else
  return true;
#endif
}

// Add the D per-thread values `v` into a rank-block row (element q at base + q*Fx + cx).
//  * Fx == 1: every channel of the block adds into the same element: reduce over the
//    warp first, lane 0 issues one atomic per element (target must be zeroed);
//  * scatter: rows shared between CTAs (sender rows of a convolution): atomics;
//  * otherwise the row is owned by this thread: plain store.
// Must be reached by all 32 lanes of a warp together (inactive lanes pass zeros).
template <typename T, int D>
FC_HD FC_INLINE void fc_scatter_rows(T* base, int Fx, int cx, const T* v, bool active, bool scatter) {
  if (Fx == 1) {
#pragma unroll
    for (int q = 0; q < D; ++q) {
      const T s = fc_warp_sum(active ? v[q] : T(0));
      if (fc_lane0()) fc_atomic_add(base + q, s);
    }
  } else if (!active) {
    return;
  } else if (scatter) {
#pragma unroll
    for (int q = 0; q < D; ++q) fc_atomic_add(base + (int64_t)q * Fx + cx, v[q]);
  } else {
#pragma unroll
    for (int q = 0; q < D; ++q) base[(int64_t)q * Fx + cx] = v[q];
  }
}

inline int fc_round_up(int x, int m) { return (x + m - 1) / m * m; }

// Parameters of the fused edge-geometry kernels (edge_geometry.cu, fc_edge_geometry_*).
struct GeomParams {
  int l_max, n_radial, cosine, poly_order, use_shifts;
  int vectors_given;  // positions holds the (n_edges, 3) edge vectors themselves
  double r_min, r_max, r_cut;
  int64_t n_nodes, n_edges, n_cells;
};

}  // namespace fc
