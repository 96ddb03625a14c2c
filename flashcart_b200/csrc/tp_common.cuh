// Tensor-product kernel wrappers shared by every generated signature file.
//
// Thread mapping (forward, backward and double backward alike): one CTA per output
// row (a receiver node of a convolution, or a row of a dense product), one thread
// per feature channel (blockDim = F rounded up to a warp, at most FC_TP_BLOCK; wider
// F loops over channel blocks). For a convolution the CTA walks the receiver's
// CSR edge range; the edge index and the in2 / weight rows are uniform across the
// CTA, the in1 gather of the sender row and the weight row are coalesced over
// channels, the per-path outputs stay in registers and are stored once.
#pragma once
#include "fc_base.cuh"

#ifndef FC_P3_FWD_MINB
#define FC_P3_FWD_MINB 5
#endif
#ifndef FC_P3_BWD_MINB
#define FC_P3_BWD_MINB 4
#endif
#ifndef FC_TP_BLOCK
#define FC_TP_BLOCK 256
#endif

namespace fc {

template <typename T>
struct TpParams {
  const T* in1; const T* in2; const T* w; T* out;
  const int64_t* rowptr; const int64_t* idx_j;
  int64_t n_rows, n_in1;
  int F, F1, F2, shared_w, reduce;
  int* status;
};

template <typename T>
struct TpBwdParams {
  const T* g_out; const T* in1; const T* in2; const T* w;
  T* g_in1; T* g_in2; T* g_w;
  const int64_t* rowptr; const int64_t* idx_j;
  int64_t n_rows, n_in1;
  int F, F1, F2, shared_w, reduce;
  int* status;
  // dense channel-pair backward only (fc_tp_bwd_residual): added to the input gradients;
  // r_in1 covers the first r1_comps components of each in1 row (row stride r1_ld), r_in2
  // whole in2 rows; either may be null, r_in2 may be g_in2 itself
  const T* r_in1 = nullptr;
  const T* r_in2 = nullptr;
  int64_t r1_ld = 0;
  int r1_comps = 0;
};

template <typename T>
struct TpDbwdParams {
  const T* g_out; const T* in1; const T* in2; const T* w;
  const T* v1; const T* v2; const T* vw;
  T* d_g; T* d_in1; T* d_in2; T* d_w;
  const int64_t* rowptr; const int64_t* idx_j;
  int64_t n_rows, n_in1;
  int F, F1, F2, shared_w, reduce;
  int* status;
};

struct TpLaunch {
  int grid;   // CTAs
  int block;  // threads
};

// Function table of one compiled signature.
struct TpTable {
  int (*fwd_f32)(const TpParams<float>&, cudaStream_t);
  int (*fwd_f64)(const TpParams<double>&, cudaStream_t);
  int (*bwd_f32)(const TpBwdParams<float>&, cudaStream_t);
  int (*bwd_f64)(const TpBwdParams<double>&, cudaStream_t);
  int (*dbwd_f32)(const TpDbwdParams<float>&, cudaStream_t);
  int (*dbwd_f64)(const TpDbwdParams<double>&, cudaStream_t);
  int nacc;       // accumulators per channel (register budget indicator)
  // convolution kernels for edge attributes shared by all channels (may be null)
  int (*fwd2_f32)(const TpParams<float>&, cudaStream_t);
  int (*fwd2_f64)(const TpParams<double>&, cudaStream_t);
  int (*bwd2_f32)(const TpBwdParams<float>&, cudaStream_t);
  int (*bwd2_f64)(const TpBwdParams<double>&, cudaStream_t);
  // channel-pair convolution kernels (float32, F = 64 or 128; may be null)
  int (*fwd3_f32)(const TpParams<float>&, cudaStream_t);
  int (*bwd3_f32)(const TpBwdParams<float>&, cudaStream_t);
  // channel-pair dense products (no edges, both inputs with F = 64 or 128 channels,
  // weights per row; float32; may be null)
  int (*dpfwd_f32)(const TpParams<float>&, cudaStream_t);
  int (*dpbwd_f32)(const TpBwdParams<float>&, cudaStream_t);
  // four-channel convolution forward (float32, F = 128; null unless the signature's
  // paths fit one group)
  int (*fwd4_f32)(const TpParams<float>&, cudaStream_t);
};

struct TpSigEntry {
  int l1, l2, lo, sym, npaths;
  const TpTable* table;
};

inline int tp_block_for(int F) {
  int b = fc_round_up(F, 32);
  return b > FC_TP_BLOCK ? FC_TP_BLOCK : b;
}

#ifndef FC_HOST_EMU
// ------------------------------------------------------------------ device helpers

// Four consecutive shared-memory values (16-byte aligned) into registers.
__device__ __forceinline__ void ld4(const float* p, float* v) {
  const float4 q = *reinterpret_cast<const float4*>(p);
  v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
__device__ __forceinline__ void ld4(const double* p, double* v) {
  const double2 a = reinterpret_cast<const double2*>(p)[0], b = reinterpret_cast<const double2*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

// ---- packed float pairs (two adjacent channels per thread) for the channel-pair kernels:
// f32x2 arithmetic (one issue slot for two FP32 operations, sm_100), 8-byte loads/stores.
__device__ __forceinline__ float2 p2(float c) { return make_float2(c, c); }
__device__ __forceinline__ float2 pmul(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 pfma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 padd(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 ldg2(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }
__device__ __forceinline__ void st2(float* p, float2 v) { *reinterpret_cast<float2*>(p) = v; }
// Four consecutive floats (16-byte aligned) as two channel pairs, and back.
__device__ __forceinline__ void ld4p(const float* p, float2& a, float2& b) {
  const float4 q = *reinterpret_cast<const float4*>(p);
  a = make_float2(q.x, q.y);
  b = make_float2(q.z, q.w);
}
__device__ __forceinline__ void st4p(float* p, float2 a, float2 b) {
  *reinterpret_cast<float4*>(p) = make_float4(a.x, a.y, b.x, b.y);
}
// Vector atomic add of a channel pair into global memory (one reduction instruction).
__device__ __forceinline__ void red2(float* p, float2 v) { atomicAdd(reinterpret_cast<float2*>(p), v); }
// Minimum resident CTAs per SM of the channel-pair kernels by thread count (F/2 consumers
// + one producer warp): caps the registers a thread may use so that enough consumer
// warps stay resident (65,536 registers per SM / (CTAs x threads)).
// Small path groups (BIG false) run uncapped: their registers already allow many CTAs.
template <int NT, bool BIG> struct P3MinBlocks { static constexpr int fwd = 1, bwd = 1; };
template <> struct P3MinBlocks<64, true> { static constexpr int fwd = 6, bwd = 6; };
template <> struct P3MinBlocks<96, true> { static constexpr int fwd = FC_P3_FWD_MINB, bwd = FC_P3_BWD_MINB; };

// Barrier among the first `count` threads of the CTA (a multiple of 32) on barrier `id`.
__device__ __forceinline__ void fc_named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---- prefetch ring of the convolution kernels: 1-D bulk async copies (global -> this
// CTA's shared memory, no multicast) completing on an mbarrier per slot.
constexpr long long FC_RING_WAIT_LIMIT = 1ll << 22;

__device__ __forceinline__ uint32_t fc_smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void fc_mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(fc_smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fc_mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fc_mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(fc_smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void fc_mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fc_smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool fc_mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(fc_smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of the given parity; false on expiry (FC_DEV_TIMEOUT is
// raised and the CTA's abort flag set) or once another thread has set the abort flag.
__device__ __forceinline__ bool fc_mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status) {
  for (long long it = 0; it < FC_RING_WAIT_LIMIT; ++it) {
    if (fc_mbar_test(bar, parity)) return true;
    if ((it & 63) == 63 && *abort_flag) return false;
  }
  *abort_flag = 1;
  fc_flag(status, FC_DEV_TIMEOUT);
  return false;
}
// Bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned) into this CTA's
// shared memory, completing as transaction bytes on `bar`.
__device__ __forceinline__ void fc_bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          fc_smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(fc_smem_addr(bar))
      : "memory");
}

// Sum N values (N a power of two <= 32) over the 32 lanes of a warp with log2(N) halving
// exchanges: at offset o a lane keeps the upper half when its bit o is set and receives
// the partner's copy of that half. Afterwards v[0] of a lane holds the warp total of one
// component, returned as the index; 32/N consecutive lanes hold the same component.
template <typename T, int N>
__device__ __forceinline__ int fc_warp_transpose_reduce(T* v) {
  const int lane = threadIdx.x & 31;
  int comp = 0;
  int n = N;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      const int half = n >> 1;
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        if (i < half) {
          const T keep = up ? v[i + half] : v[i];
          const T send = up ? v[i] : v[i + half];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      if (up) comp += half;
      n = half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
  return comp;
}

// ------------------------------------------------------------------ device wrappers

template <typename T, typename S>
__global__ void __launch_bounds__(FC_TP_BLOCK) tp_fwd_kernel(TpParams<T> P) {
  for (int cb = 0; cb < P.F; cb += blockDim.x) {
    const int c = cb + threadIdx.x;
    if (c >= P.F) break;
    for (int64_t row = blockIdx.x; row < P.n_rows; row += gridDim.x) S::template fwd<T>(P, row, c);
  }
}

template <typename T, typename S>
__global__ void __launch_bounds__(FC_TP_BLOCK) tp_bwd_kernel(TpBwdParams<T> P) {
  for (int cb = 0; cb < P.F; cb += blockDim.x) {
    const int c = cb + threadIdx.x;
    const bool active = c < P.F;
    T keep[S::NP];
    for (int q = 0; q < S::NP; ++q) keep[q] = T(0);
    for (int64_t row = blockIdx.x; row < P.n_rows; row += gridDim.x)
      S::template bwd<T>(P, row, active ? c : 0, active, keep);
    if (P.shared_w && P.g_w != nullptr && active)
      for (int q = 0; q < S::NP; ++q) atomicAdd(P.g_w + (int64_t)q * P.F + c, keep[q]);
  }
}

template <typename T, typename S>
__global__ void __launch_bounds__(FC_TP_BLOCK) tp_dbwd_kernel(TpDbwdParams<T> P) {
  for (int cb = 0; cb < P.F; cb += blockDim.x) {
    const int c = cb + threadIdx.x;
    const bool active = c < P.F;
    T keep[S::NP];
    for (int q = 0; q < S::NP; ++q) keep[q] = T(0);
    for (int64_t row = blockIdx.x; row < P.n_rows; row += gridDim.x)
      S::template dbwd<T>(P, row, active ? c : 0, active, keep);
    if (P.shared_w && P.d_w != nullptr && active)
      for (int q = 0; q < S::NP; ++q) atomicAdd(P.d_w + (int64_t)q * P.F + c, keep[q]);
  }
}

inline int tp_grid_for(int64_t n_rows, bool shared_accumulate) {
  // One CTA per row; rows accumulating a shared weight gradient use a bounded grid so
  // that each thread folds many rows before its single atomic per path.
  int64_t g = n_rows;
  const int64_t cap = shared_accumulate ? 148 * 16 : ((int64_t)1 << 31) - 1;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

template <typename T, typename S>
int tp_fwd_launch(const TpParams<T>& P, cudaStream_t s) {
  if (P.n_rows == 0) return 0;
  tp_fwd_kernel<T, S><<<tp_grid_for(P.n_rows, false), tp_block_for(P.F), 0, s>>>(P);
  return fc_check_launch();
}
template <typename T, typename S>
int tp_bwd_launch(const TpBwdParams<T>& P, cudaStream_t s) {
  if (P.n_rows == 0) return 0;
  tp_bwd_kernel<T, S><<<tp_grid_for(P.n_rows, P.shared_w && P.g_w), tp_block_for(P.F), 0, s>>>(P);
  return fc_check_launch();
}
template <typename T, typename S>
int tp_dbwd_launch(const TpDbwdParams<T>& P, cudaStream_t s) {
  if (P.n_rows == 0) return 0;
  tp_dbwd_kernel<T, S><<<tp_grid_for(P.n_rows, P.shared_w && P.d_w), tp_block_for(P.F), 0, s>>>(P);
  return fc_check_launch();
}

#else
// ------------------------------------------------------------------ host emulation

template <typename T, typename S>
int tp_fwd_launch(const TpParams<T>& P, cudaStream_t) {
  for (int64_t row = 0; row < P.n_rows; ++row)
    for (int c = 0; c < P.F; ++c) S::template fwd<T>(P, row, c);
  return 0;
}
template <typename T, typename S>
int tp_bwd_launch(const TpBwdParams<T>& P, cudaStream_t) {
  for (int c = 0; c < P.F; ++c) {
    T keep[S::NP];
    for (int q = 0; q < S::NP; ++q) keep[q] = T(0);
    for (int64_t row = 0; row < P.n_rows; ++row) S::template bwd<T>(P, row, c, true, keep);
    if (P.shared_w && P.g_w != nullptr)
      for (int q = 0; q < S::NP; ++q) P.g_w[(int64_t)q * P.F + c] += keep[q];
  }
  return 0;
}
template <typename T, typename S>
int tp_dbwd_launch(const TpDbwdParams<T>& P, cudaStream_t) {
  for (int c = 0; c < P.F; ++c) {
    T keep[S::NP];
    for (int q = 0; q < S::NP; ++q) keep[q] = T(0);
    for (int64_t row = 0; row < P.n_rows; ++row) S::template dbwd<T>(P, row, c, true, keep);
    if (P.shared_w && P.d_w != nullptr)
      for (int q = 0; q < S::NP; ++q) P.d_w[(int64_t)q * P.F + c] += keep[q];
  }
  return 0;
}
#endif

}  // namespace fc

// Instantiate the launch table of a generated signature; NS::Ops supplies the bodies.
#ifndef FC_HOST_EMU
#define FC_CONV2_ENTRIES(NS)                                                              \
  , &NS::Ops::fwd2<float>, &NS::Ops::fwd2<double>, &NS::Ops::bwd2<float>, &NS::Ops::bwd2<double>, \
      &NS::Ops::fwd3, &NS::Ops::bwd3, &NS::Ops::dpfwd, &NS::Ops::dpbwd, NS::Ops::fwd4_fn
#else
#define FC_CONV2_ENTRIES(NS) , nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr
#endif
#define FC_DEFINE_TP_SIGNATURE(NAME, NS)                                                  \
  extern const TpTable tp_table_##NAME;                                                   \
  const TpTable tp_table_##NAME = {                                                       \
      &tp_fwd_launch<float, NS::Ops>,  &tp_fwd_launch<double, NS::Ops>,                   \
      &tp_bwd_launch<float, NS::Ops>,  &tp_bwd_launch<double, NS::Ops>,                   \
      &tp_dbwd_launch<float, NS::Ops>, &tp_dbwd_launch<double, NS::Ops>, NS::Ops::NACC    \
      FC_CONV2_ENTRIES(NS)};

#define FC_DECLARE_TP_SIGNATURE(NAME) extern const TpTable tp_table_##NAME
