// Newton-Schulz orthogonalisation of Muon updates on tcgen05 tensor cores (bf16).
//
// For a batch of matrices X (rows <= cols, bf16, row-major) and coefficients (a, b, c):
//     X <- X / max(||X||_F, eps)
//     repeat: G = X X^T;  U = b G + c G G;  X = a X + U X
// which is the reference's batched iteration (training/muon.py:27-61: bmm / baddbmm in
// bf16 with fp32 accumulation, every product rounded to bf16 once).
//
// All three products are D = alpha * A B^T + beta * C with A (M x K) and B (N x K) both
// K-major (row-major with k contiguous): G = X X^T takes A = B = X; G G takes A = B = G
// (G is symmetric); U X takes A = U and B = X^T, which a transpose kernel writes each
// step. One CTA computes a 128 x BN tile of one matrix of the batch: TMA loads 64-wide k
// slabs of A and B (128-byte swizzle, 3-D tensor maps with the batch as the outer
// dimension, zero fill outside the matrix), one thread issues tcgen05.mma.kind::f16
// (bf16 x bf16 -> fp32 in tensor memory, 4 instructions of k = 16 per slab) and manages the
// 4-stage ring, and the epilogue forms alpha * acc + beta * C in fp32 and rounds once to
// bf16, as cuBLAS does for bf16 bmm / baddbmm. Every wait is bounded.
#include "fc_base.cuh"

#ifndef FC_HOST_EMU

#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

namespace fc {
namespace ns {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 64;                 // bf16 elements per 128-byte swizzle row
constexpr int TILE_A = BM * BK * 2;    // 16 KB
constexpr int TILE_B = BN * BK * 2;    // 16 KB
constexpr int STAGE = TILE_A + TILE_B;
constexpr int STAGES = 4;
constexpr int SMEM = STAGES * STAGE + 1024 + 128;
constexpr long long WAIT_LIMIT = 1ll << 22;

struct GemmArgs {
  int M, N, K, batch;
  float alpha, beta;
  const __nv_bfloat16* C;   // (batch, M, N) or null
  __nv_bfloat16* D;         // (batch, M, N)
  int* status;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t make_desc(uint32_t saddr) {
  // K-major, 128-byte swizzle, descriptor version 1; 1024 B between 8-row groups.
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f16 instruction descriptor: D fp32, A and B bf16, both K-major, M = 128, N = BN.
__host__ __device__ constexpr uint32_t idesc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ bool wait_parity(uint32_t mbar, uint32_t parity, int* status) {
  for (long long it = 0; it < WAIT_LIMIT; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(mbar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  fc_flag(status, FC_DEV_TIMEOUT);
  return false;
}

__global__ void __launch_bounds__(128, 1)
    ns_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM, bz = blockIdx.z;
  const int nk = (a.K + BK - 1) / BK;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < STAGES; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&empty[s])));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(done)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;

  bool healthy = true;
  if (threadIdx.x == 0) {
    auto load = [&](int kt) {
      const int s = kt % STAGES;
      uint8_t* st = smem + s * STAGE;
      const uint32_t fb = smem_u32(&full[s]);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb), "r"(STAGE) : "memory");
      asm volatile(
          "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
              "r"(smem_u32(st)),
          "l"(reinterpret_cast<uint64_t>(&map_a)), "r"(kt * BK), "r"(m0), "r"(bz), "r"(fb)
          : "memory");
      asm volatile(
          "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
              "r"(smem_u32(st + TILE_A)),
          "l"(reinterpret_cast<uint64_t>(&map_b)), "r"(kt * BK), "r"(n0), "r"(bz), "r"(fb)
          : "memory");
    };
    const int pre = nk < STAGES ? nk : STAGES;
    for (int kt = 0; kt < pre; ++kt) load(kt);
    int issued = pre;
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % STAGES;
      if (healthy && !wait_parity(smem_u32(&full[s]), (uint32_t)((kt / STAGES) & 1), a.status)) healthy = false;
      asm volatile("tcgen05.fence::after_thread_sync;");
      if (healthy) {
        uint8_t* st = smem + s * STAGE;
        const uint64_t da = make_desc(smem_u32(st)), db = make_desc(smem_u32(st + TILE_A));
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t off = (uint64_t)((kk * 32) >> 4);
          const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
          asm volatile(
              "{\n\t.reg .pred p;\n\t"
              "setp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
              "l"(da + off), "l"(db + off), "r"(idesc_bf16()), "r"(acc));
        }
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(&empty[s]))
                   : "memory");
      if (issued < nk) {
        // the stage being refilled is the one just committed: wait for its MMAs
        if (healthy && !wait_parity(smem_u32(&empty[s]), (uint32_t)((kt / STAGES) & 1), a.status)) healthy = false;
        load(issued++);
      }
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(done))
                 : "memory");
  }
  __syncwarp();
  // all threads: wait for the accumulator, then alpha * acc + beta * C -> bf16
  const bool ready = wait_parity(smem_u32(done), 0, a.status);
  asm volatile("tcgen05.fence::after_thread_sync;");
  const int r = m0 + warp * 32 + lane;
#pragma unroll 1
  for (int cb = 0; cb < BN; cb += 32) {
    uint32_t v[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
          "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
          "=r"(v[30]), "=r"(v[31])
        : "r"(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)cb));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    if (ready && r < a.M) {
      const int64_t row = ((int64_t)bz * a.M + r) * a.N;
      for (int j = 0; j < 32; ++j) {
        const int n = n0 + cb + j;
        if (n < a.N) {
          float x = a.alpha * __uint_as_float(v[j]);
          if (a.C) x += a.beta * __bfloat162float(a.C[row + n]);
          a.D[row + n] = __float2bfloat16_rn(x);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
  }
}

// X / max(||X||_F, eps) per matrix (fp32 sum of squares of the input; the norm is
// rounded to bf16 and the quotient of the bf16 values rounded to bf16, as in bf16 torch).
template <typename Tin>
__global__ void ns_normalize_kernel(const Tin* __restrict__ in, __nv_bfloat16* __restrict__ out, int64_t per,
                                    int transposed, int rows_in, int cols_in, float eps) {
  const int64_t b = blockIdx.x;
  const Tin* src = in + b * per;
  __shared__ float red[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < per; i += blockDim.x) {
    const float x = __bfloat162float(__float2bfloat16_rn((float)src[i]));
    s += x * x;
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float nrm = __bfloat162float(__float2bfloat16_rn(sqrtf(red[0])));
  const float den = nrm > eps ? nrm : __bfloat162float(__float2bfloat16_rn(eps));
  __nv_bfloat16* dst = out + b * per;
  for (int64_t i = threadIdx.x; i < per; i += blockDim.x) {
    // output element i of the (rows <= cols) matrix; read transposed when the input is tall
    int64_t j = i;
    if (transposed) {
      const int64_t r = i / rows_in, c = i % rows_in;  // out (cols_in x rows_in) row r, column c
      j = c * cols_in + r;
    }
    const float x = __bfloat162float(__float2bfloat16_rn((float)src[j]));
    dst[i] = __float2bfloat16_rn(x / den);
  }
}

// (batch, R, C) -> (batch, C, R), bf16, 32 x 32 tiles through shared memory.
__global__ void ns_transpose_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int R,
                                    int C) {
  __shared__ __nv_bfloat16 t[32][33];
  const int64_t b = blockIdx.z;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) t[i][threadIdx.x] = in[(b * R + r) * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) out[(b * C + c) * R + r] = t[threadIdx.x][i];
  }
}

// ---------------------------------------------------------------------------------- host

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// (batch, rows, k) bf16, k contiguous; box (64, 128, 1) with 128-byte swizzle.
static bool encode_kmajor(CUtensorMap* map, const void* base, int rows, int k, int batch) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (k % 8) != 0) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)rows, (cuuint64_t)batch};
  const cuuint64_t strides[2] = {(cuuint64_t)k * 2, (cuuint64_t)k * rows * 2};
  const cuuint32_t box[3] = {(cuuint32_t)BK, 128u, 1u};
  const cuuint32_t estr[3] = {1, 1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int gemm(const __nv_bfloat16* A, const __nv_bfloat16* B, int M, int N, int K, int batch, float alpha,
                float beta, const __nv_bfloat16* C, __nv_bfloat16* D, int* status, cudaStream_t s) {
  CUtensorMap ma, mb;
  if (!encode_kmajor(&ma, A, M, K, batch) || !encode_kmajor(&mb, B, N, K, batch)) return FC_ERR_UNSUPPORTED;
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FC_ERR_LAUNCH;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(ns_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
      return FC_ERR_LAUNCH;
    configured[dev] = true;
  }
  GemmArgs g{M, N, K, batch, alpha, beta, C, D, status};
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, batch);
  ns_gemm_kernel<<<grid, 128, SMEM, s>>>(ma, mb, g);
  return fc_check_launch();
}

}  // namespace ns

// Newton-Schulz iterations of a batch of (rows <= cols after the optional transpose)
// matrices; see include/flashcart_b200.h.
int ns_orthogonalize(const void* update, int dtype_in, int64_t batch, int rows_in, int cols_in, const float* coeffs,
                     int steps, const float* polish, int polish_steps, float eps, void* out, int32_t* status,
                     cudaStream_t s) {
  using namespace ns;
  if (batch <= 0) return 0;
  if (!encode_fn()) return FC_ERR_UNSUPPORTED;
  const bool transposed = rows_in > cols_in;
  const int R = transposed ? cols_in : rows_in, C = transposed ? rows_in : cols_in;
  if (C % 8 != 0 || R % 8 != 0) return FC_ERR_UNSUPPORTED;  // 16-byte TMA strides
  const int64_t per = (int64_t)R * C;
  // workspace: X, X^T, G, U (bf16); the result is written to `out` in the caller's layout
  const size_t bytes = (size_t)batch * (2 * per + 2 * (int64_t)R * R) * 2;
  __nv_bfloat16* ws = nullptr;
  if (cudaMallocAsync(reinterpret_cast<void**>(&ws), bytes, s) != cudaSuccess) return FC_ERR_LAUNCH;
  __nv_bfloat16 *X = ws, *XT = X + batch * per, *G = XT + batch * per, *U = G + batch * (int64_t)R * R;
  int rc = 0;
  if (dtype_in == FC_F32)
    ns_normalize_kernel<float><<<(unsigned)batch, 256, 0, s>>>(reinterpret_cast<const float*>(update), X, per,
                                                              transposed, rows_in, cols_in, eps);
  else
    ns_normalize_kernel<__nv_bfloat16><<<(unsigned)batch, 256, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(update), X, per, transposed, rows_in, cols_in, eps);
  rc = fc_check_launch();
  for (int phase = 0; phase < 2 && rc == 0; ++phase) {
    const float* cf = phase == 0 ? coeffs : polish;
    const int n = phase == 0 ? steps : polish_steps;
    for (int it = 0; it < n && rc == 0; ++it) {
      // G = X X^T
      rc = gemm(X, X, R, R, C, (int)batch, 1.f, 0.f, nullptr, G, status, s);
      // U = b G + c G G
      if (rc == 0) rc = gemm(G, G, R, R, R, (int)batch, cf[2], cf[1], G, U, status, s);
      // X = a X + U X   (B operand = X^T, k = rows)
      if (rc == 0) {
        dim3 tg((C + 31) / 32, (R + 31) / 32, (unsigned)batch);
        ns_transpose_kernel<<<tg, dim3(32, 8), 0, s>>>(X, XT, R, C);
        rc = fc_check_launch();
      }
      if (rc == 0) rc = gemm(U, XT, R, C, R, (int)batch, 1.f, cf[0], X, X, status, s);
    }
  }
  // result in the caller's orientation
  if (rc == 0) {
    if (transposed) {
      dim3 tg((C + 31) / 32, (R + 31) / 32, (unsigned)batch);
      ns_transpose_kernel<<<tg, dim3(32, 8), 0, s>>>(X, reinterpret_cast<__nv_bfloat16*>(out), R, C);
      rc = fc_check_launch();
    } else {
      if (cudaMemcpyAsync(out, X, (size_t)batch * per * 2, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
        rc = FC_ERR_LAUNCH;
    }
  }
  if (cudaFreeAsync(ws, s) != cudaSuccess && rc == 0) rc = FC_ERR_LAUNCH;
  return rc;
}

}  // namespace fc

#endif  // FC_HOST_EMU
