// bf16 equivariant linear maps on tcgen05 tensor cores (sm_100a): the bf16 storage
// variant of fc_linear_fwd (dtype FC_BF16).
//
// y[(node, m), n] = scale_l * sum_k x[(node, m), k] * W_l[n, k] for every rank block l, with
// x, W and y in bf16 and the products accumulated in fp32 (tensor memory), rounded once to
// bf16 on the way out: the "bf16 tensor-core path" of the edge-expansion + linear-map
// workload, which moves half the bytes of the float32 maps (the maps are HBM-bound). Same
// layout as the float32 maps (o3/linear.py:88-128): each rank block of a row is (2l+1)
// components of f_in (f_out) channels, so for a fixed m the rows form a strided matrix,
// described to the TMA unit as a 3-D tensor (k, node, m).
//
// One CTA per 128-node x 128-column tile of one m (grid x: tiles, grid y: m). TMA loads
// 64-wide k slabs of x and W (bf16, 128-byte swizzle) into a 2-stage ring (three CTAs per
// SM overlap one another's loads, MMAs and stores); one thread issues
// tcgen05.mma.kind::f16 (both operands bf16) into a 128 x 128 fp32 accumulator; after the last
// slab every warp reads its 32 rows from tensor memory, scales, rounds to bf16, stages them
// in the freed operand buffers as two 128-byte-swizzled 64-column boxes and stores them with
// TMA (16-byte row stores when the output block is not 16-byte aligned). Every wait is bounded (FC_DEV_TIMEOUT); the MMAs are drained before the
// tensor memory is freed.
#include "fc_base.cuh"

#ifndef FC_HOST_EMU

#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>
#include <mutex>

namespace fc {
namespace lbf {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 64;  // bf16 per 128-byte swizzle row
constexpr int TILE_A = BM * BK * 2;
constexpr int TILE_B = BN * BK * 2;
constexpr int STAGE = TILE_A + TILE_B;
constexpr int STAGES = 2;  // k <= 128 per rank block here: two slabs; 3 CTAs fit an SM
constexpr int SMEM = STAGES * STAGE + 1024 + 128;
constexpr long long WAIT_LIMIT = 1ll << 22;

struct Args {
  int64_t nodes;
  int K, N;
  int n_col_tiles;
  int64_t row_tiles;
  const float* scale;   // this rank's scale (float32)
  __nv_bfloat16* out;   // first element of the output rank block
  int64_t out_ld, out_ms;
  int vec;              // aligned output block: staged TMA stores through map_c
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

// kind::f16 instruction descriptor: D fp32, A and B bf16, both K-major, M = 128, N = 128.
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

__global__ void __launch_bounds__(128, 3)
    lin_bf16_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_c, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile = blockIdx.x;
  const int ct = (int)(tile % a.n_col_tiles);
  const int64_t node0 = (tile / a.n_col_tiles) * BM;
  const int n0 = ct * BN, m = blockIdx.y;
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
          "l"(reinterpret_cast<uint64_t>(&map_a)), "r"(kt * BK), "r"((int)node0), "r"(m), "r"(fb)
          : "memory");
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
              "r"(smem_u32(st + TILE_A)),
          "l"(reinterpret_cast<uint64_t>(&map_b)), "r"(kt * BK), "r"(n0), "r"(fb)
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
  const bool ready = wait_parity(smem_u32(done), 0, a.status);
  asm volatile("tcgen05.fence::after_thread_sync;");
  const int64_t node = node0 + warp * 32 + lane;
  const float sc = *a.scale;
  __nv_bfloat16* orow = a.out + node * a.out_ld + (int64_t)m * a.out_ms;
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
    const int col = n0 + cb;
    if (a.vec) {
      if (!ready) continue;
      // staged for the TMA store: this warp's 32 rows as two 64-column boxes (128-byte rows,
      // 16-byte chunk c of row r at c ^ (r & 7)) in the operand stages, free after `done`
      uint8_t* box = smem + warp * 8192 + (cb >> 6) * 4096 + lane * 128;
      const int c0 = ((cb & 63) * 2) >> 4;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w4[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int j = 4 * q + t;
          const __nv_bfloat162 b2 =
              __floats2bfloat162_rn(sc * __uint_as_float(v[2 * j]), sc * __uint_as_float(v[2 * j + 1]));
          w4[t] = *reinterpret_cast<const uint32_t*>(&b2);
        }
        *reinterpret_cast<uint4*>(box + (((c0 + q) ^ (lane & 7)) << 4)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
      continue;
    }
    if (!ready || node >= a.nodes || col >= a.N) continue;
    // unaligned output block: element stores
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col + j < a.N) orow[col + j] = __float2bfloat16_rn(sc * __uint_as_float(v[j]));
  }
  if (a.vec) {
    // TMA stores of the warp's two boxes (rows beyond the nodes and columns beyond N are
    // clipped by the unit); the smem reads finish before the CTA exits
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0 && ready && node0 + warp * 32 < a.nodes) {
      for (int h = 0; h < 2; ++h) {
        const int x = n0 + 64 * h;
        if (x >= a.N) break;
        asm volatile(
            "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                reinterpret_cast<uint64_t>(&map_c)),
            "r"(smem_u32(smem + warp * 8192 + h * 4096)), "r"(x), "r"((int)(node0 + warp * 32)), "r"(m)
            : "memory");
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    __syncwarp();
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
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

}  // namespace lbf

// One rank block: x rows (node, m) at x + off + node * ld + m * ms (k contiguous), W (N, K)
// row-major bf16, y rows at y + out_off + node * out_ld + m * out_ms. Returns
// FC_ERR_UNSUPPORTED when a base or stride is not 16-byte aligned (TMA).
int lin_bf16_rank(const void* x, int64_t ld, int64_t off, int64_t ms, int M, int64_t nodes, const void* w, int K,
                  int N, const float* scale, void* y, int64_t out_ld, int64_t out_off, int64_t out_ms, int* status,
                  cudaStream_t s) {
  using namespace lbf;
  if (nodes <= 0 || M <= 0 || N <= 0) return 0;
  if (!encode_fn()) return FC_ERR_UNSUPPORTED;
  const __nv_bfloat16* xa = reinterpret_cast<const __nv_bfloat16*>(x) + off;
  if ((reinterpret_cast<uintptr_t>(xa) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) || (ld % 8) ||
      (M > 1 && (ms % 8)) || (K % 8))
    return FC_ERR_UNSUPPORTED;
  CUtensorMap ma, mb;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)nodes, (cuuint64_t)M};
    const cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)(M > 1 ? ms : ld * nodes) * 2};
    const cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)BM, 1u};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode_fn()(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<__nv_bfloat16*>(xa), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return FC_ERR_UNSUPPORTED;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BN};
    const cuuint32_t estr[2] = {1, 1};
    if (encode_fn()(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return FC_ERR_UNSUPPORTED;
  }
  static bool configured[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FC_ERR_LAUNCH;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      if (cudaFuncSetAttribute(lin_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
        return FC_ERR_LAUNCH;
      configured[dev] = true;
    }
  }
  Args a;
  a.nodes = nodes;
  a.K = K;
  a.N = N;
  a.n_col_tiles = (N + BN - 1) / BN;
  a.row_tiles = (nodes + BM - 1) / BM;
  a.scale = scale;
  a.out = reinterpret_cast<__nv_bfloat16*>(y) + out_off;
  a.out_ld = out_ld;
  a.out_ms = M > 1 ? out_ms : 0;
  a.vec = ((reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && out_ld % 8 == 0 && (M == 1 || out_ms % 8 == 0)) ? 1 : 0;
  CUtensorMap mc;
  std::memset(&mc, 0, sizeof(mc));
  if (a.vec) {
    // (n, node, m) rows of the output block, box 64 x 32 x 1, 128-byte swizzle (the staging layout)
    const cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)nodes, (cuuint64_t)M};
    const cuuint64_t strides[2] = {(cuuint64_t)out_ld * 2, (cuuint64_t)(M > 1 ? out_ms : out_ld * nodes) * 2};
    const cuuint32_t box[3] = {64u, 32u, 1u};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode_fn()(&mc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a.out, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      a.vec = 0;
  }
  a.status = status;
  const int64_t tiles = a.row_tiles * a.n_col_tiles;
  if (tiles > 0x7fffffffLL || M > 65535) return FC_ERR_UNSUPPORTED;
  lin_bf16_kernel<<<dim3((unsigned)tiles, (unsigned)M), 128, SMEM, s>>>(ma, mb, mc, a);
  return fc_check_launch();
}

}  // namespace fc

#endif  // FC_HOST_EMU
