// Equivariant linear maps on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// C[r, n] = scale * sum_k A[r, k] * B(k, n) for one rank l, rows r = (node, m).
// One CTA (256 threads) owns a 128-row x 64-column output tile whose fp32
// accumulator lives in tensor memory (128 lanes x 64 columns); 96 KB of shared memory
// per CTA lets two CTAs share an SM and overlap their load / MMA / store phases. The k dimension is
// consumed in 32-element slabs (one 128-byte swizzle row): threads 0-127 load one
// 128-byte row of A each (rows are addressed through the (node, m) strides of the
// layout, so no tensor map is needed), threads 128-191 one row of the weight slab;
// every row is split into tf32 hi + lo parts in registers and written into
// 128B-swizzled K-major shared-memory tiles. The next slab is loaded into registers
// before the barrier and the MMAs of the current one, hiding the global latency. One thread issues, per 8-wide k step,
//     D += A_hi B_hi,  D += A_hi B_lo,  D += A_lo B_hi        ("3xTF32")
// which keeps the result at fp32 accuracy (the dropped lo*lo term is ~2^-22 relative).
// Two smem stages let the loads of slab k+1 overlap the MMAs of slab k; a stage is
// reused only after tcgen05.commit has signalled (through an mbarrier) that the MMAs
// reading it completed. Every wait is bounded: on expiry the kernel flags an error in
// the status word, still drains, frees its tensor memory and returns.
// The epilogue reads the accumulator with tcgen05.ld (warp w owns lanes 32*(w%4)..,
// column half w/4), transposes through shared memory (the operand stages are free by
// then) and stores whole rows with coalesced 16-byte stores, applying the scale.
#include "linear.cuh"

namespace fc {

#ifndef FC_HOST_EMU

namespace tc {

constexpr int BM = 128;   // rows per tile (TMEM lanes)
constexpr int BN = 64;    // output columns per tile (TMEM columns); 64 keeps smem at 96 KB -> 2 CTAs/SM
constexpr int BK = 32;    // k per stage: one 128-byte swizzle row of fp32/tf32
constexpr int TILE_A = BM * BK * 4;  // bytes of one A tile (16 KB)
constexpr int TILE_B = BN * BK * 4;  // bytes of one B tile (16 KB)
constexpr int STAGE = 2 * TILE_A + 2 * TILE_B;  // hi + lo of A and B
constexpr int NSTAGE = 2;
constexpr int SMEM_BYTES = NSTAGE * STAGE + 1024 /* alignment slack */ + 64;
static_assert(BM * (BN + 1) * 4 <= NSTAGE * STAGE, "epilogue transpose must fit in the operand stages");
constexpr long long WAIT_LIMIT = 1ll << 20;  // polls of try_wait (each may suspend briefly): ~0.1-1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// K-major, 128-byte swizzle, Blackwell descriptor (version 1); SBO = 1024 B between
// 8-row groups, LBO unused for swizzled K-major layouts (set to 1 as CUTLASS does).
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::tf32 instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = BN.
__host__ __device__ constexpr uint32_t idesc_tf32() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
      :
      : "r"(tmem_d), "l"(da), "l"(db), "r"(idesc_tf32()), "r"(accumulate));
}

__device__ __forceinline__ void commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar) : "memory");
}

// Bounded wait on an mbarrier phase; returns false on timeout.
__device__ __forceinline__ bool wait_parity(uint32_t mbar, uint32_t parity) {
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
  return false;
}

// Write 32 consecutive values of one tile row (128 bytes) into a 128B-swizzled tile:
// 16-byte chunk c of row r lands at chunk c ^ (r & 7).
__device__ __forceinline__ void put_row(uint8_t* tile, int r, const uint32_t* v) {
  uint8_t* row = tile + r * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 q = make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = q;
  }
}

template <bool SPLIT>
__device__ __forceinline__ void split_store(uint8_t* hi_tile, uint8_t* lo_tile, int r, const float* x) {
  uint32_t hi[32], lo[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    hi[k] = to_tf32(x[k]);
    if (SPLIT) lo[k] = to_tf32(x[k] - __uint_as_float(hi[k]));
  }
  put_row(hi_tile, r, hi);
  if (SPLIT) put_row(lo_tile, r, lo);
}

template <bool SPLIT>
__global__ void __launch_bounds__(256, 2) lin_tc_kernel(LinGemmArgs<float> a, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + NSTAGE * STAGE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + NSTAGE * STAGE + 32);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // 1-D grid, column tiles fastest: the CTAs that share a row tile of A run together,
  // so A is fetched from DRAM once and re-read from L2 for the other column tiles.
  const int n_col_tiles = (a.N + BN - 1) / BN;
  const int64_t row0 = (int64_t)(blockIdx.x / n_col_tiles) * BM;
  const int col0 = (int)(blockIdx.x % n_col_tiles) * BN;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&mbar[s])));
    asm volatile("fence.mbarrier_init.release.cluster;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;

  // Threads 0..127 load row tid of the A tile, threads 128..255 row tid-128 of the B tile.
  const bool is_a = tid < BM;
  const int trow = is_a ? tid : tid - BM;
  const bool b_slot = !is_a && trow < BN;  // threads BM+BN.. have no B row (BN < BM)
  const int64_t ar = row0 + trow;
  const int bn = col0 + trow;
  const bool ok = is_a ? (ar < a.R) : (b_slot && bn < a.N);
  const float* src = nullptr;
  if (is_a) src = ok ? a.a.row(ar) : a.a.p;
  else if (a.trans_b) src = a.w + (int64_t)(ok ? bn : 0) * a.ldw;
  const bool strided = !is_a && !a.trans_b;  // B(k, n) = W[k*ldw + n]: coalesced across threads

  auto load_slab = [&](int k0, float* x) {
    if (strided) {
#pragma unroll
      for (int k = 0; k < 32; ++k) x[k] = (ok && k0 + k < a.K) ? __ldg(a.w + (int64_t)(k0 + k) * a.ldw + bn) : 0.f;
    } else if (ok && k0 + BK <= a.K && ((reinterpret_cast<uintptr_t>(src + k0) & 15) == 0)) {
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(src + k0) + c);
        x[4 * c] = q.x; x[4 * c + 1] = q.y; x[4 * c + 2] = q.z; x[4 * c + 3] = q.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) x[k] = (ok && k0 + k < a.K) ? __ldg(src + k0 + k) : 0.f;
    }
  };

  const int nk = (a.K + BK - 1) / BK;
  bool healthy = true;
  float x[32];
  if (nk > 0 && (is_a || b_slot)) load_slab(0, x);
  for (int kt = 0; kt < nk; ++kt) {
    const int s = kt & 1;
    uint8_t* st = smem + s * STAGE;
    uint8_t *a_hi = st, *a_lo = st + TILE_A, *b_hi = st + 2 * TILE_A, *b_lo = st + 2 * TILE_A + TILE_B;
    if (kt >= NSTAGE && healthy) {
      // the MMAs issued NSTAGE slabs ago read this stage; wait until they completed
      if (!wait_parity(smem_u32(&mbar[s]), ((kt - NSTAGE) / NSTAGE) & 1)) {
        healthy = false;
        fc_flag(status, FC_DEV_TIMEOUT);
      }
    }
    if (is_a) split_store<SPLIT>(a_hi, a_lo, trow, x);
    else if (b_slot) split_store<SPLIT>(b_hi, b_lo, trow, x);
    if (kt + 1 < nk && (is_a || b_slot)) load_slab((kt + 1) * BK, x);  // in flight during the barrier and MMAs
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0 && healthy) {
      asm volatile("tcgen05.fence::after_thread_sync;");
      const uint64_t dah = make_desc(smem_u32(a_hi)), dal = make_desc(smem_u32(a_lo));
      const uint64_t dbh = make_desc(smem_u32(b_hi)), dbl = make_desc(smem_u32(b_lo));
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint64_t off = (uint64_t)((kk * 32) >> 4);  // advance 32 bytes along K inside the swizzle row
        mma_tf32(tmem, dah + off, dbh + off, (kt > 0 || kk > 0) ? 1u : 0u);
        if (SPLIT) {
          mma_tf32(tmem, dah + off, dbl + off, 1u);
          mma_tf32(tmem, dal + off, dbh + off, 1u);
        }
      }
      commit(smem_u32(&mbar[s]));
    }
  }
  // wait for the last commit (covers every earlier MMA of the issuing thread)
  if (healthy && nk > 0) {
    const int s = (nk - 1) & 1;
    if (!wait_parity(smem_u32(&mbar[s]), ((nk - 1) / NSTAGE) & 1)) {
      healthy = false;
      fc_flag(status, FC_DEV_TIMEOUT);
    }
  }
  // warp-collective tcgen05.ld below: make the outcome of the bounded waits block-uniform
  healthy = __syncthreads_and(healthy ? 1 : 0) != 0;
  asm volatile("tcgen05.fence::after_thread_sync;");
  // Epilogue: TMEM -> registers -> shared-memory transpose -> coalesced row stores.
  // Warp w reads TMEM lanes 32*(w%4).. (tile rows) and column half w/4.
  float* tr = reinterpret_cast<float*>(smem);  // [BM][TSTRIDE], reuses the operand stages
  constexpr int TSTRIDE = BN + 1;
  const int q = warp & 3, half = warp >> 2;
  const int trow_e = q * 32 + lane;
#pragma unroll 1
  for (int cb = half * (BN / 2); cb < (half + 1) * (BN / 2); cb += 32) {  // BN/2 = 32: one load
    uint32_t v[32];
    if (nk > 0 && healthy) {
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)cb;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
          "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
            "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
            "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
            "=r"(v[30]), "=r"(v[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0u;  // empty contraction (or an expired wait): zero
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) tr[trow_e * TSTRIDE + cb + j] = __uint_as_float(v[j]);
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  {
    const float sc = *a.scale;
    const int ncol = min(BN, a.N - col0);
    // each warp stores two rows per step: half-warp h writes row r + h, lane l columns 4(l%16)..+3
    constexpr int LPR = BN / 4;  // lanes per row
    for (int r0 = warp * (32 / LPR); r0 < BM; r0 += 8 * (32 / LPR)) {
      const int r = r0 + lane / LPR;
      const int64_t gr = row0 + r;
      if (gr < a.R) {
        float* crow = const_cast<float*>(a.c.row(gr)) + col0;
        const int c = 4 * (lane % LPR);
        if (c + 4 <= ncol && ((reinterpret_cast<uintptr_t>(crow + c) & 15) == 0)) {
          const float* t = tr + r * TSTRIDE + c;
          *reinterpret_cast<float4*>(crow + c) = make_float4(sc * t[0], sc * t[1], sc * t[2], sc * t[3]);
        } else {
          for (int j = c; j < c + 4 && j < ncol; ++j) crow[j] = sc * tr[r * TSTRIDE + j];
        }
      }
    }
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
  }
}

}  // namespace tc

int lin_gemm_tc(const LinGemmArgs<float>& a, bool split, int* status, cudaStream_t s) {
  if (a.R == 0 || a.N == 0) return 0;
  // TMA-fed persistent kernel where the layout allows it, else this one
  const int rc = lin_gemm_tma(a, split, status, s);
  if (rc != 1) return rc;
  if (a.act != 0) return FC_ERR_UNSUPPORTED;  // activations exist on the TMA path only
  const int64_t tiles = ((a.R + tc::BM - 1) / tc::BM) * ((a.N + tc::BN - 1) / tc::BN);
  if (tiles > 0x7fffffff) return FC_ERR_UNSUPPORTED;
  dim3 grid((unsigned)tiles);
  // the dynamic shared-memory opt-in is a per-device function attribute
  static bool configured[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FC_ERR_LAUNCH;
  if (!configured[dev][split ? 1 : 0]) {
    cudaError_t e = split ? cudaFuncSetAttribute(tc::lin_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 tc::SMEM_BYTES)
                          : cudaFuncSetAttribute(tc::lin_tc_kernel<false>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, tc::SMEM_BYTES);
    if (e != cudaSuccess) return FC_ERR_LAUNCH;
    configured[dev][split ? 1 : 0] = true;
  }
  if (split)
    tc::lin_tc_kernel<true><<<grid, 256, tc::SMEM_BYTES, s>>>(a, status);
  else
    tc::lin_tc_kernel<false><<<grid, 256, tc::SMEM_BYTES, s>>>(a, status);
  return fc_check_launch();
}

#else

int lin_gemm_tc(const LinGemmArgs<float>& a, bool, int*, cudaStream_t s) {
  if (a.act != 0) return FC_ERR_UNSUPPORTED;  // input activations exist on the GPU's TMA path only
  return lin_gemm<float>(a, s);
}

// host emulation of the split (same integer rounding to tf32 as the kernel)
int lin_presplit(const float* w, int ldw, int trans_b, int K, int N, float* out, cudaStream_t) {
  const int kp = (K + 3) & ~3;
  const int64_t total = (int64_t)N * kp;
  auto rnd = [](float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    u = (u + 0x1000u) & 0xFFFFE000u;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
  };
  for (int64_t i = 0; i < total; ++i) {
    const int n = (int)(i / kp), k = (int)(i - (int64_t)n * kp);
    const float x = k < K ? (trans_b ? w[(int64_t)n * ldw + k] : w[(int64_t)k * ldw + n]) : 0.f;
    out[i] = rnd(x);
    out[total + i] = rnd(x - out[i]);
  }
  return 0;
}

#endif

}  // namespace fc
