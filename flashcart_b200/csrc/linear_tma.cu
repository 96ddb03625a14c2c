// fp32 equivariant linear maps on tcgen05 tensor cores, fed by TMA (sm_100a).
//
// C[(m, node), n] = scale * sum_k A[(m, node), k] * B(k, n) for one rank l. The rows of
// A and C are the (node, m) rows of the rank block; for a fixed m they form a plain
// strided matrix, so A and C are described to the TMA unit as 3-D tensors
// (k | n, node, m) and one tile covers 128 nodes of one m. The weights B come as tf32
// hi / lo parts stored n-major (k contiguous): the caller's pre-split copy
// (fc_linear_fwd/bwd_presplit: the operator layer splits a frozen weight set once and
// keeps it), or else a split made per call into a stream-ordered workspace. TMA fetches
// them as well.
//
// One persistent CTA per SM (320 threads) walks its share of the output tiles:
//   warp 0     TMA producer: fp32 A slab (128 x 32) + B hi / lo slabs (BN x 32); optional L2
//              prefetch of A slabs further ahead (FC_TMA_PF_AHEAD, off: it did not raise the
//              measured rate)
//   warp 1     MMA issue (one thread): D += Ahi Bhi + Ahi Blo + Alo Bhi  ("3xTF32")
//   warps 2-5  splitters: round the A slab to tf32 and form its residual; for BN = 128
//              tiles both parts go to tensor memory (one lane quarter per warp) and the
//              MMAs read A from there, otherwise they go back to shared memory
//   warps 6-9  epilogue: TMEM -> registers -> scale -> swizzled staging -> TMA store
// Operand stages cycle through full (TMA landed) -> split (hi / lo ready) -> empty (MMAs
// done, tcgen05.commit) mbarriers. The k range of a tile is cut into units of 128 (KG
// slabs of 32); each
// unit accumulates into the next of a ring of TMEM accumulators (acc_full / acc_empty)
// and the epilogue adds the units in fp32 registers, so the epilogue of one unit
// overlaps the MMAs of the next. Every wait is bounded: on expiry
// the CTA raises FC_DEV_TIMEOUT in the status word, all roles stop, outstanding TMA
// loads and MMAs are drained, tensor memory is freed and the kernel returns.
//
// The 128-byte swizzle TMA applies to a 32-float box row (16-byte chunk c of row r at
// c ^ (r & 7)) is the K-major SW128 layout the UMMA descriptors describe, so the tiles
// go to the tensor cores as they land. Operand boxes start at k = 32 * slab (128-byte
// aligned x coordinate); store boxes start at n = 32 * chunk.
#include "linear.cuh"

#ifndef FC_HOST_EMU

#include <cuda.h>  // CUtensorMap and the driver enums (header only; the entry point is fetched at run time)

#include <algorithm>
#include <mutex>

namespace fc {
namespace tma {

constexpr int BM = 128;
constexpr int BK = 32;
#ifndef FC_TMA_SPLIT_WARPS
#define FC_TMA_SPLIT_WARPS 4
#endif
constexpr int SPLIT_WARPS = FC_TMA_SPLIT_WARPS;
constexpr int EPI_WARP0 = 2 + SPLIT_WARPS;
// 10 warps by default (4 splitters: splitting, not the MMAs, limited the slab rate with 2)
constexpr int THREADS = (EPI_WARP0 + 4) * 32;
constexpr int RING_BYTES = 192 * 1024;
constexpr int EPI_BYTES = 4 * 2 * 32 * 128;  // two 4 KB staging buffers per epilogue warp
constexpr int BAR_BYTES = 256;
constexpr long long WAIT_LIMIT = 1ll << 22;
// k slabs per accumulation unit. The tensor cores accumulate in fp32 but not with
// IEEE round-to-nearest at every step; over thousands of k the error grows beyond
// what an fp32 dot product shows. Each unit of KG slabs (128 k; as accurate against float64
// as 64 k, with half the epilogue handshakes) therefore starts a
// fresh TMEM accumulator, and the epilogue sums the units in fp32 registers.
#ifndef FC_TMA_KG
#define FC_TMA_KG 4
#endif
#ifndef FC_TMA_ATM64
#define FC_TMA_ATM64 1
#endif
#ifndef FC_TMA_WIDE64
#define FC_TMA_WIDE64 1
#endif
constexpr int KG = FC_TMA_KG;
constexpr int PF_SLABS = 4;   // k slabs per L2 prefetch box (512 bytes of each row)
#ifndef FC_TMA_PF_AHEAD
#define FC_TMA_PF_AHEAD 0
#endif
constexpr int PF_AHEAD = FC_TMA_PF_AHEAD;  // slabs between the prefetch cursor and the loads

template <int BN>
struct Cfg {
  static constexpr int TILE_A = BM * BK * 4;  // 16 KB
  static constexpr int TILE_B = BN * BK * 4;
  // ATM: the splitters write the tf32 hi / lo parts of A into tensor memory and the MMAs
  // read A from there, so shared memory carries A once (TMA in, splitters out) instead of
  // five times (TMA in, splitters in / hi out / lo out, three MMA reads). Taken for
  // BN = 128 (the node-level maps: measured 10-38% faster) and BN = 64 (the radial input
  // gradient 2944 -> 64 on 1.49 M rows: 6.08 -> 5.79 ms); BN = 256 tiles (k <= 64) keep A
  // in shared memory and all of tensor memory for accumulators.
  static constexpr bool ATM = BN == 128 || (BN == 64 && FC_TMA_ATM64);
  static constexpr int STAGE = ATM ? TILE_A + 2 * TILE_B : 2 * TILE_A + 2 * TILE_B;
  static constexpr int STAGES = ATM ? 4 : RING_BYTES / STAGE;
  static constexpr int A_COLS = ATM ? STAGES * 2 * BK : 0;  // tensor-memory A stages: hi | lo columns
  static constexpr int SMEM = STAGES * STAGE + EPI_BYTES + BAR_BYTES + 1024;
  // WIDE (BN = 64, 3xTF32): per k step one N = 128 MMA Ahi x [Bhi | Blo] (the two B parts
  // are adjacent in the stage) and one N = 64 MMA Alo x Bhi, instead of three N = 64 MMAs;
  // an N = 64 MMA costs about as much time as an N = 128 one. Each accumulation unit then
  // holds two 64-column halves that the epilogue adds.
  static constexpr bool WIDE = BN == 64 && FC_TMA_WIDE64;
  static constexpr int ACC_W = WIDE ? 2 * BN : BN;  // accumulator columns per unit (3xTF32)
  static constexpr int NACC = (512 - A_COLS) / ACC_W;  // TMEM accumulators in the ring (the other columns)
  static constexpr int TMEM_COLS = 512;
  static_assert(STAGES >= 2 && STAGES <= 8, "operand ring");
  static_assert(NACC >= 2, "accumulator ring");
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

struct Args {
  int64_t nodes;          // rows per m
  int M;                  // number of m (2l+1)
  int K, N, nk;           // reduction length, output columns, 32-wide k slabs
  int nu;                 // accumulation units per tile (ceil(nk / KG))
  int n_col_tiles;
  int64_t row_tiles;      // 128-node tiles per m
  int64_t n_tiles;
  const float* aux;       // ACT == 2: silu' of these values multiplies C; ACT == 3: added to C (laid out like C)
  int64_t aux_ld, aux_ms;
  const float* scale;     // per rank (indexed by rank_of_m)
  int n_ranks;            // weight sets in this launch (grouped launch: all ranks of a map)
  int rank_of_m[16];      // rank whose weights and scale row m of the tile uses
  int* status;
};

// The weights of every rank of a grouped launch (unused entries are never read).
struct BMaps {
  CUtensorMap hi[4];
  CUtensorMap lo[4];
  CUtensorMap r;  // ACT >= 2: the aux rows, laid out like C (loaded per 32 x 32 box by the epilogue)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 32 consecutive tensor-memory columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

#ifndef FC_TMA_INT_ROUND
#define FC_TMA_INT_ROUND 1
#endif
// fp32 -> tf32 (10 explicit mantissa bits), round to nearest with ties away from zero:
// add half a tf32 unit in the last place to the magnitude bits and clear the 13 dropped
// bits (integer add + and; a carry into the exponent is the correct rounding up to the
// next binade). Infinities are kept; a NaN whose payload sits only in the dropped bits
// becomes an infinity, and in the 3xTF32 split the residual x - hi is then NaN, so NaN
// still reaches the result.
__device__ __forceinline__ float round_tf32(float x) {
#if FC_TMA_INT_ROUND
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
#else
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
#endif
}

// SiLU and its derivative for the activation modes (fast exp / divide intrinsics; the
// argument is clamped to +-80, where the sigmoid is 0 or 1 to float32 precision).
__device__ __forceinline__ float act_sigmoid(float z) {
  z = fminf(fmaxf(z, -80.f), 80.f);
  return __fdividef(1.f, 1.f + __expf(-z));
}
__device__ __forceinline__ float act_silu(float z) { return z * act_sigmoid(z); }
__device__ __forceinline__ float act_dsilu(float z) {
  const float sg = act_sigmoid(z);
  return sg * (1.f + z * (1.f - sg));
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

template <int BN>
__host__ __device__ constexpr uint32_t idesc_tf32() {
  // D f32, A / B tf32, both K-major, M = 128, N = BN.
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// D (tensor memory) += A (tensor memory: row m in lane m, 8 k in consecutive columns) x B.
template <int BN>
__device__ __forceinline__ void mma_ta(uint32_t d, uint32_t ta, uint64_t db, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n"
      :
      : "r"(d), "r"(ta), "l"(db), "r"(idesc_tf32<BN>()), "r"(acc));
}

template <int BN>
__device__ __forceinline__ void mma(uint32_t d, uint64_t da, uint64_t db, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
      :
      : "r"(d), "l"(da), "l"(db), "r"(idesc_tf32<BN>()), "r"(acc));
}

__device__ __forceinline__ void commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar) : "memory");
}

__device__ __forceinline__ void arrive(uint32_t mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(mbar) : "memory");
}

__device__ __forceinline__ void arrive_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mbar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool test_parity(uint32_t mbar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(mbar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of the given parity. Gives up early (returning false)
// once another role has raised the CTA's abort flag.
__device__ __forceinline__ bool wait_parity(uint32_t mbar, uint32_t parity, volatile int* abort_flag,
                                            int* status) {
  for (long long it = 0; it < WAIT_LIMIT; ++it) {
    if (test_parity(mbar, parity)) return true;
    if ((it & 255) == 255 && *abort_flag) return false;
  }
  *abort_flag = 1;
  fc_flag(status, FC_DEV_TIMEOUT);
  return false;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                            uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(mbar)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}

// L2 prefetch of a box of A (no shared-memory destination): keeps more HBM traffic in
// flight than the shared-memory ring alone can hold.
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}

struct TileCoord {
  int col0, node0, m;
};

__device__ __forceinline__ TileCoord tile_coord(const Args& a, int64_t t) {
  const int ct = (int)(t % a.n_col_tiles);
  const int64_t rt = t / a.n_col_tiles;
  TileCoord c;
  c.col0 = ct;
  c.m = (int)(rt / a.row_tiles);
  c.node0 = (int)((rt - (int64_t)c.m * a.row_tiles) * BM);
  return c;
}

// ACT: 0 plain; 1 the splitters apply SiLU to A; 2 the epilogue multiplies by SiLU'(aux);
// 3 the epilogue adds aux (a residual laid out like C; it may be C itself).
template <int BN, bool SPLIT, int ACT>
__global__ void __launch_bounds__(THREADS, 1)
    lin_tma_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ BMaps bm,
                   const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_pf,
                   const Args a) {
  using C = Cfg<BN>;
  constexpr int S = C::STAGES;
  constexpr bool WIDE = C::WIDE && SPLIT;
  constexpr int AW = C::ACC_W;  // ring stride of the accumulators (the same without SPLIT: only WIDE fills 2 BN)
  constexpr int B_OFF = C::ATM ? C::TILE_A : 2 * C::TILE_A;  // B hi | lo after the A slab (and its lo half)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi = smem + S * C::STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi + EPI_BYTES);
  uint64_t* split = full + S;
  uint64_t* empty = split + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + C::NACC;
  uint64_t* drain = acc_empty + C::NACC;
  uint64_t* aux_bar = drain + 1;  // per epilogue warp and staging buffer: the aux box has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aux_bar + 8);
  static_assert((3 * S + 2 * C::NACC + 1 + 8) * 8 + 8 <= BAR_BYTES, "barrier area");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < S; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&split[s])), "r"(SPLIT_WARPS * 32));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&empty[s])));
    }
    for (int b = 0; b < C::NACC; ++b) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&acc_full[b])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 4;" ::"r"(smem_u32(&acc_empty[b])));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(drain)));
    for (int b = 0; b < 8; ++b) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&aux_bar[b])));
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;
  const int64_t my_tiles = (a.n_tiles > blockIdx.x) ? (a.n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_pf)) : "memory");
      for (int r = 0; r < a.n_ranks; ++r) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&bm.hi[r])) : "memory");
        if (SPLIT) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&bm.lo[r])) : "memory");
      }
      constexpr uint32_t bytes = C::TILE_A + (SPLIT ? 2 : 1) * C::TILE_B;
      // prefetch cursor: PF_AHEAD slabs ahead of the loads, one L2 prefetch per PF_SLABS slabs
      int64_t pi = 0;
      int pk = 0;
      auto advance_prefetch = [&]() {
        if (PF_AHEAD == 0 || pi >= my_tiles) return;
        if (pk % PF_SLABS == 0) {
          const TileCoord pc = tile_coord(a, blockIdx.x + pi * gridDim.x);
          tma_prefetch_3d(&map_pf, pk * BK, pc.node0, pc.m);
        }
        if (++pk == a.nk) {
          pk = 0;
          ++pi;
        }
      };
      for (int q = 0; q < PF_AHEAD; ++q) advance_prefetch();  // (no-op loop when PF_AHEAD is 0)
      int64_t g = 0;
      for (int64_t i = 0; i < my_tiles && !*abort_flag; ++i) {
        const TileCoord tc = tile_coord(a, blockIdx.x + i * gridDim.x);
        for (int kt = 0; kt < a.nk; ++kt, ++g) {
          advance_prefetch();
          const int s = (int)(g % S);
          if (g >= S && !wait_parity(smem_u32(&empty[s]), (uint32_t)(((g / S) - 1) & 1), abort_flag, a.status))
            break;
          uint8_t* st = smem + s * C::STAGE;
          const uint32_t fb = smem_u32(&full[s]);
          arrive_tx(fb, bytes);
          const int r = a.rank_of_m[tc.m];
          tma_load_3d(smem_u32(st), &map_a, kt * BK, tc.node0, tc.m, fb);
          tma_load_2d(smem_u32(st + B_OFF), &bm.hi[r], kt * BK, tc.col0 * BN, fb);
          if (SPLIT) tma_load_2d(smem_u32(st + B_OFF + C::TILE_B), &bm.lo[r], kt * BK, tc.col0 * BN, fb);
        }
      }
      // drain: the last load issued into every stage must have landed before the CTA exits
      for (int s = 0; s < S; ++s) {
        const int64_t uses = g > s ? (g - 1 - s) / S + 1 : 0;
        if (uses > 0) {
          for (long long it = 0; it < WAIT_LIMIT; ++it)
            if (test_parity(smem_u32(&full[s]), (uint32_t)((uses - 1) & 1))) break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issue
    if (lane == 0) {
      int64_t g = 0, u = 0;  // slab and accumulation-unit counters of this CTA
      bool ok = true;
      for (int64_t i = 0; i < my_tiles && ok && !*abort_flag; ++i) {
        for (int j = 0; j < a.nu && ok; ++j, ++u) {
          const int b = (int)(u % C::NACC);
          const int64_t v = u / C::NACC;
          if (v >= 1 && !wait_parity(smem_u32(&acc_empty[b]), (uint32_t)((v - 1) & 1), abort_flag, a.status)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;");
          const uint32_t d = tmem + (uint32_t)(C::A_COLS + b * AW);
          const int k_end = min(a.nk, (j + 1) * KG);
          for (int kt = j * KG; kt < k_end; ++kt, ++g) {
            const int s = (int)(g % S);
            if (!wait_parity(smem_u32(&split[s]), (uint32_t)((g / S) & 1), abort_flag, a.status)) {
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;");
            uint8_t* st = smem + s * C::STAGE;
            const uint64_t dbh = make_desc(smem_u32(st + B_OFF));
            const uint64_t dbl = make_desc(smem_u32(st + B_OFF + C::TILE_B));
            if constexpr (C::ATM) {
              const uint32_t tah = tmem + (uint32_t)(s * 2 * BK), tal = tah + (uint32_t)BK;
#pragma unroll
              for (int kk = 0; kk < BK / 8; ++kk) {
                const uint64_t off = (uint64_t)((kk * 32) >> 4);
                const uint32_t acc = (kt > j * KG || kk > 0) ? 1u : 0u;
                if (WIDE) {
                  mma_ta<2 * BN>(d, tah + kk * 8, dbh + off, acc);  // [Ahi Bhi | Ahi Blo]
                  mma_ta<BN>(d, tal + kk * 8, dbh + off, 1u);       // + Alo Bhi in the first half
                } else if (SPLIT) {
                  mma_ta<BN>(d, tal + kk * 8, dbh + off, acc);
                  mma_ta<BN>(d, tah + kk * 8, dbl + off, 1u);
                  mma_ta<BN>(d, tah + kk * 8, dbh + off, 1u);
                } else {
                  mma_ta<BN>(d, tah + kk * 8, dbh + off, acc);
                }
              }
            } else {
              const uint64_t dah = make_desc(smem_u32(st)), dal = make_desc(smem_u32(st + C::TILE_A));
#pragma unroll
              for (int kk = 0; kk < BK / 8; ++kk) {
                const uint64_t off = (uint64_t)((kk * 32) >> 4);
                const uint32_t acc = (kt > j * KG || kk > 0) ? 1u : 0u;
                if (WIDE) {
                  mma<2 * BN>(d, dah + off, dbh + off, acc);
                  mma<BN>(d, dal + off, dbh + off, 1u);
                } else if (SPLIT) {
                  mma<BN>(d, dal + off, dbh + off, acc);
                  mma<BN>(d, dah + off, dbl + off, 1u);
                  mma<BN>(d, dah + off, dbh + off, 1u);
                } else {
                  mma<BN>(d, dah + off, dbh + off, acc);
                }
              }
            }
            commit(smem_u32(&empty[s]));  // the stage is free once these MMAs have completed
          }
          if (ok) commit(smem_u32(&acc_full[b]));  // this unit's partial accumulator is complete
        }
      }
      // drain: every MMA issued by this thread completes before tensor memory is freed
      commit(smem_u32(drain));
      for (long long it = 0; it < WAIT_LIMIT; ++it)
        if (test_parity(smem_u32(drain), 0)) break;
    }
  } else if (warp < EPI_WARP0) {
    // ------------------------------------------------------------------ splitters
    const int t = threadIdx.x - 64;  // 0 .. 32 * SPLIT_WARPS - 1
    int64_t g = 0;
    for (int64_t i = 0; i < my_tiles && !*abort_flag; ++i) {
      bool ok = true;
      for (int kt = 0; kt < a.nk; ++kt, ++g) {
        const int s = (int)(g % S);
        if (!wait_parity(smem_u32(&full[s]), (uint32_t)((g / S) & 1), abort_flag, a.status)) {
          ok = false;
          break;
        }
        if constexpr (C::ATM) {
          // this warp's lane quarter: row r of the slab (128-byte swizzled, 16-byte chunk c
          // at c ^ (r & 7)) -> 32 hi and 32 lo columns of lane r in tensor-memory stage s
          const int r = (warp & 3) * 32 + lane;
          const uint8_t* row = smem + s * C::STAGE + r * 128;
          uint32_t h[32], l[32];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 x = *reinterpret_cast<const float4*>(row + ((c ^ (r & 7)) << 4));
            float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (ACT == 1) xs[e] = act_silu(xs[e]);
              const float hv = round_tf32(xs[e]);
              h[4 * c + e] = __float_as_uint(hv);
              l[4 * c + e] = __float_as_uint(SPLIT ? round_tf32(xs[e] - hv) : 0.f);
            }
          }
          const uint32_t ta = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(s * 2 * BK);
          tmem_st32(ta, h);
          if (SPLIT) tmem_st32(ta + BK, l);
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        } else {
          float4* hi = reinterpret_cast<float4*>(smem + s * C::STAGE);
          float4* lo = reinterpret_cast<float4*>(smem + s * C::STAGE + C::TILE_A);
#pragma unroll
          for (int j = 0; j < C::TILE_A / 16 / (32 * SPLIT_WARPS); ++j) {
            const int q = t + 32 * SPLIT_WARPS * j;
            float4 x = hi[q];
            if (ACT == 1) x = make_float4(act_silu(x.x), act_silu(x.y), act_silu(x.z), act_silu(x.w));
            const float4 h = make_float4(round_tf32(x.x), round_tf32(x.y), round_tf32(x.z), round_tf32(x.w));
            hi[q] = h;
            if (SPLIT)
              lo[q] = make_float4(round_tf32(x.x - h.x), round_tf32(x.y - h.y), round_tf32(x.z - h.z),
                                  round_tf32(x.w - h.w));
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        arrive(smem_u32(&split[s]));
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    float sc = a.scale[0];   // the scale of the current tile's rank
    uint8_t* stage0 = epi + (warp - EPI_WARP0) * 2 * 4096;
    int nbuf = 0;
    uint32_t aux_ph = 0;  // bit b: phase of this warp's aux barrier of staging buffer b
    int64_t u = 0;
    // one staged TMA store of 32 columns (this warp's 32 rows) from registers
    auto store_chunk = [&](const float* vals, int col, const TileCoord& tc) {
      float f[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) f[c] = sc * vals[c];
      if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");  // buffer used two stores ago
      __syncwarp();
      uint8_t* buf = stage0 + nbuf * 4096;
      uint8_t* row = buf + lane * 128;
      if constexpr (ACT >= 2) {
        // the aux box of this chunk (32 rows x 32 columns, laid out like C) comes into the
        // staging buffer by TMA, in the swizzled layout the store uses; each lane then reads
        // its row, applies it, and writes the result over it (the same bytes, same thread)
        const uint32_t rb = smem_u32(&aux_bar[(warp - EPI_WARP0) * 2 + nbuf]);
        if (lane == 0) {
          arrive_tx(rb, 4096);
          tma_load_3d(smem_u32(buf), &bm.r, col, tc.node0 + q * 32, tc.m, rb);
        }
        const uint32_t par = (aux_ph >> nbuf) & 1u;
        aux_ph ^= 1u << nbuf;
        if (!wait_parity(rb, par, abort_flag, a.status)) {
          // the load may still land: let it finish (bounded) before the buffer is reused
          for (long long it = 0; it < WAIT_LIMIT; ++it)
            if (test_parity(rb, par)) break;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 z = *reinterpret_cast<const float4*>(row + ((c ^ (lane & 7)) << 4));
          if constexpr (ACT == 2) {
            f[4 * c] *= act_dsilu(z.x);
            f[4 * c + 1] *= act_dsilu(z.y);
            f[4 * c + 2] *= act_dsilu(z.z);
            f[4 * c + 3] *= act_dsilu(z.w);
          } else {
            f[4 * c] += z.x;
            f[4 * c + 1] += z.y;
            f[4 * c + 2] += z.z;
            f[4 * c + 3] += z.w;
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<float4*>(row + ((c ^ (lane & 7)) << 4)) =
            make_float4(f[4 * c], f[4 * c + 1], f[4 * c + 2], f[4 * c + 3]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&map_c, smem_u32(buf), col, tc.node0 + q * 32, tc.m);
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
      nbuf ^= 1;
    };
    auto load32 = [&](uint32_t taddr, float* f) {
      uint32_t v[32];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
          "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
            "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
            "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
            "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int c = 0; c < 32; ++c) f[c] = __uint_as_float(v[c]);
    };
    for (int64_t i = 0; i < my_tiles && !*abort_flag; ++i) {
      const TileCoord tc = tile_coord(a, blockIdx.x + i * gridDim.x);
      sc = a.scale[a.rank_of_m[tc.m]];
      const int col0 = tc.col0 * BN;
      const int nchunks = min(BN, a.N - col0 + 31) / 32;
      bool ok = true;
      if (a.nu == 1) {
        // one unit: stream the accumulator out chunk by chunk
        const int b = (int)(u % C::NACC);
        if (!wait_parity(smem_u32(&acc_full[b]), (uint32_t)((u / C::NACC) & 1), abort_flag, a.status)) break;
        asm volatile("tcgen05.fence::after_thread_sync;");
        for (int cb = 0; cb < nchunks; ++cb) {
          float f[32];
          const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(C::A_COLS + b * AW + cb * 32);
          load32(ta, f);
          if constexpr (WIDE) {
            float f2[32];
            load32(ta + BN, f2);
#pragma unroll
            for (int c = 0; c < 32; ++c) f[c] += f2[c];
          }
          store_chunk(f, col0 + cb * 32, tc);
        }
        asm volatile("tcgen05.fence::before_thread_sync;");
        __syncwarp();
        if (lane == 0) arrive(smem_u32(&acc_empty[b]));
        ++u;
      } else if constexpr (BN <= 128) {
        // several units: sum their partial accumulators in fp32 registers
        float acc[BN];
#pragma unroll
        for (int c = 0; c < BN; ++c) acc[c] = 0.f;
        for (int j = 0; j < a.nu; ++j, ++u) {
          const int b = (int)(u % C::NACC);
          if (!wait_parity(smem_u32(&acc_full[b]), (uint32_t)((u / C::NACC) & 1), abort_flag, a.status)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll
          for (int cb = 0; cb < (WIDE ? 2 * BN : BN) / 32; ++cb) {
            float f[32];
            load32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(C::A_COLS + b * AW + cb * 32), f);
#pragma unroll
            for (int c = 0; c < 32; ++c) acc[(cb % (BN / 32)) * 32 + c] += f[c];
          }
          asm volatile("tcgen05.fence::before_thread_sync;");
          __syncwarp();
          if (lane == 0) arrive(smem_u32(&acc_empty[b]));
        }
        if (!ok) break;
#pragma unroll
        for (int cb = 0; cb < BN / 32; ++cb)
          if (cb < nchunks) store_chunk(acc + cb * 32, col0 + cb * 32, tc);
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
  }
}

// Weights -> n-major (k contiguous, row length kp) tf32 hi / lo parts; k >= K is zero.
__global__ void presplit_kernel(const float* __restrict__ w, int ldw, int trans_b, int K, int N, int kp,
                                float* __restrict__ hi, float* __restrict__ lo) {
  const int64_t total = (int64_t)N * kp;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(i / kp), k = (int)(i - (int64_t)n * kp);
    const float x = k < K ? (trans_b ? w[(int64_t)n * ldw + k] : w[(int64_t)k * ldw + n]) : 0.f;
    const float h = round_tf32(x);
    hi[i] = h;
    if (lo) lo[i] = round_tf32(x - h);
  }
}

// ---------------------------------------------------------------------------------- host

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DeviceState {
  bool ready = false;
  int sms = 0;
  bool attr_set[3][2][4] = {};
};

static std::mutex g_mu;
static EncodeTiledFn g_encode = nullptr;
static DeviceState g_dev[64];

static EncodeTiledFn encode_fn() {
  if (g_encode) return g_encode;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  return g_encode;
}

static DeviceState* device_state(int dev) {
  DeviceState& d = g_dev[dev];
  if (d.ready) return &d;
  if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return nullptr;
  d.ready = true;
  return &d;
}

// 3-D map over (inner, node, m) rows of a LinRows block; box (box_inner, box_rows, 1), 128-byte
// swizzle for operand / store boxes (box_inner 32) or none for L2 prefetch boxes.
static bool encode_rows(CUtensorMap* map, const float* base, int64_t inner, int64_t nodes, int M, int64_t ld,
                        int64_t ms, int box_rows, int box_inner = 32) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld & 3) || (M > 1 && (ms & 3)) || inner <= 0 || nodes <= 0)
    return false;
  const cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)nodes, (cuuint64_t)M};
  const cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)(M > 1 ? ms : ld * nodes) * 4};
  const cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     box_inner == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool encode_b(CUtensorMap* map, const float* base, int kp, int N, int box_n) {
  const cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)N};
  const cuuint64_t strides[1] = {(cuuint64_t)kp * 4};
  const cuuint32_t box[2] = {32, (cuuint32_t)box_n};
  const cuuint32_t estr[2] = {1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, bool SPLIT, int ACT>
static int launch(const CUtensorMap& ma, const BMaps& bm, const CUtensorMap& mc, const CUtensorMap& mpf,
                  const Args& args, DeviceState* ds, int grid, cudaStream_t s) {
  constexpr int bi = BN == 64 ? 0 : BN == 128 ? 1 : 2;
  if (!ds->attr_set[bi][SPLIT][ACT]) {
    if (cudaFuncSetAttribute(lin_tma_kernel<BN, SPLIT, ACT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<BN>::SMEM) != cudaSuccess)
      return FC_ERR_LAUNCH;
    ds->attr_set[bi][SPLIT][ACT] = true;
  }
  lin_tma_kernel<BN, SPLIT, ACT><<<grid, THREADS, Cfg<BN>::SMEM, s>>>(ma, bm, mc, mpf, args);
  return fc_check_launch();
}

// the activation modes instantiated: SiLU on the input for every tile width (the radial
// MLP's second and last layers), SiLU' epilogue for the 64-column input gradients, the
// residual-add epilogue for 64- and 128-column tiles (node-level maps)
template <int BN, bool SPLIT>
static int launch_act(int act, const CUtensorMap& ma, const BMaps& bm, const CUtensorMap& mc,
                      const CUtensorMap& mpf, const Args& args, DeviceState* ds, int grid, cudaStream_t s) {
  if (act == 1) return launch<BN, SPLIT, 1>(ma, bm, mc, mpf, args, ds, grid, s);
  if (act == 2) {
    if constexpr (BN == 64) return launch<BN, SPLIT, 2>(ma, bm, mc, mpf, args, ds, grid, s);
    return 1;
  }
  if (act == 3) {
    if constexpr (BN <= 128) return launch<BN, SPLIT, 3>(ma, bm, mc, mpf, args, ds, grid, s);
    return 1;
  }
  return launch<BN, SPLIT, 0>(ma, bm, mc, mpf, args, ds, grid, s);
}

}  // namespace tma

// One launch over the rank blocks a[0..n) of one map (n = 1: a single rank). The caller has
// checked that the blocks share K, N, row strides and node count and lie back to back in
// the row (a[l].off == a[l-1].off + a[l-1].M * ms), so one 3-D map over (k, node, m) with
// m_total rows covers all of them; each tile's m selects its rank's weights and scale.
// Returns 1 when the layout is not eligible (the caller uses another path).
static int run_tma(const LinGemmArgs<float>* a, int n, bool split, int* status, cudaStream_t s) {
  using namespace tma;
  int m_total = 0;
  for (int l = 0; l < n; ++l) m_total += a[l].a.M;
  if (n < 1 || n > 4 || m_total > 16) return 1;
  const LinGemmArgs<float>& a0 = a[0];
  if (a0.K <= 0 || a0.R <= 0 || a0.N <= 0 || a0.a.M != a0.c.M || a0.R % a0.a.M) return 1;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!encode_fn()) return 1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FC_ERR_LAUNCH;
  DeviceState* ds = device_state(dev);
  if (!ds) return FC_ERR_LAUNCH;
  const int64_t nodes = a0.R / a0.a.M;
  const int nk = (a0.K + BK - 1) / BK;
  const int nu = (nk + KG - 1) / KG;
  // 256-column tiles only when one unit covers k (their sum would need 256 registers)
  const int BN = (a0.N > 128 && nu == 1) ? 256 : a0.N > 64 ? 128 : 64;
  const int kp = (a0.K + 3) & ~3;
  if (nodes > 0x7fffffffLL) return 1;
  if (a0.act == 2 && BN != 64) return 1;  // the SiLU' epilogue is instantiated for 64-column tiles
  if (a0.act == 3 && BN > 128) return 1;   // the residual epilogue: 64- and 128-column tiles
  if (a0.act >= 2 && ((reinterpret_cast<uintptr_t>(a0.aux.p + a0.aux.off) & 15) || (a0.aux.ld & 3) ||
                      (m_total > 1 && (a0.aux.ms & 3)) || (a0.N & 3)))
    return 1;  // the epilogue reads aux rows as 16-byte vectors

  CUtensorMap ma, mc, mpf;
  BMaps bm;
  if (!encode_rows(&ma, a0.a.p + a0.a.off, a0.K, nodes, m_total, a0.a.ld, a0.a.ms, BM)) return 1;
  if (!encode_rows(&mpf, a0.a.p + a0.a.off, a0.K, nodes, m_total, a0.a.ld, a0.a.ms, BM, PF_SLABS * BK)) return 1;
  if (!encode_rows(&mc, a0.c.p + a0.c.off, a0.N, nodes, m_total, a0.c.ld, a0.c.ms, 32)) return 1;
  if (a0.act >= 2) {
    if (!encode_rows(&bm.r, a0.aux.p + a0.aux.off, a0.N, nodes, m_total, a0.aux.ld, a0.aux.ms, 32)) return 1;
  } else {
    bm.r = mc;  // unused
  }

  const size_t per_rank = (size_t)a0.N * kp * (split ? 2 : 1);
  float* ws = nullptr;
  if (!a0.bsplit && fc_pool_alloc(reinterpret_cast<void**>(&ws), per_rank * n * 4, s)) return FC_ERR_LAUNCH;
  int rc = 0;
  for (int l = 0; l < n && rc == 0; ++l) {
    // split once by the caller (lin_presplit layout), else into this call's workspace
    float* bhi = a0.bsplit ? const_cast<float*>(a[l].bsplit) : ws + per_rank * l;
    float* blo = split ? bhi + (size_t)a0.N * kp : nullptr;
    if (!encode_b(&bm.hi[l], bhi, kp, a0.N, BN) || (split && !encode_b(&bm.lo[l], blo, kp, a0.N, BN))) {
      rc = 1;
      break;
    }
    if (!split) bm.lo[l] = bm.hi[l];
    if (!a0.bsplit) {
      const int64_t total = (int64_t)a0.N * kp;
      const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4 * ds->sms);
      presplit_kernel<<<blocks, 256, 0, s>>>(a[l].w, a[l].ldw, a[l].trans_b, a0.K, a0.N, kp, bhi, blo);
      if (cudaGetLastError() != cudaSuccess) rc = FC_ERR_LAUNCH;
    }
  }
  if (rc == 0) {
    Args args;
    args.nodes = nodes;
    args.M = m_total;
    args.K = a0.K;
    args.N = a0.N;
    args.nk = nk;
    args.nu = nu;
    args.n_col_tiles = (a0.N + BN - 1) / BN;
    args.row_tiles = (nodes + BM - 1) / BM;
    args.n_tiles = args.row_tiles * m_total * args.n_col_tiles;
    args.scale = a0.scale;  // scales of consecutive ranks are consecutive (scale + l)
    args.n_ranks = n;
    for (int l = 0, m = 0; l < n; ++l)
      for (int j = 0; j < a[l].a.M; ++j) args.rank_of_m[m++] = l;
    for (int m = m_total; m < 16; ++m) args.rank_of_m[m] = 0;
    args.status = status;
    args.aux = a0.act >= 2 ? a0.aux.p + a0.aux.off : nullptr;
    args.aux_ld = a0.aux.ld;
    args.aux_ms = m_total > 1 ? a0.aux.ms : 0;
    const int act = a0.act;
    const int grid = (int)std::min<int64_t>(args.n_tiles, ds->sms);
    if (BN == 64)
      rc = split ? launch_act<64, true>(act, ma, bm, mc, mpf, args, ds, grid, s)
                 : launch_act<64, false>(act, ma, bm, mc, mpf, args, ds, grid, s);
    else if (BN == 128)
      rc = split ? launch_act<128, true>(act, ma, bm, mc, mpf, args, ds, grid, s)
                 : launch_act<128, false>(act, ma, bm, mc, mpf, args, ds, grid, s);
    else
      rc = split ? launch_act<256, true>(act, ma, bm, mc, mpf, args, ds, grid, s)
                 : launch_act<256, false>(act, ma, bm, mc, mpf, args, ds, grid, s);
  }
  // stream-ordered: the workspace returns to the pool after the kernels that read it
  if (ws && fc_pool_free(ws, s) && rc == 0) rc = FC_ERR_LAUNCH;
  return rc;
}

// Returns 1 when the shape / layout is not eligible (the caller uses the non-TMA kernel).
int lin_gemm_tma(const LinGemmArgs<float>& a, bool split, int* status, cudaStream_t s) {
  return run_tma(&a, 1, split, status, s);
}

// All ranks of one linear map in one launch when their blocks are uniform (same K, N,
// strides and node count, back to back in the row); 1 = not eligible.
int lin_gemm_tma_grouped(const LinGemmArgs<float>* a, int n, bool split, int* status, cudaStream_t s) {
  if (n < 2 || n > 4) return 1;
  const LinGemmArgs<float>& a0 = a[0];
  for (int l = 1; l < n; ++l) {
    const LinGemmArgs<float>& b = a[l];
    const LinGemmArgs<float>& p = a[l - 1];
    if (b.K != a0.K || b.N != a0.N || b.a.p != a0.a.p || b.c.p != a0.c.p || b.a.ld != a0.a.ld ||
        b.c.ld != a0.c.ld || b.a.ms != a0.a.ms || b.c.ms != a0.c.ms || b.a.M != b.c.M ||
        (b.bsplit == nullptr) != (a0.bsplit == nullptr) || b.scale != p.scale + 1)
      return 1;
    if (b.a.M < 1 || b.R % b.a.M || b.R / b.a.M != a0.R / a0.a.M) return 1;
    if (b.act != a0.act) return 1;
    if (a0.act >= 2 && (b.aux.p != a0.aux.p || b.aux.ld != a0.aux.ld || b.aux.ms != a0.aux.ms ||
                        b.aux.off != p.aux.off + (int64_t)p.aux.M * p.aux.ms))
      return 1;
    if (b.a.off != p.a.off + (int64_t)p.a.M * p.a.ms || b.c.off != p.c.off + (int64_t)p.c.M * p.c.ms) return 1;
  }
  return run_tma(a, n, split, status, s);
}

int lin_presplit(const float* w, int ldw, int trans_b, int K, int N, float* out, cudaStream_t s) {
  const int kp = (K + 3) & ~3;
  const int64_t total = (int64_t)N * kp;
  if (total == 0) return 0;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 4);
  tma::presplit_kernel<<<blocks, 256, 0, s>>>(w, ldw, trans_b, K, N, kp, out, out + total);
  return fc_check_launch();
}

}  // namespace fc

#endif  // FC_HOST_EMU
