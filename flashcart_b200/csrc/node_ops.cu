// Fused RMS layer norm and equivariant gate of Cartesian node features (forward and
// first-order backward).
//
// One node row holds the rank blocks l = 0..L of F channels each, component axis outer
// and channels contiguous (row length (L+1)^2 F). Per row:
//   q_c  = sum_l w_l * x_{l,.,c}^T K_l x_{l,.,c}     (K_l the (l,l)->0 coupling)
//   ms   = (1/F) sum_c q_c,   r = (ms + eps)^(-1/2)
//   y    = x * r * gain_{l,c}
// and, for the backward with S = sum_{l,m,c} g x gain,
//   dx   = r gain g - (r^3 / 2) S (w_l / F) (K_l + K_l^T) x .
// One CTA per row and one thread per channel: each thread reads its (L+1)^2 components
// (coalesced over channels), the per-row sums are block reductions in a fixed order, so
// every thread sees the same r and S and the result does not depend on timing.
#include "fc_base.cuh"
#include "gen/rms_quad.cuh"
#include "tp_common.cuh"  // fc_warp_transpose_reduce

namespace fc {

template <typename T, int L>
FC_HD FC_INLINE T rms_row_quad(const T* v, const T* lw) {
  T q = lw[0] * rms_quad_l0<T>(v);
  if constexpr (L >= 1) q += lw[1] * rms_quad_l1<T>(v + 1);
  if constexpr (L >= 2) q += lw[2] * rms_quad_l2<T>(v + 4);
  if constexpr (L >= 3) q += lw[3] * rms_quad_l3<T>(v + 9);
  return q;
}

template <typename T, int L>
FC_HD FC_INLINE void rms_row_quad_grad(const T* v, T* gq) {
  rms_quad_grad_l0<T>(v, gq);
  if constexpr (L >= 1) rms_quad_grad_l1<T>(v + 1, gq + 1);
  if constexpr (L >= 2) rms_quad_grad_l2<T>(v + 4, gq + 4);
  if constexpr (L >= 3) rms_quad_grad_l3<T>(v + 9, gq + 9);
}

FC_HD FC_INLINE int rms_rank_of(int comp) { return comp < 1 ? 0 : comp < 4 ? 1 : comp < 9 ? 2 : 3; }

FC_HD FC_INLINE float rms_rsqrt(float x) {
#if defined(__CUDA_ARCH__)
  return rsqrtf(x);
#else
  return 1.0f / std::sqrt(x);
#endif
}
FC_HD FC_INLINE double rms_rsqrt(double x) {
#if defined(__CUDA_ARCH__)
  return rsqrt(x);
#else
  return 1.0 / std::sqrt(x);
#endif
}

#ifndef FC_HOST_EMU

// Sum over the CTA (blockDim a multiple of 32, at most 1024); every thread gets the total.
template <typename T>
__device__ __forceinline__ T rms_block_sum(T v, T* sh) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) sh[warp] = v;
  __syncthreads();
  T t = T(0);
  for (int k = 0; k < nw; ++k) t += sh[k];
  __syncthreads();
  return t;
}

template <typename T, int L>
__global__ void __launch_bounds__(1024) rms_fwd_kernel(const T* __restrict__ x, const T* __restrict__ gains,
                                                      const T* __restrict__ lw, T eps, int F, int64_t n_rows,
                                                      T* __restrict__ y, T* __restrict__ rstd) {
  constexpr int NC = (L + 1) * (L + 1);
  __shared__ T sh[32];
  const int c = threadIdx.x;
  const bool on = c < F;
  T lwv[L + 1];
  for (int l = 0; l <= L; ++l) lwv[l] = lw[l];
  for (int64_t row = blockIdx.x; row < n_rows; row += gridDim.x) {
    const T* xr = x + row * (int64_t)(NC * F) + c;
    T v[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) v[k] = on ? fc_ldg(xr + k * F) : T(0);
    const T tot = rms_block_sum<T>(on ? rms_row_quad<T, L>(v, lwv) : T(0), sh);
    const T r = rms_rsqrt(tot / T(F) + eps);
    if (on) {
      T* yr = y + row * (int64_t)(NC * F) + c;
#pragma unroll
      for (int k = 0; k < NC; ++k) yr[k * F] = v[k] * r * fc_ldg(gains + rms_rank_of(k) * F + c);
    }
    if (c == 0) rstd[row] = r;
  }
}

template <typename T, int L>
__global__ void __launch_bounds__(1024) rms_bwd_kernel(const T* __restrict__ g, const T* __restrict__ x,
                                                      const T* __restrict__ gains, const T* __restrict__ lw,
                                                      const T* __restrict__ rstd, int F, int64_t n_rows,
                                                      T* __restrict__ gx) {
  constexpr int NC = (L + 1) * (L + 1);
  __shared__ T sh[32];
  const int c = threadIdx.x;
  const bool on = c < F;
  T lwv[L + 1], gn[L + 1];
  for (int l = 0; l <= L; ++l) {
    lwv[l] = lw[l];
    gn[l] = on ? fc_ldg(gains + l * F + c) : T(0);
  }
  for (int64_t row = blockIdx.x; row < n_rows; row += gridDim.x) {
    const T* xr = x + row * (int64_t)(NC * F) + c;
    const T* gr = g + row * (int64_t)(NC * F) + c;
    T v[NC], gv[NC];
    T s = T(0);
#pragma unroll
    for (int k = 0; k < NC; ++k) {
      v[k] = on ? fc_ldg(xr + k * F) : T(0);
      gv[k] = on ? fc_ldg(gr + k * F) : T(0);
      s += gv[k] * v[k] * gn[rms_rank_of(k)];
    }
    const T S = rms_block_sum<T>(s, sh);
    const T r = fc_ldg(rstd + row);
    const T coef = T(0.5) * r * r * r * S / T(F);
    if (on) {
      T gq[NC];
      rms_row_quad_grad<T, L>(v, gq);
      T* o = gx + row * (int64_t)(NC * F) + c;
#pragma unroll
      for (int k = 0; k < NC; ++k) {
        const int l = rms_rank_of(k);
        o[k * F] = r * gn[l] * gv[k] - coef * lwv[l] * gq[k];
      }
    }
  }
}

template <typename T, int L>
static int rms_fwd_launch(const T* x, const T* gains, const T* lw, T eps, int F, int64_t n, T* y, T* rstd,
                          cudaStream_t s) {
  const int block = fc_round_up(F, 32);
  const int grid = (int)(n < ((int64_t)1 << 30) ? n : ((int64_t)1 << 30));
  rms_fwd_kernel<T, L><<<grid, block, 0, s>>>(x, gains, lw, eps, F, n, y, rstd);
  return fc_check_launch();
}
template <typename T, int L>
static int rms_bwd_launch(const T* g, const T* x, const T* gains, const T* lw, const T* rstd, int F, int64_t n,
                          T* gx, cudaStream_t s) {
  const int block = fc_round_up(F, 32);
  const int grid = (int)(n < ((int64_t)1 << 30) ? n : ((int64_t)1 << 30));
  rms_bwd_kernel<T, L><<<grid, block, 0, s>>>(g, x, gains, lw, rstd, F, n, gx);
  return fc_check_launch();
}

#else  // host emulation: the same per-channel arithmetic, rows and channels in loops

template <typename T, int L>
static int rms_fwd_launch(const T* x, const T* gains, const T* lw, T eps, int F, int64_t n, T* y, T* rstd,
                          cudaStream_t) {
  constexpr int NC = (L + 1) * (L + 1);
  for (int64_t row = 0; row < n; ++row) {
    T tot = T(0);
    for (int c = 0; c < F; ++c) {
      T v[NC];
      for (int k = 0; k < NC; ++k) v[k] = x[row * NC * F + k * F + c];
      tot += rms_row_quad<T, L>(v, lw);
    }
    const T r = rms_rsqrt(tot / T(F) + eps);
    for (int c = 0; c < F; ++c)
      for (int k = 0; k < NC; ++k)
        y[row * NC * F + k * F + c] = x[row * NC * F + k * F + c] * r * gains[rms_rank_of(k) * F + c];
    rstd[row] = r;
  }
  return 0;
}
template <typename T, int L>
static int rms_bwd_launch(const T* g, const T* x, const T* gains, const T* lw, const T* rstd, int F, int64_t n,
                          T* gx, cudaStream_t) {
  constexpr int NC = (L + 1) * (L + 1);
  for (int64_t row = 0; row < n; ++row) {
    T S = T(0);
    for (int c = 0; c < F; ++c)
      for (int k = 0; k < NC; ++k)
        S += g[row * NC * F + k * F + c] * x[row * NC * F + k * F + c] * gains[rms_rank_of(k) * F + c];
    const T r = rstd[row];
    const T coef = T(0.5) * r * r * r * S / T(F);
    for (int c = 0; c < F; ++c) {
      T v[NC], gq[NC];
      for (int k = 0; k < NC; ++k) v[k] = x[row * NC * F + k * F + c];
      rms_row_quad_grad<T, L>(v, gq);
      for (int k = 0; k < NC; ++k) {
        const int l = rms_rank_of(k);
        gx[row * NC * F + k * F + c] = r * gains[l * F + c] * g[row * NC * F + k * F + c] - coef * lw[l] * gq[k];
      }
    }
  }
  return 0;
}

#endif

template <typename T>
int rms_norm_fwd_dispatch(int l_max, const T* x, const T* gains, const T* lw, T eps, int F, int64_t n, T* y, T* rstd,
                          cudaStream_t s) {
  switch (l_max) {
    case 0: return rms_fwd_launch<T, 0>(x, gains, lw, eps, F, n, y, rstd, s);
    case 1: return rms_fwd_launch<T, 1>(x, gains, lw, eps, F, n, y, rstd, s);
    case 2: return rms_fwd_launch<T, 2>(x, gains, lw, eps, F, n, y, rstd, s);
    default: return rms_fwd_launch<T, 3>(x, gains, lw, eps, F, n, y, rstd, s);
  }
}
template <typename T>
int rms_norm_bwd_dispatch(int l_max, const T* g, const T* x, const T* gains, const T* lw, const T* rstd, int F,
                          int64_t n, T* gx, cudaStream_t s) {
  switch (l_max) {
    case 0: return rms_bwd_launch<T, 0>(g, x, gains, lw, rstd, F, n, gx, s);
    case 1: return rms_bwd_launch<T, 1>(g, x, gains, lw, rstd, F, n, gx, s);
    case 2: return rms_bwd_launch<T, 2>(g, x, gains, lw, rstd, F, n, gx, s);
    default: return rms_bwd_launch<T, 3>(g, x, gains, lw, rstd, F, n, gx, s);
  }
}

template int rms_norm_fwd_dispatch<float>(int, const float*, const float*, const float*, float, int, int64_t, float*,
                                          float*, cudaStream_t);
template int rms_norm_fwd_dispatch<double>(int, const double*, const double*, const double*, double, int, int64_t,
                                           double*, double*, cudaStream_t);
template int rms_norm_bwd_dispatch<float>(int, const float*, const float*, const float*, const float*, const float*,
                                          int, int64_t, float*, cudaStream_t);
template int rms_norm_bwd_dispatch<double>(int, const double*, const double*, const double*, const double*,
                                           const double*, int, int64_t, double*, cudaStream_t);

}  // namespace fc

// ------------------------------------------------------------------ equivariant gate
// y[n, (l, m), c] = v[n, (l, m), c] * gate[n, l, c] over the rank blocks of a row, and its
// first-order backward: grad_v = g * gate, grad_gate[n, l, c] = sum_m g v. One thread per
// (row, channel) walks the (L+1)^2 components, so every access is coalesced over channels.
namespace fc {

template <typename T, int L>
FC_HD FC_INLINE void gate_fwd_one(const T* __restrict__ v, const T* __restrict__ gate, T* __restrict__ y, int F,
                                  int64_t row, int c) {
  constexpr int NC = (L + 1) * (L + 1);
  const T* vr = v + row * (int64_t)(NC * F) + c;
  T* yr = y + row * (int64_t)(NC * F) + c;
  const T* gr = gate + row * (int64_t)((L + 1) * F) + c;
  T gl[L + 1];
  for (int l = 0; l <= L; ++l) gl[l] = fc_ldg(gr + l * F);
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int k = 0; k < NC; ++k) yr[k * F] = fc_ldg(vr + k * F) * gl[rms_rank_of(k)];
}

template <typename T, int L>
FC_HD FC_INLINE void gate_bwd_one(const T* __restrict__ g, const T* __restrict__ v, const T* __restrict__ gate,
                                  T* __restrict__ gv, T* __restrict__ ggate, int F, int64_t row, int c) {
  constexpr int NC = (L + 1) * (L + 1);
  const int64_t o = row * (int64_t)(NC * F) + c;
  const T* gr = gate + row * (int64_t)((L + 1) * F) + c;
  T gl[L + 1], acc[L + 1];
  for (int l = 0; l <= L; ++l) {
    gl[l] = fc_ldg(gr + l * F);
    acc[l] = T(0);
  }
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int k = 0; k < NC; ++k) {
    const int l = rms_rank_of(k);
    const T gk = fc_ldg(g + o + k * F);
    if (gv) gv[o + k * F] = gk * gl[l];
    acc[l] += gk * fc_ldg(v + o + k * F);
  }
  if (ggate)
    for (int l = 0; l <= L; ++l) ggate[row * (int64_t)((L + 1) * F) + l * F + c] = acc[l];
}

#ifndef FC_HOST_EMU
template <typename T, int L>
__global__ void gate_fwd_kernel(const T* v, const T* gate, T* y, int F, int64_t n) {
  const int64_t total = n * F;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x)
    gate_fwd_one<T, L>(v, gate, y, F, t / F, (int)(t % F));
}
template <typename T, int L>
__global__ void gate_bwd_kernel(const T* g, const T* v, const T* gate, T* gv, T* ggate, int F, int64_t n) {
  const int64_t total = n * F;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x)
    gate_bwd_one<T, L>(g, v, gate, gv, ggate, F, t / F, (int)(t % F));
}
static int gate_grid(int64_t threads) {
  const int64_t b = (threads + 255) / 256;
  return (int)(b < 148 * 64 ? (b < 1 ? 1 : b) : 148 * 64);
}
template <typename T, int L>
static int gate_fwd_launch(const T* v, const T* gate, T* y, int F, int64_t n, cudaStream_t s) {
  gate_fwd_kernel<T, L><<<gate_grid(n * F), 256, 0, s>>>(v, gate, y, F, n);
  return fc_check_launch();
}
template <typename T, int L>
static int gate_bwd_launch(const T* g, const T* v, const T* gate, T* gv, T* ggate, int F, int64_t n,
                           cudaStream_t s) {
  gate_bwd_kernel<T, L><<<gate_grid(n * F), 256, 0, s>>>(g, v, gate, gv, ggate, F, n);
  return fc_check_launch();
}
#else
template <typename T, int L>
static int gate_fwd_launch(const T* v, const T* gate, T* y, int F, int64_t n, cudaStream_t) {
  for (int64_t r = 0; r < n; ++r)
    for (int c = 0; c < F; ++c) gate_fwd_one<T, L>(v, gate, y, F, r, c);
  return 0;
}
template <typename T, int L>
static int gate_bwd_launch(const T* g, const T* v, const T* gate, T* gv, T* ggate, int F, int64_t n, cudaStream_t) {
  for (int64_t r = 0; r < n; ++r)
    for (int c = 0; c < F; ++c) gate_bwd_one<T, L>(g, v, gate, gv, ggate, F, r, c);
  return 0;
}
#endif

template <typename T>
int gate_fwd_dispatch(int l_max, const T* v, const T* gate, T* y, int F, int64_t n, cudaStream_t s) {
  switch (l_max) {
    case 0: return gate_fwd_launch<T, 0>(v, gate, y, F, n, s);
    case 1: return gate_fwd_launch<T, 1>(v, gate, y, F, n, s);
    case 2: return gate_fwd_launch<T, 2>(v, gate, y, F, n, s);
    default: return gate_fwd_launch<T, 3>(v, gate, y, F, n, s);
  }
}
template <typename T>
int gate_bwd_dispatch(int l_max, const T* g, const T* v, const T* gate, T* gv, T* ggate, int F, int64_t n,
                      cudaStream_t s) {
  switch (l_max) {
    case 0: return gate_bwd_launch<T, 0>(g, v, gate, gv, ggate, F, n, s);
    case 1: return gate_bwd_launch<T, 1>(g, v, gate, gv, ggate, F, n, s);
    case 2: return gate_bwd_launch<T, 2>(g, v, gate, gv, ggate, F, n, s);
    default: return gate_bwd_launch<T, 3>(g, v, gate, gv, ggate, F, n, s);
  }
}

template int gate_fwd_dispatch<float>(int, const float*, const float*, float*, int, int64_t, cudaStream_t);
template int gate_fwd_dispatch<double>(int, const double*, const double*, double*, int, int64_t, cudaStream_t);
template int gate_bwd_dispatch<float>(int, const float*, const float*, const float*, float*, float*, int, int64_t,
                                      cudaStream_t);
template int gate_bwd_dispatch<double>(int, const double*, const double*, const double*, double*, double*, int,
                                       int64_t, cudaStream_t);

}  // namespace fc

// ------------------------------------------------------------------ edge expansion
// out[e, k, c] = T[e, k] * h[e, r, c] for the (L+1)^2 stored components k of the
// direction moments T (rows of Irreps(L)), r = 0 when h is shared by all ranks (h: (E, C))
// or r = rank of k when h holds one row per rank (h: (E, L+1, C), the factorised form
// T_l (x) (h W_l^T) of an equivariant linear map applied to T (x) h). The output rows are
// the rank-block layout (rank l at l^2 C, component axis outer, channels contiguous).
// Backward: grad_h[e, r, c] = sum_{k of r} g[e, k, c] T[e, k] and grad_T[e, k] =
// sum_c g[e, k, c] h[e, r(k), c], the channel sum reduced over a warp (transpose-reduce).
namespace fc {

#ifndef FC_HOST_EMU
template <typename T, int L>
__global__ void edge_expand_fwd_kernel(const T* __restrict__ tm, const T* __restrict__ h, int F, int per_rank,
                                       int64_t n, T* __restrict__ out) {
  constexpr int NC = (L + 1) * (L + 1);
  const int64_t total = n * F;
  const int R = per_rank ? L + 1 : 1;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = t / F;
    const int c = (int)(t - e * F);
    T hv[L + 1];
    for (int r = 0; r <= L; ++r) hv[r] = r < R ? fc_ldg(h + (e * R + r) * F + c) : hv[0];
    T* o = out + e * (int64_t)(NC * F) + c;
#pragma unroll
    for (int k = 0; k < NC; ++k) o[k * F] = fc_ldg(tm + e * NC + k) * hv[per_rank ? rms_rank_of(k) : 0];
  }
}

// One warp per edge row; lane handles channels lane, lane + 32, ...
template <typename T, int L>
__global__ void edge_expand_bwd_kernel(const T* __restrict__ g, const T* __restrict__ tm, const T* __restrict__ h,
                                       int F, int per_rank, int64_t n, T* __restrict__ gt, T* __restrict__ gh) {
  constexpr int NC = (L + 1) * (L + 1);
  constexpr int NP = NC <= 1 ? 1 : NC <= 4 ? 4 : NC <= 8 ? 8 : NC <= 16 ? 16 : 32;
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int R = per_rank ? L + 1 : 1;
  for (int64_t e = warp0; e < n; e += nwarps) {
    T tv[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) tv[k] = fc_ldg(tm + e * NC + k);
    T acc[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) acc[k] = T(0);
    const T* gr = g + e * (int64_t)(NC * F);
    for (int c = lane; c < F; c += 32) {
      T hv[L + 1], ghv[L + 1];
      for (int r = 0; r <= L; ++r) {
        hv[r] = r < R ? fc_ldg(h + (e * R + r) * F + c) : hv[0];
        ghv[r] = T(0);
      }
#pragma unroll
      for (int k = 0; k < NC; ++k) {
        const int r = per_rank ? rms_rank_of(k) : 0;
        const T gk = fc_ldg(gr + k * F + c);
        acc[k] += gk * hv[r];
        ghv[r] += gk * tv[k];
      }
      if (gh)
        for (int r = 0; r < R; ++r) gh[(e * R + r) * F + c] = ghv[r];
    }
    if (gt) {
      const int comp = fc_warp_transpose_reduce<T, NP>(acc);
      if ((lane & (32 / NP - 1)) == 0 && comp < NC) gt[e * NC + comp] = acc[0];
    }
  }
}

template <typename T, int L>
static int edge_expand_fwd_launch(const T* tm, const T* h, int F, int per_rank, int64_t n, T* out, cudaStream_t s) {
  edge_expand_fwd_kernel<T, L><<<gate_grid(n * F), 256, 0, s>>>(tm, h, F, per_rank, n, out);
  return fc_check_launch();
}
template <typename T, int L>
static int edge_expand_bwd_launch(const T* g, const T* tm, const T* h, int F, int per_rank, int64_t n, T* gt, T* gh,
                                  cudaStream_t s) {
  edge_expand_bwd_kernel<T, L><<<gate_grid(n * 32), 256, 0, s>>>(g, tm, h, F, per_rank, n, gt, gh);
  return fc_check_launch();
}
#else
template <typename T, int L>
static int edge_expand_fwd_launch(const T* tm, const T* h, int F, int per_rank, int64_t n, T* out, cudaStream_t) {
  constexpr int NC = (L + 1) * (L + 1);
  const int R = per_rank ? L + 1 : 1;
  for (int64_t e = 0; e < n; ++e)
    for (int k = 0; k < NC; ++k)
      for (int c = 0; c < F; ++c)
        out[e * NC * F + k * F + c] = tm[e * NC + k] * h[(e * R + (per_rank ? rms_rank_of(k) : 0)) * F + c];
  return 0;
}
template <typename T, int L>
static int edge_expand_bwd_launch(const T* g, const T* tm, const T* h, int F, int per_rank, int64_t n, T* gt, T* gh,
                                  cudaStream_t) {
  constexpr int NC = (L + 1) * (L + 1);
  const int R = per_rank ? L + 1 : 1;
  for (int64_t e = 0; e < n; ++e) {
    if (gh)
      for (int r = 0; r < R; ++r)
        for (int c = 0; c < F; ++c) gh[(e * R + r) * F + c] = T(0);
    for (int k = 0; k < NC; ++k) {
      const int r = per_rank ? rms_rank_of(k) : 0;
      T a = T(0);
      for (int c = 0; c < F; ++c) {
        const T gk = g[e * NC * F + k * F + c];
        a += gk * h[(e * R + r) * F + c];
        if (gh) gh[(e * R + r) * F + c] += gk * tm[e * NC + k];
      }
      if (gt) gt[e * NC + k] = a;
    }
  }
  return 0;
}
#endif

template <typename T>
int edge_expand_fwd_dispatch(int l_max, const T* tm, const T* h, int F, int per_rank, int64_t n, T* out,
                             cudaStream_t s) {
  switch (l_max) {
    case 0: return edge_expand_fwd_launch<T, 0>(tm, h, F, per_rank, n, out, s);
    case 1: return edge_expand_fwd_launch<T, 1>(tm, h, F, per_rank, n, out, s);
    case 2: return edge_expand_fwd_launch<T, 2>(tm, h, F, per_rank, n, out, s);
    default: return edge_expand_fwd_launch<T, 3>(tm, h, F, per_rank, n, out, s);
  }
}
template <typename T>
int edge_expand_bwd_dispatch(int l_max, const T* g, const T* tm, const T* h, int F, int per_rank, int64_t n, T* gt,
                             T* gh, cudaStream_t s) {
  switch (l_max) {
    case 0: return edge_expand_bwd_launch<T, 0>(g, tm, h, F, per_rank, n, gt, gh, s);
    case 1: return edge_expand_bwd_launch<T, 1>(g, tm, h, F, per_rank, n, gt, gh, s);
    case 2: return edge_expand_bwd_launch<T, 2>(g, tm, h, F, per_rank, n, gt, gh, s);
    default: return edge_expand_bwd_launch<T, 3>(g, tm, h, F, per_rank, n, gt, gh, s);
  }
}

template int edge_expand_fwd_dispatch<float>(int, const float*, const float*, int, int, int64_t, float*,
                                             cudaStream_t);
template int edge_expand_fwd_dispatch<double>(int, const double*, const double*, int, int, int64_t, double*,
                                              cudaStream_t);
template int edge_expand_bwd_dispatch<float>(int, const float*, const float*, const float*, int, int, int64_t,
                                             float*, float*, cudaStream_t);
template int edge_expand_bwd_dispatch<double>(int, const double*, const double*, const double*, int, int, int64_t,
                                              double*, double*, cudaStream_t);

}  // namespace fc
