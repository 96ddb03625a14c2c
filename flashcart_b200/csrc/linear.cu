// Equivariant linear maps (per-rank channel mixing), exact-arithmetic path.
//
// For rank l the map is a GEMM over the rows r = (n, m), m = 0..2l, whose operand
// rows are not uniformly strided: row (n, m) starts at n*ld + off_l + m*width. The
// kernels therefore address rows through (ld, off, mstride) and tile 64x64 outputs
// per CTA with a 16-deep k-slab in shared memory (256 threads, 4x4 per thread).
// grad_W folds rows in split-K fashion with one atomic per output element per CTA.
#include "linear.cuh"

namespace fc {

#ifndef FC_HOST_EMU
constexpr int LB = 64, LK = 16;

template <typename T>
__global__ void __launch_bounds__(256) lin_gemm_kernel(LinGemmArgs<T> a) {
  __shared__ T As[LK][LB + 4];
  __shared__ T Bs[LK][LB + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t row0 = (int64_t)blockIdx.x * LB;
  const int col0 = blockIdx.y * LB;
  const T* arow[4];
  bool aok[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = (tid + i * 256) >> 4;
    aok[i] = row0 + r < a.R;
    arow[i] = aok[i] ? a.a.row(row0 + r) : a.a.p;
  }
  T acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = T(0);
  for (int k0 = 0; k0 < a.K; k0 += LK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * 256, r = idx >> 4, kk = idx & 15, kg = k0 + kk;
      As[kk][r] = (aok[i] && kg < a.K) ? arow[i][kg] : T(0);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * 256;
      int kk, cc;
      if (a.trans_b) { kk = idx & 15; cc = idx >> 4; } else { cc = idx & 63; kk = idx >> 6; }
      const int kg = k0 + kk, cg = col0 + cc;
      T v = T(0);
      if (kg < a.K && cg < a.N) v = a.trans_b ? a.w[(int64_t)cg * a.ldw + kg] : a.w[(int64_t)kg * a.ldw + cg];
      Bs[kk][cc] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < LK; ++kk) {
      T av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
    }
    __syncthreads();
  }
  const T s = *a.scale;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = row0 + ty * 4 + i;
    if (r >= a.R) continue;
    T* crow = const_cast<T*>(a.c.row(r));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int cg = col0 + tx * 4 + j;
      if (cg < a.N) crow[cg] = s * acc[i][j];
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) lin_wgrad_kernel(LinWgradArgs<T> a) {
  __shared__ T Gs[LK][LB + 4];
  __shared__ T Xs[LK][LB + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int o0 = blockIdx.x * LB, f0 = blockIdx.y * LB;
  const int64_t rbeg = (int64_t)blockIdx.z * a.rows_per_split;
  int64_t rend = rbeg + a.rows_per_split;
  if (rend > a.R) rend = a.R;
  T acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = T(0);
  for (int64_t r0 = rbeg; r0 < rend; r0 += LK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * 256, cc = idx & 63, rr = idx >> 6;
      const int64_t r = r0 + rr;
      const bool rok = r < rend;
      Gs[rr][cc] = (rok && o0 + cc < a.n_out) ? a.g.row(r)[o0 + cc] : T(0);
      Xs[rr][cc] = (rok && f0 + cc < a.k_in) ? a.x.row(r)[f0 + cc] : T(0);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < LK; ++kk) {
      T gv[4], xv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) gv[i] = Gs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) xv[j] = Xs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += gv[i] * xv[j];
    }
    __syncthreads();
  }
  const T s = *a.scale;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int o = o0 + ty * 4 + i;
    if (o >= a.n_out) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int f = f0 + tx * 4 + j;
      if (f < a.k_in) atomicAdd(a.gw + (int64_t)o * a.k_in + f, s * acc[i][j]);
    }
  }
}
#endif

template <typename T>
int lin_gemm(const LinGemmArgs<T>& a, cudaStream_t s) {
  if (a.R == 0 || a.N == 0) return 0;
#ifdef FC_HOST_EMU
  const T sc = *a.scale;
  for (int64_t r = 0; r < a.R; ++r) {
    const T* ar = a.a.row(r);
    T* cr = const_cast<T*>(a.c.row(r));
    for (int c = 0; c < a.N; ++c) {
      T acc = T(0);
      for (int k = 0; k < a.K; ++k)
        acc += ar[k] * (a.trans_b ? a.w[(int64_t)c * a.ldw + k] : a.w[(int64_t)k * a.ldw + c]);
      cr[c] = sc * acc;
    }
  }
  return 0;
#else
  const int64_t gx = (a.R + LB - 1) / LB;
  if (gx > 0x7fffffff) return FC_ERR_UNSUPPORTED;
  dim3 grid((unsigned)gx, (unsigned)((a.N + LB - 1) / LB));
  lin_gemm_kernel<T><<<grid, 256, 0, s>>>(a);
  return fc_check_launch();
#endif
}

template <typename T>
int lin_wgrad(LinWgradArgs<T> a, cudaStream_t s) {
  // gw must be zero on entry
  if (a.R == 0 || a.n_out == 0 || a.k_in == 0) return 0;
#ifdef FC_HOST_EMU
  const T sc = *a.scale;
  for (int64_t r = 0; r < a.R; ++r) {
    const T* gr = a.g.row(r);
    const T* xr = a.x.row(r);
    for (int o = 0; o < a.n_out; ++o)
      for (int f = 0; f < a.k_in; ++f) a.gw[(int64_t)o * a.k_in + f] += sc * gr[o] * xr[f];
  }
  return 0;
#else
  const int to = (a.n_out + LB - 1) / LB, tf = (a.k_in + LB - 1) / LB;
  int64_t splits = (a.R + 1023) / 1024;
  const int64_t max_splits = (148 * 8 + to * tf - 1) / (to * tf);
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  if (splits > 65535) splits = 65535;
  a.rows_per_split = (a.R + splits - 1) / splits;
  a.rows_per_split = (a.rows_per_split + LK - 1) / LK * LK;
  splits = (a.R + a.rows_per_split - 1) / a.rows_per_split;
  dim3 grid(to, tf, (unsigned)splits);
  lin_wgrad_kernel<T><<<grid, 256, 0, s>>>(a);
  return fc_check_launch();
#endif
}

template int lin_gemm<float>(const LinGemmArgs<float>&, cudaStream_t);
template int lin_gemm<double>(const LinGemmArgs<double>&, cudaStream_t);
template int lin_wgrad<float>(LinWgradArgs<float>, cudaStream_t);
template int lin_wgrad<double>(LinWgradArgs<double>, cudaStream_t);

}  // namespace fc
