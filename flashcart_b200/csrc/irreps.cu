// Direction tensors T^l(x) of unit vectors (edge attributes) and their derivatives,
// plus the receiver-CSR builder used by the tensor-product convolution.
//
// One thread per vector: the 3 inputs are read once, (l_max+1)^2 outputs are
// written as one contiguous 4*(l_max+1)^2-byte run per thread, so a warp stores a
// contiguous block. The polynomials come from flashcart_b200/codegen/emit.py.
#include "irreps_common.cuh"
#include "gen/irreps_poly.cuh"

namespace fc {

template <typename T, int L>
FC_HD FC_INLINE void irreps_fwd_row(const T* x, T* o) {
  const T a = x[0], b = x[1], c = x[2];
  if constexpr (L == 0) irreps_fwd_l0<T>(a, b, c, o);
  else if constexpr (L == 1) irreps_fwd_l1<T>(a, b, c, o);
  else if constexpr (L == 2) irreps_fwd_l2<T>(a, b, c, o);
  else irreps_fwd_l3<T>(a, b, c, o);
}
template <typename T, int L>
FC_HD FC_INLINE void irreps_bwd_row(const T* x, const T* g, T* gx) {
  const T a = x[0], b = x[1], c = x[2];
  if constexpr (L == 0) irreps_bwd_l0<T>(a, b, c, g, gx);
  else if constexpr (L == 1) irreps_bwd_l1<T>(a, b, c, g, gx);
  else if constexpr (L == 2) irreps_bwd_l2<T>(a, b, c, g, gx);
  else irreps_bwd_l3<T>(a, b, c, g, gx);
}
template <typename T, int L>
FC_HD FC_INLINE void irreps_dbwd_row(const T* x, const T* g, const T* v, T* dg, T* dx) {
  const T a = x[0], b = x[1], c = x[2];
  if constexpr (L == 0) irreps_dbwd_l0<T>(a, b, c, g, v, dg, dx);
  else if constexpr (L == 1) irreps_dbwd_l1<T>(a, b, c, g, v, dg, dx);
  else if constexpr (L == 2) irreps_dbwd_l2<T>(a, b, c, g, v, dg, dx);
  else irreps_dbwd_l3<T>(a, b, c, g, v, dg, dx);
}

template <typename T, int L>
FC_HD FC_INLINE void irreps_fwd_one(const T* __restrict__ x, T* __restrict__ out, int64_t i) {
  constexpr int D = (L + 1) * (L + 1);
  T xv[3] = {fc_ldg(x + 3 * i), fc_ldg(x + 3 * i + 1), fc_ldg(x + 3 * i + 2)};
  T o[D];
  irreps_fwd_row<T, L>(xv, o);
  for (int k = 0; k < D; ++k) out[i * D + k] = o[k];
}
template <typename T, int L>
FC_HD FC_INLINE void irreps_bwd_one(const T* __restrict__ g, const T* __restrict__ x, T* __restrict__ gx,
                                    int64_t i) {
  constexpr int D = (L + 1) * (L + 1);
  T xv[3] = {fc_ldg(x + 3 * i), fc_ldg(x + 3 * i + 1), fc_ldg(x + 3 * i + 2)};
  T gv[D];
  for (int k = 0; k < D; ++k) gv[k] = fc_ldg(g + i * D + k);
  T r[3];
  irreps_bwd_row<T, L>(xv, gv, r);
  for (int k = 0; k < 3; ++k) gx[3 * i + k] = r[k];
}
template <typename T, int L>
FC_HD FC_INLINE void irreps_dbwd_one(const T* __restrict__ g, const T* __restrict__ x, const T* __restrict__ v,
                                     T* __restrict__ dgo, T* __restrict__ dx, int64_t i) {
  constexpr int D = (L + 1) * (L + 1);
  T xv[3] = {fc_ldg(x + 3 * i), fc_ldg(x + 3 * i + 1), fc_ldg(x + 3 * i + 2)};
  T vv[3] = {fc_ldg(v + 3 * i), fc_ldg(v + 3 * i + 1), fc_ldg(v + 3 * i + 2)};
  T gv[D];
  for (int k = 0; k < D; ++k) gv[k] = fc_ldg(g + i * D + k);
  T a[D], b[3];
  irreps_dbwd_row<T, L>(xv, gv, vv, a, b);
  if (dgo)
    for (int k = 0; k < D; ++k) dgo[i * D + k] = a[k];
  if (dx)
    for (int k = 0; k < 3; ++k) dx[3 * i + k] = b[k];
}

#ifndef FC_HOST_EMU
template <typename T, int L>
__global__ void irreps_fwd_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    irreps_fwd_one<T, L>(x, out, i);
}
template <typename T, int L>
__global__ void irreps_bwd_kernel(const T* __restrict__ g, const T* __restrict__ x, T* __restrict__ gx, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    irreps_bwd_one<T, L>(g, x, gx, i);
}
template <typename T, int L>
__global__ void irreps_dbwd_kernel(const T* __restrict__ g, const T* __restrict__ x, const T* __restrict__ v,
                                   T* __restrict__ dgo, T* __restrict__ dx, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    irreps_dbwd_one<T, L>(g, x, v, dgo, dx, i);
}
static inline int elem_grid(int64_t n, int block) {
  int64_t g = (n + block - 1) / block;
  const int64_t cap = 148 * 32;
  return (int)(g > cap ? cap : (g < 1 ? 1 : g));
}
#endif

template <typename T, int L>
int irreps_fwd_launch(const T* x, T* out, int64_t n, cudaStream_t s) {
#ifdef FC_HOST_EMU
  for (int64_t i = 0; i < n; ++i) irreps_fwd_one<T, L>(x, out, i);
  return 0;
#else
  if (n == 0) return 0;
  irreps_fwd_kernel<T, L><<<elem_grid(n, 256), 256, 0, s>>>(x, out, n);
  return fc_check_launch();
#endif
}
template <typename T, int L>
int irreps_bwd_launch(const T* g, const T* x, T* gx, int64_t n, cudaStream_t s) {
#ifdef FC_HOST_EMU
  for (int64_t i = 0; i < n; ++i) irreps_bwd_one<T, L>(g, x, gx, i);
  return 0;
#else
  if (n == 0) return 0;
  irreps_bwd_kernel<T, L><<<elem_grid(n, 256), 256, 0, s>>>(g, x, gx, n);
  return fc_check_launch();
#endif
}
template <typename T, int L>
int irreps_dbwd_launch(const T* g, const T* x, const T* v, T* dgo, T* dx, int64_t n, cudaStream_t s) {
#ifdef FC_HOST_EMU
  for (int64_t i = 0; i < n; ++i) irreps_dbwd_one<T, L>(g, x, v, dgo, dx, i);
  return 0;
#else
  if (n == 0) return 0;
  irreps_dbwd_kernel<T, L><<<elem_grid(n, 256), 256, 0, s>>>(g, x, v, dgo, dx, n);
  return fc_check_launch();
#endif
}

template <typename T>
int irreps_fwd_dispatch(const T* x, T* out, int64_t n, int l, cudaStream_t s) {
  switch (l) {
    case 0: return irreps_fwd_launch<T, 0>(x, out, n, s);
    case 1: return irreps_fwd_launch<T, 1>(x, out, n, s);
    case 2: return irreps_fwd_launch<T, 2>(x, out, n, s);
    case 3: return irreps_fwd_launch<T, 3>(x, out, n, s);
  }
  return FC_ERR_UNSUPPORTED;
}
template <typename T>
int irreps_bwd_dispatch(const T* g, const T* x, T* gx, int64_t n, int l, cudaStream_t s) {
  switch (l) {
    case 0: return irreps_bwd_launch<T, 0>(g, x, gx, n, s);
    case 1: return irreps_bwd_launch<T, 1>(g, x, gx, n, s);
    case 2: return irreps_bwd_launch<T, 2>(g, x, gx, n, s);
    case 3: return irreps_bwd_launch<T, 3>(g, x, gx, n, s);
  }
  return FC_ERR_UNSUPPORTED;
}
template <typename T>
int irreps_dbwd_dispatch(const T* g, const T* x, const T* v, T* dgo, T* dx, int64_t n, int l, cudaStream_t s) {
  switch (l) {
    case 0: return irreps_dbwd_launch<T, 0>(g, x, v, dgo, dx, n, s);
    case 1: return irreps_dbwd_launch<T, 1>(g, x, v, dgo, dx, n, s);
    case 2: return irreps_dbwd_launch<T, 2>(g, x, v, dgo, dx, n, s);
    case 3: return irreps_dbwd_launch<T, 3>(g, x, v, dgo, dx, n, s);
  }
  return FC_ERR_UNSUPPORTED;
}

template int irreps_fwd_dispatch<float>(const float*, float*, int64_t, int, cudaStream_t);
template int irreps_fwd_dispatch<double>(const double*, double*, int64_t, int, cudaStream_t);
template int irreps_bwd_dispatch<float>(const float*, const float*, float*, int64_t, int, cudaStream_t);
template int irreps_bwd_dispatch<double>(const double*, const double*, double*, int64_t, int, cudaStream_t);
template int irreps_dbwd_dispatch<float>(const float*, const float*, const float*, float*, float*, int64_t, int,
                                         cudaStream_t);
template int irreps_dbwd_dispatch<double>(const double*, const double*, const double*, double*, double*, int64_t,
                                          int, cudaStream_t);

// ---------------------------------------------------------------- receiver CSR
// rowptr[k] = #{e : idx_i[e] < k} (lower bound, identical to torch.searchsorted with
// side="left" on an ascending array), k = 0..n_nodes. One thread per k does a
// binary search; threads over the edges flag unsorted / out-of-range receivers.
FC_HD FC_INLINE void rowptr_one(const int64_t* __restrict__ idx, int64_t n_edges, int64_t k, int64_t* rowptr) {
  int64_t lo = 0, hi = n_edges;
  while (lo < hi) {
    const int64_t mid = lo + ((hi - lo) >> 1);
    if (fc_ldg(idx + mid) < k) lo = mid + 1; else hi = mid;
  }
  rowptr[k] = lo;
}
FC_HD FC_INLINE void rowptr_check_one(const int64_t* __restrict__ idx, int64_t e, int64_t n_nodes, int* status) {
  const int64_t v = fc_ldg(idx + e);
  if (v < 0 || v >= n_nodes) fc_flag(status, FC_DEV_BAD_INDEX);
  if (e > 0 && fc_ldg(idx + e - 1) > v) fc_flag(status, FC_DEV_UNSORTED);
}

#ifndef FC_HOST_EMU
__global__ void rowptr_kernel(const int64_t* __restrict__ idx, int64_t n_edges, int64_t n_nodes,
                              int64_t* __restrict__ rowptr, int* status) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  for (int64_t k = t0; k <= n_nodes; k += stride) rowptr_one(idx, n_edges, k, rowptr);
  if (status)
    for (int64_t e = t0; e < n_edges; e += stride) rowptr_check_one(idx, e, n_nodes, status);
}
#endif

int build_rowptr(const int64_t* idx, int64_t n_edges, int64_t n_nodes, int64_t* rowptr, int* status,
                 cudaStream_t s) {
#ifdef FC_HOST_EMU
  for (int64_t k = 0; k <= n_nodes; ++k) rowptr_one(idx, n_edges, k, rowptr);
  if (status)
    for (int64_t e = 0; e < n_edges; ++e) rowptr_check_one(idx, e, n_nodes, status);
  return 0;
#else
  const int64_t work = n_edges > n_nodes + 1 ? n_edges : n_nodes + 1;
  rowptr_kernel<<<elem_grid(work, 256), 256, 0, s>>>(idx, n_edges, n_nodes, rowptr, status);
  return fc_check_launch();
#endif
}

}  // namespace fc
