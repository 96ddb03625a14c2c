// Row gather / scatter of node features for ghost-atom (halo) exchange, and an in-place
// row sum.
//
// A domain decomposition keeps the features of its owned atoms first and those of its
// ghost atoms (copies of atoms owned by other ranks) after them. Between interaction
// layers the owners' rows are gathered into per-peer send buffers (pack), moved by the
// transport the caller owns (NCCL, MPI, an MD engine's own communicator), and written into
// the ghost rows (unpack, copy). In the backward pass the ghost rows' gradients travel the
// other way and are added to the owners' rows (unpack, accumulate). Reference semantics:
// `lammps_forward_exchange` / `lammps_reverse_exchange` (utils/lammps.py:67-118)
// copy owner rows into ghost rows and add ghost-row gradients into owner rows.
//
// One CTA walks whole rows (grid-stride over the index list), its threads the row's
// elements, so each row moves as one coalesced segment; an index outside [0, n_rows) sets
// FC_DEV_BAD_INDEX and its row is skipped (pack writes zeros there).
#include "fc_base.cuh"

namespace fc {

template <typename T>
FC_HD FC_INLINE void pack_row(const T* x, int64_t n_rows, int64_t re, const int64_t* idx, int64_t k, T* buf,
                              int* status, int64_t c0, int64_t dc) {
  const int64_t r = idx[k];
  const bool ok = r >= 0 && r < n_rows;
  if (!ok && c0 == 0) fc_flag(status, FC_DEV_BAD_INDEX);
  for (int64_t c = c0; c < re; c += dc) buf[k * re + c] = ok ? x[r * re + c] : T(0);
}

template <typename T>
FC_HD FC_INLINE void unpack_row(const T* buf, int64_t re, const int64_t* idx, int64_t k, T* x, int64_t n_rows,
                                bool accumulate, int* status, int64_t c0, int64_t dc) {
  const int64_t r = idx[k];
  if (r < 0 || r >= n_rows) {
    if (c0 == 0) fc_flag(status, FC_DEV_BAD_INDEX);
    return;
  }
  if (accumulate) {
    for (int64_t c = c0; c < re; c += dc) fc_atomic_add(x + r * re + c, buf[k * re + c]);
  } else {
    for (int64_t c = c0; c < re; c += dc) x[r * re + c] = buf[k * re + c];
  }
}

#ifndef FC_HOST_EMU
template <typename T>
__global__ void __launch_bounds__(128) halo_pack_kernel(const T* x, int64_t n_rows, int64_t re, const int64_t* idx,
                                                        int64_t n_idx, T* buf, int* status) {
  for (int64_t k = blockIdx.x; k < n_idx; k += gridDim.x)
    pack_row<T>(x, n_rows, re, idx, k, buf, status, threadIdx.x, blockDim.x);
}
template <typename T>
__global__ void __launch_bounds__(128) halo_unpack_kernel(const T* buf, int64_t re, const int64_t* idx, int64_t n_idx,
                                                          T* x, int64_t n_rows, int accumulate, int* status) {
  for (int64_t k = blockIdx.x; k < n_idx; k += gridDim.x)
    unpack_row<T>(buf, re, idx, k, x, n_rows, accumulate != 0, status, threadIdx.x, blockDim.x);
}
template <typename T>
__global__ void __launch_bounds__(256) add_rows_kernel(T* dst, const T* src, int64_t count) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < count; t += (int64_t)gridDim.x * blockDim.x)
    dst[t] += src[t];
}
// rows per CTA: enough CTAs to fill 148 SMs several times over, never more than rows
static unsigned row_grid(int64_t rows) { return (unsigned)(rows < 148 * 16 ? rows : 148 * 16); }
#endif

template <typename T>
int halo_pack_dispatch(const T* x, int64_t n_rows, int64_t re, const int64_t* idx, int64_t n_idx, T* buf, int* status,
                       cudaStream_t s) {
#ifndef FC_HOST_EMU
  halo_pack_kernel<T><<<row_grid(n_idx), 128, 0, s>>>(x, n_rows, re, idx, n_idx, buf, status);
  return fc_check_launch();
#else
  (void)s;
  for (int64_t k = 0; k < n_idx; ++k) pack_row<T>(x, n_rows, re, idx, k, buf, status, 0, 1);
  return 0;
#endif
}

template <typename T>
int halo_unpack_dispatch(const T* buf, int64_t re, const int64_t* idx, int64_t n_idx, T* x, int64_t n_rows,
                         int accumulate, int* status, cudaStream_t s) {
#ifndef FC_HOST_EMU
  halo_unpack_kernel<T><<<row_grid(n_idx), 128, 0, s>>>(buf, re, idx, n_idx, x, n_rows, accumulate, status);
  return fc_check_launch();
#else
  (void)s;
  for (int64_t k = 0; k < n_idx; ++k) unpack_row<T>(buf, re, idx, k, x, n_rows, accumulate != 0, status, 0, 1);
  return 0;
#endif
}

template <typename T>
int add_rows_dispatch(T* dst, const T* src, int64_t count, cudaStream_t s) {
  if (count <= 0) return 0;
#ifndef FC_HOST_EMU
  const int64_t b = (count + 255) / 256;
  add_rows_kernel<T><<<(unsigned)(b < 148 * 64 ? b : 148 * 64), 256, 0, s>>>(dst, src, count);
  return fc_check_launch();
#else
  (void)s;
  for (int64_t t = 0; t < count; ++t) dst[t] += src[t];
  return 0;
#endif
}

template int halo_pack_dispatch<float>(const float*, int64_t, int64_t, const int64_t*, int64_t, float*, int*,
                                       cudaStream_t);
template int halo_pack_dispatch<double>(const double*, int64_t, int64_t, const int64_t*, int64_t, double*, int*,
                                        cudaStream_t);
template int halo_unpack_dispatch<float>(const float*, int64_t, const int64_t*, int64_t, float*, int64_t, int, int*,
                                         cudaStream_t);
template int halo_unpack_dispatch<double>(const double*, int64_t, const int64_t*, int64_t, double*, int64_t, int,
                                          int*, cudaStream_t);
template int add_rows_dispatch<float>(float*, const float*, int64_t, cudaStream_t);
template int add_rows_dispatch<double>(double*, const double*, int64_t, cudaStream_t);

}  // namespace fc
