// C ABI of flashcart_b200 (declared in include/flashcart_b200.h): argument checks,
// zero-filling of accumulated outputs, and dispatch to the compiled kernels.
#include <string>
#include <cstdio>
#include <cstdarg>
#include <mutex>
#include <vector>
#include <initializer_list>

#include "tp_common.cuh"
#include "linear.cuh"
#include "gen/tp_dispatch.inc"

#ifndef FC_VERSION_STRING
#define FC_VERSION_STRING "0.1.0"
#endif

namespace fc {

template <typename T> int irreps_fwd_dispatch(const T*, T*, int64_t, int, cudaStream_t);
template <typename T> int irreps_bwd_dispatch(const T*, const T*, T*, int64_t, int, cudaStream_t);
template <typename T>
int irreps_dbwd_dispatch(const T*, const T*, const T*, T*, T*, int64_t, int, cudaStream_t);
int build_rowptr(const int64_t*, int64_t, int64_t, int64_t*, int*, cudaStream_t);
template <typename T>
int rms_norm_fwd_dispatch(int, const T*, const T*, const T*, T, int, int64_t, T*, T*, cudaStream_t);
template <typename T>
int rms_norm_bwd_dispatch(int, const T*, const T*, const T*, const T*, const T*, int, int64_t, T*, cudaStream_t);
int64_t nl_workspace_bytes(int64_t n, int64_t nbins);
#ifndef FC_HOST_EMU
int nl_count(const fc_nl_desc*, const double*, int64_t, void*, int64_t*, int*, cudaStream_t);
int nl_fill(const fc_nl_desc*, int64_t, const void*, const int64_t*, int64_t, int64_t*, int32_t*, int*, cudaStream_t);
#endif
template <typename T>
int edge_expand_fwd_dispatch(int, const T*, const T*, int, int, int64_t, T*, cudaStream_t);
template <typename T>
int edge_expand_bwd_dispatch(int, const T*, const T*, const T*, int, int, int64_t, T*, T*, cudaStream_t);
#ifndef FC_HOST_EMU
int lin_bf16_rank(const void* x, int64_t ld, int64_t off, int64_t ms, int M, int64_t nodes, const void* w, int K,
                  int N, const float* scale, void* y, int64_t out_ld, int64_t out_off, int64_t out_ms, int* status,
                  cudaStream_t s);
#endif
template <typename T>
int geom_fwd_dispatch(const GeomParams&, const T*, const T*, const int32_t*, const int64_t*, const int64_t*, T*, T*,
                      int*, cudaStream_t);
template <typename T>
int geom_bwd_dispatch(const GeomParams&, const T*, const T*, const int32_t*, const int64_t*, const int64_t*,
                      const T*, const T*, T*, T*, int*, cudaStream_t);
template <typename T>
int gate_fwd_dispatch(int, const T*, const T*, T*, int, int64_t, cudaStream_t);
template <typename T>
int halo_pack_dispatch(const T*, int64_t, int64_t, const int64_t*, int64_t, T*, int*, cudaStream_t);
template <typename T>
int halo_unpack_dispatch(const T*, int64_t, const int64_t*, int64_t, T*, int64_t, int, int*, cudaStream_t);
template <typename T>
int add_rows_dispatch(T*, const T*, int64_t, cudaStream_t);
template <typename T>
int gate_bwd_dispatch(int, const T*, const T*, const T*, T*, T*, int, int64_t, cudaStream_t);

static thread_local std::string g_last_error;

static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

static int launch_status(int rc, const char* what) {
  if (rc == 0) return FC_OK;
#ifndef FC_HOST_EMU
  if (rc == FC_ERR_LAUNCH) {
    cudaError_t e = fc_noted_error();
    fc_noted_error() = cudaSuccess;
    if (e == cudaSuccess) e = cudaGetLastError();
    return fail(FC_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  }
#endif
  return fail(rc, "%s failed with status %d", what, rc);
}

static int zero_fill(void* p, int64_t bytes, cudaStream_t s) {
  if (p == nullptr || bytes <= 0) return 0;
#ifdef FC_HOST_EMU
  std::memset(p, 0, (size_t)bytes);
  return 0;
#else
  return cudaMemsetAsync(p, 0, (size_t)bytes, s) == cudaSuccess ? 0 : FC_ERR_LAUNCH;
#endif
}

static bool path_ok(int l1, int l2, int lo) {
  if (l1 < 0 || l2 < 0 || lo < 0) return false;
  const int d = l1 > l2 ? l1 - l2 : l2 - l1;
  return d <= lo && lo <= l1 + l2 && ((l1 + l2 + lo) & 1) == 0;
}

// Path counts per output rank, same enumeration as o3/utils.py:157-203.
static void count_paths(const fc_tp_desc* d, int* npl) {
  const int lmax = d->in1_l_max > d->in2_l_max ? d->in1_l_max : d->in2_l_max;
  for (int lo = 0; lo <= d->out_l_max; ++lo) {
    npl[lo] = 0;
    for (int l1 = 0; l1 <= lmax; ++l1)
      for (int l2 = 0; l2 <= l1; ++l2) {
        if (path_ok(l1, l2, lo) && l1 <= d->in1_l_max && l2 <= d->in2_l_max) ++npl[lo];
        if (!d->symmetric_product && l2 < l1 && path_ok(l1, l2, lo) && l1 <= d->in2_l_max && l2 <= d->in1_l_max)
          ++npl[lo];
      }
  }
}

static int check_desc(const fc_tp_desc* d) {
  if (d == nullptr) return fail(FC_ERR_INVALID, "tensor product: null descriptor");
  if (d->in1_l_max < 0 || d->in2_l_max < 0 || d->out_l_max < 0)
    return fail(FC_ERR_INVALID, "tensor product: negative rank");
  if (d->in1_l_max > FC_MAX_L || d->in2_l_max > FC_MAX_L || d->out_l_max > FC_MAX_L)
    return fail(FC_ERR_UNSUPPORTED,
                "tensor product supports l_max <= %d; got in1_l_max=%d, in2_l_max=%d, out_l_max=%d.", FC_MAX_L,
                d->in1_l_max, d->in2_l_max, d->out_l_max);
  if (d->in1_features < 1 || d->in2_features < 1)
    return fail(FC_ERR_INVALID, "tensor product: features must be positive");
  if (!(d->in1_features == d->in2_features || d->in1_features == 1 || d->in2_features == 1))
    return fail(FC_ERR_INVALID,
                "Input dimensions must match unless one of them is 1. Got in1_features=%d and in2_features=%d.",
                d->in1_features, d->in2_features);
  if (d->dtype != FC_F32 && d->dtype != FC_F64) return fail(FC_ERR_INVALID, "tensor product: bad dtype %d", d->dtype);
  return FC_OK;
}

static const TpSigEntry* find_sig(const fc_tp_desc* d) {
  const int sym = d->symmetric_product ? 1 : 0;
  for (int k = 0; k < kNumTpSignatures; ++k) {
    const TpSigEntry& e = kTpSignatures[k];
    if (e.l1 == d->in1_l_max && e.l2 == d->in2_l_max && e.lo == d->out_l_max && e.sym == sym) return &e;
  }
  return nullptr;
}

static int64_t out_dim(const fc_tp_desc* d) {
  int npl[FC_MAX_L + 1];
  count_paths(d, npl);
  const int F = d->in1_features > d->in2_features ? d->in1_features : d->in2_features;
  int64_t s = 0;
  for (int l = 0; l <= d->out_l_max; ++l) {
    if (d->reduce_paths) s += npl[l] ? (2 * l + 1) * (int64_t)F : 0;
    else s += (int64_t)npl[l] * (2 * l + 1) * F;
  }
  return s;
}

// The shared-attribute convolution kernels: edge attributes shared by every channel,
// one thread per channel (F a multiple of 32, at most 256), per-edge weights, paths kept.
// Their bulk copies of in1 rows and weight rows need 16-byte aligned base pointers.
static bool conv2_eligible(const fc_tp_desc* d, bool conv, const void* in1, const void* w) {
  const int F = d->in1_features > d->in2_features ? d->in1_features : d->in2_features;
  const bool aligned = ((reinterpret_cast<uintptr_t>(in1) | reinterpret_cast<uintptr_t>(w)) & 15) == 0;
  return conv && aligned && d->in2_features == 1 && d->in1_features == F && F % 32 == 0 && F <= 256 &&
         !d->shared_weights && !d->reduce_paths;
}

// The channel-pair kernels (two adjacent channels per thread, packed f32x2 arithmetic)
// take float32 convolutions with 64 or 128 channels (F/2 threads, whole warps, plus a
// producer warp); conv2_eligible has checked the rest of the layout.
static bool pair_eligible(const fc_tp_desc* d, const void* in2) {
  // in2 rows are bulk-copied (16-byte aligned base; the row offsets are multiples of 16 B)
  return d->dtype == FC_F32 && (d->in1_features == 64 || d->in1_features == 128) &&
         (reinterpret_cast<uintptr_t>(in2) & 15) == 0;
}

// The dense channel-pair kernels: no edges, both inputs with the same 64 or 128 channels,
// paths kept, float32, 8-byte aligned tensors (float2 loads and stores; every row offset
// is a multiple of F floats); weights per row, or shared when no shared weight gradient
// (a reduction over rows) is asked for.
#ifndef FC_FWD4
#define FC_FWD4 1
#endif
#ifndef FC_DENSE_PAIR
#define FC_DENSE_PAIR 1
#endif
static bool dense_pair_eligible(const fc_tp_desc* d, bool conv, const void* grad_weights,
                                std::initializer_list<const void*> ptrs) {
  if (!FC_DENSE_PAIR || conv || d->dtype != FC_F32 || d->reduce_paths) return false;
  if (d->shared_weights && grad_weights != nullptr) return false;
  if (d->in1_features != d->in2_features || (d->in1_features != 64 && d->in1_features != 128)) return false;
  uintptr_t bits = 0;
  for (const void* q : ptrs) bits |= reinterpret_cast<uintptr_t>(q);
  return (bits & 7) == 0;
}

template <typename P>
static void fill_common(P& p, const fc_tp_desc* d, const int64_t* rowptr, const int64_t* idx_j, int64_t n_rows,
                        int64_t n_in1, int32_t* status) {
  p.rowptr = rowptr;
  p.idx_j = idx_j;
  p.n_rows = n_rows;
  p.n_in1 = n_in1;
  p.F1 = d->in1_features;
  p.F2 = d->in2_features;
  p.F = p.F1 > p.F2 ? p.F1 : p.F2;
  p.shared_w = d->shared_weights ? 1 : 0;
  p.reduce = d->reduce_paths ? 1 : 0;
  p.status = reinterpret_cast<int*>(status);
}

// ------------------------------------------------------------------ linear helpers

static int check_linear(const fc_linear_desc* d) {
  if (d == nullptr) return fail(FC_ERR_INVALID, "linear: null descriptor");
  if (d->n_active < 0 || d->n_active > FC_MAX_L + 1)
    return fail(FC_ERR_UNSUPPORTED, "linear supports at most %d ranks, got %d", FC_MAX_L + 1, d->n_active);
  if (d->in_dim < 0 || d->out_dim < 0) return fail(FC_ERR_INVALID, "linear: negative row width");
  for (int l = 0; l < d->n_active; ++l) {
    if (d->m_values[l] < 1 || d->f_in_values[l] < 1 || d->f_out_values[l] < 1)
      return fail(FC_ERR_INVALID, "linear: bad metadata for rank %d", l);
    if (d->in_offsets[l] < 0 || d->in_offsets[l] + (int64_t)d->m_values[l] * d->f_in_values[l] > d->in_dim)
      return fail(FC_ERR_INVALID, "linear: rank %d exceeds the input row", l);
    if (d->out_offsets[l] < 0 || d->out_offsets[l] + (int64_t)d->m_values[l] * d->f_out_values[l] > d->out_dim)
      return fail(FC_ERR_INVALID, "linear: rank %d exceeds the output row", l);
  }
  if (d->dtype != FC_F32 && d->dtype != FC_F64 && d->dtype != FC_BF16) return fail(FC_ERR_INVALID, "linear: bad dtype");
  if (d->precision != FC_PREC_IEEE && d->precision != FC_PREC_TF32)
    return fail(FC_ERR_INVALID, "linear: bad precision");
  if (d->act != FC_ACT_NONE && d->act != FC_ACT_SILU) return fail(FC_ERR_INVALID, "linear: bad activation");
  if (d->act != FC_ACT_NONE && d->dtype != FC_F32)
    return fail(FC_ERR_UNSUPPORTED, "linear: input activations are float32 (tensor-core path) only");
  return FC_OK;
}

template <typename T>
static int gemm_dispatch(const LinGemmArgs<T>& a, int precision, int* status, cudaStream_t s);
template <>
int gemm_dispatch<double>(const LinGemmArgs<double>& a, int, int*, cudaStream_t s) {
  return lin_gemm<double>(a, s);
}
template <>
int gemm_dispatch<float>(const LinGemmArgs<float>& a, int precision, int* status, cudaStream_t s) {
  return lin_gemm_tc(a, precision != FC_PREC_TF32, status, s);
}

// All ranks of a map in one launch where the layout allows (float32 on the TMA path);
// 1 = not taken, the caller launches per rank.
template <typename T>
static int gemm_dispatch_grouped(const LinGemmArgs<T>*, int, int, int*, cudaStream_t) {
  return 1;
}
#ifndef FC_HOST_EMU
template <>
int gemm_dispatch_grouped<float>(const LinGemmArgs<float>* a, int n, int precision, int* status, cudaStream_t s) {
  return lin_gemm_tma_grouped(a, n, precision != FC_PREC_TF32, status, s);
}
#endif

// zero columns [from, width) of every row
template <typename T>
static int zero_tail(T* p, int64_t rows, int64_t width, int64_t from, cudaStream_t s) {
  if (rows <= 0 || from >= width) return 0;
#ifdef FC_HOST_EMU
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t k = from; k < width; ++k) p[r * width + k] = T(0);
  return 0;
#else
  return cudaMemset2DAsync(p + from, width * sizeof(T), 0, (width - from) * sizeof(T), rows, s) == cudaSuccess
             ? 0
             : FC_ERR_LAUNCH;
#endif
}

template <typename T>
static int linear_fwd_t(const fc_linear_desc* d, const T* x, const void* const* weights, const T* scale, int64_t n,
                        T* out, int* status, cudaStream_t s, const void* const* bsplit = nullptr) {
  int64_t end = 0;
  if (d->n_active > 0) {
    const int l = d->n_active - 1;
    end = d->out_offsets[l] + (int64_t)d->m_values[l] * d->f_out_values[l];
  }
  if (int rc = zero_tail(out, n, d->out_dim, end, s)) return rc;
  LinGemmArgs<T> args[FC_MAX_L + 1];
  for (int l = 0; l < d->n_active; ++l) {
    LinGemmArgs<T>& a = args[l];
    a.a = LinRows<T>{x, d->in_dim, d->in_offsets[l], d->f_in_values[l], d->m_values[l]};
    a.w = (const T*)weights[l];
    a.ldw = d->f_in_values[l];
    a.trans_b = 1;
    a.bsplit = bsplit ? (const T*)bsplit[l] : nullptr;
    a.scale = scale + l;
    a.c = LinRows<T>{out, d->out_dim, d->out_offsets[l], d->f_out_values[l], d->m_values[l]};
    a.R = n * d->m_values[l];
    a.K = d->f_in_values[l];
    a.N = d->f_out_values[l];
    a.act = d->act == FC_ACT_SILU ? 1 : 0;
  }
  const int g = d->n_active > 1 ? gemm_dispatch_grouped<T>(args, d->n_active, d->precision, status, s) : 1;
  if (g != 1) return g;
  for (int l = 0; l < d->n_active; ++l)
    if (int rc = gemm_dispatch<T>(args[l], d->precision, status, s)) return rc;
  return 0;
}

template <typename T>
static int linear_bwd_t(const fc_linear_desc* d, const T* g, const T* x, const void* const* weights, const T* scale,
                        int64_t n, T* gx, void* const* gw, int* status, cudaStream_t s,
                        const void* const* bsplit = nullptr) {
  if (n == 0) {
    // no rows: grad_x is empty and every weight gradient is an empty sum
    for (int l = 0; gw && l < d->n_active; ++l)
      if (gw[l] && zero_fill(gw[l], (int64_t)d->f_out_values[l] * d->f_in_values[l] * sizeof(T), s))
        return FC_ERR_LAUNCH;
    return 0;
  }
  if (gx) {
    // columns of x outside the active ranks get zero gradient
    int64_t prev = 0;
    for (int l = 0; l < d->n_active; ++l) {
      if (d->in_offsets[l] > prev)
        if (int rc = zero_tail(gx, n, d->in_offsets[l], prev, s)) return rc;  // gap before rank l
      prev = d->in_offsets[l] + (int64_t)d->m_values[l] * d->f_in_values[l];
    }
    if (int rc = zero_tail(gx, n, d->in_dim, prev, s)) return rc;
    LinGemmArgs<T> args[FC_MAX_L + 1];
    for (int l = 0; l < d->n_active; ++l) {
      LinGemmArgs<T>& a = args[l];
      a.a = LinRows<T>{g, d->out_dim, d->out_offsets[l], d->f_out_values[l], d->m_values[l]};
      a.w = (const T*)weights[l];
      a.ldw = d->f_in_values[l];
      a.trans_b = 0;
      a.bsplit = bsplit ? (const T*)bsplit[l] : nullptr;
      a.scale = scale + l;
      a.c = LinRows<T>{gx, d->in_dim, d->in_offsets[l], d->f_in_values[l], d->m_values[l]};
      a.R = n * d->m_values[l];
      a.K = d->f_out_values[l];
      a.N = d->f_in_values[l];
      if (d->act == FC_ACT_SILU) {
        a.act = 2;
        a.aux = LinRows<T>{x, d->in_dim, d->in_offsets[l], d->f_in_values[l], d->m_values[l]};
      }
    }
    const int grp = d->n_active > 1 ? gemm_dispatch_grouped<T>(args, d->n_active, d->precision, status, s) : 1;
    if (grp != 1 && grp != 0) return grp;
    for (int l = 0; grp == 1 && l < d->n_active; ++l)
      if (int rc = gemm_dispatch<T>(args[l], d->precision, status, s)) return rc;
  }
  if (gw && d->act != FC_ACT_NONE) {
    for (int l = 0; l < d->n_active; ++l)
      if (gw[l]) return fail(FC_ERR_UNSUPPORTED, "linear: no weight gradients with an input activation");
  }
  if (gw) {
    for (int l = 0; l < d->n_active; ++l) {
      if (gw[l] == nullptr) continue;
      if (zero_fill(gw[l], (int64_t)d->f_out_values[l] * d->f_in_values[l] * sizeof(T), s)) return FC_ERR_LAUNCH;
      LinWgradArgs<T> a;
      a.g = LinRows<T>{g, d->out_dim, d->out_offsets[l], d->f_out_values[l], d->m_values[l]};
      a.x = LinRows<T>{x, d->in_dim, d->in_offsets[l], d->f_in_values[l], d->m_values[l]};
      a.scale = scale + l;
      a.gw = (T*)gw[l];
      a.R = n * d->m_values[l];
      a.n_out = d->f_out_values[l];
      a.k_in = d->f_in_values[l];
      a.rows_per_split = 0;
      if (int rc = lin_wgrad<T>(a, s)) return rc;
    }
  }
  return 0;
}

// VJP of linear_bwd_t (see fc_linear_dbwd in the header) from the forward / backward GEMMs.
template <typename T>
static int linear_dbwd_t(const fc_linear_desc* d, const T* g, const T* x, const void* const* weights, const T* vx,
                         const void* const* vw, const T* scale, int64_t n, T* dg, T* dx, void* const* dw, int* status,
                         cudaStream_t s) {
  const size_t esz = sizeof(T);
  if (dg) {
    if (vx) {
      if (int rc = linear_fwd_t<T>(d, vx, weights, scale, n, dg, status, s)) return rc;
    }
    if (vw) {
      if (!vx) {
        if (int rc = linear_fwd_t<T>(d, x, vw, scale, n, dg, status, s)) return rc;
      } else {
        const int64_t count = n * d->out_dim;
#ifndef FC_HOST_EMU
        void* tmp = nullptr;
        if (fc_pool_alloc(&tmp, (size_t)count * esz, s)) return FC_ERR_LAUNCH;
        int rc = linear_fwd_t<T>(d, x, vw, scale, n, (T*)tmp, status, s);
        if (!rc) rc = add_rows_dispatch<T>(dg, (const T*)tmp, count, s);
        if (fc_pool_free(tmp, s) && !rc) rc = FC_ERR_LAUNCH;
#else
        std::vector<T> tmp((size_t)count);
        int rc = linear_fwd_t<T>(d, x, vw, scale, n, tmp.data(), status, s);
        if (!rc) rc = add_rows_dispatch<T>(dg, tmp.data(), count, s);
#endif
        if (rc) return rc;
      }
    }
    if (!vx && !vw && zero_fill(dg, n * d->out_dim * (int64_t)esz, s)) return FC_ERR_LAUNCH;
  }
  if (dx) {
    if (vw) {
      if (int rc = linear_bwd_t<T>(d, g, x, vw, scale, n, dx, nullptr, status, s)) return rc;
    } else if (zero_fill(dx, n * d->in_dim * (int64_t)esz, s)) {
      return FC_ERR_LAUNCH;
    }
  }
  if (dw) {
    if (vx) {
      if (int rc = linear_bwd_t<T>(d, g, vx, weights, scale, n, nullptr, dw, status, s)) return rc;
    } else {
      for (int l = 0; l < d->n_active; ++l)
        if (dw[l] && zero_fill(dw[l], (int64_t)d->f_out_values[l] * d->f_in_values[l] * (int64_t)esz, s))
          return FC_ERR_LAUNCH;
    }
  }
  return 0;
}

// ------------------------------------------------------------------ allocation-free entry
// Receiver-CSR workspace of fc_tp_conv_fwd_noalloc: a fixed array in the library's own
// device memory (every device that loads the library holds it until process exit), so
// that entry point never allocates. Host code must not take the array's address
// directly (its name is a host-side stand-in): the device address comes from
// cudaGetSymbolAddress, looked up once per device and cached.
constexpr int64_t kNoAllocMaxNodes = int64_t(1) << 18;  // 262,144 receivers -> 2 MiB of int64
#ifndef FC_HOST_EMU
static __device__ __align__(256) int64_t g_noalloc_rowptr[kNoAllocMaxNodes + 1];
static std::mutex g_noalloc_mutex;
constexpr int kNoAllocMaxDevices = 64;
static int64_t* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// The address is looked up once per device and kept for the life of the process; it does
// not survive cudaDeviceReset (a reset device gets a new module load and a new address).
static int noalloc_rowptr(int64_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess)
    return fail(FC_ERR_LAUNCH, "fc_tp_conv_fwd_noalloc: no current CUDA device");
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(FC_ERR_UNSUPPORTED, "fc_tp_conv_fwd_noalloc: device ordinal %d beyond the %d devices it serves", dev,
                kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_rowptr);
    if (e != cudaSuccess || ptr == nullptr)
      return fail(FC_ERR_LAUNCH, "fc_tp_conv_fwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<int64_t*>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return FC_OK;
}
#else
static int64_t g_noalloc_rowptr_host[kNoAllocMaxNodes + 1];
static int noalloc_rowptr(int64_t** out) {
  *out = g_noalloc_rowptr_host;
  return FC_OK;
}
#endif

}  // namespace fc

using namespace fc;

#ifndef FC_HOST_EMU
namespace fc {
int ns_orthogonalize(const void* update, int dtype_in, int64_t batch, int rows_in, int cols_in, const float* coeffs,
                     int steps, const float* polish, int polish_steps, float eps, void* out, int32_t* status,
                     cudaStream_t s);
}
#endif

extern "C" {

const char* fc_version(void) {
#ifdef FC_HOST_EMU
  return "flashcart_b200 " FC_VERSION_STRING " (host emulation build, test only)";
#else
  return "flashcart_b200 " FC_VERSION_STRING " (sm_100a)";
#endif
}

const char* fc_last_error(void) { return g_last_error.c_str(); }

int fc_build_rowptr(const int64_t* idx_i, int64_t n_edges, int64_t n_nodes, int64_t* rowptr, int32_t* status,
                    fc_stream_t stream) {
  if (n_edges < 0 || n_nodes < 0) return fail(FC_ERR_INVALID, "fc_build_rowptr: negative size");
  if (rowptr == nullptr || (n_edges > 0 && idx_i == nullptr)) return fail(FC_ERR_INVALID, "fc_build_rowptr: null");
  return launch_status(build_rowptr(idx_i, n_edges, n_nodes, rowptr, reinterpret_cast<int*>(status),
                                    (cudaStream_t)stream),
                       "fc_build_rowptr");
}

int fc_tp_num_paths(const fc_tp_desc* desc) {
  if (int rc = check_desc(desc)) return rc;
  int npl[FC_MAX_L + 1];
  count_paths(desc, npl);
  int s = 0;
  for (int l = 0; l <= desc->out_l_max; ++l) s += npl[l];
  return s;
}

int64_t fc_tp_out_dim(const fc_tp_desc* desc) {
  if (int rc = check_desc(desc)) return rc;
  return out_dim(desc);
}

int fc_tp_fwd(const fc_tp_desc* desc, const void* in1, const void* in2, const void* weights, const int64_t* rowptr,
              const int64_t* idx_j, int64_t n_out_rows, int64_t n_in1_rows, int64_t n_in2_rows, void* out,
              int32_t* status, fc_stream_t stream) {
  if (int rc = check_desc(desc)) return rc;
  if (n_out_rows < 0 || n_in1_rows < 0 || n_in2_rows < 0) return fail(FC_ERR_INVALID, "fc_tp_fwd: negative size");
  if (rowptr == nullptr && n_out_rows != n_in1_rows)
    return fail(FC_ERR_INVALID, "fc_tp_fwd: dense product needs n_out_rows == n_in1_rows");
  if (rowptr != nullptr && idx_j == nullptr && n_in2_rows > 0)
    return fail(FC_ERR_INVALID, "fc_tp_fwd: convolution needs idx_j");
  if (n_out_rows == 0) return FC_OK;
  const TpSigEntry* sig = find_sig(desc);
  if (sig == nullptr || sig->npaths == 0) {
    // no path: output has zero width
    return FC_OK;
  }
  cudaStream_t s = (cudaStream_t)stream;
  if (rowptr != nullptr && n_in2_rows == 0) {
    // convolution over no edges (isolated receivers only): every output row is an empty sum
    if (!out) return fail(FC_ERR_INVALID, "fc_tp_fwd: null tensor");
    return launch_status(zero_fill(out, n_out_rows * out_dim(desc) * (desc->dtype == FC_F32 ? 4 : 8), s),
                         "fc_tp_fwd (zero fill)");
  }
  if (!in1 || !in2 || !weights || !out) return fail(FC_ERR_INVALID, "fc_tp_fwd: null tensor");
  const bool v2 = conv2_eligible(desc, rowptr != nullptr, in1, weights) && sig->table->fwd2_f32 != nullptr;
  if (desc->dtype == FC_F32) {
    TpParams<float> p;
    fill_common(p, desc, rowptr, idx_j, n_out_rows, n_in1_rows, status);
    p.in1 = (const float*)in1; p.in2 = (const float*)in2; p.w = (const float*)weights; p.out = (float*)out;
    if (v2 && pair_eligible(desc, in2) && sig->table->fwd3_f32) {
      // 128 channels: the four-channel forward (one consumer warp per receiver; 16-byte
      // output stores need a 16-byte aligned output)
      if (FC_FWD4 && desc->in1_features == 128 && sig->table->fwd4_f32 &&
          (reinterpret_cast<uintptr_t>(out) & 15) == 0)
        return launch_status(sig->table->fwd4_f32(p, s), "fc_tp_fwd");
      return launch_status(sig->table->fwd3_f32(p, s), "fc_tp_fwd");
    }
    if (sig->table->dpfwd_f32 && dense_pair_eligible(desc, rowptr != nullptr, nullptr, {in1, in2, weights, out}))
      return launch_status(sig->table->dpfwd_f32(p, s), "fc_tp_fwd");
    return launch_status(v2 ? sig->table->fwd2_f32(p, s) : sig->table->fwd_f32(p, s), "fc_tp_fwd");
  }
  TpParams<double> p;
  fill_common(p, desc, rowptr, idx_j, n_out_rows, n_in1_rows, status);
  p.in1 = (const double*)in1; p.in2 = (const double*)in2; p.w = (const double*)weights; p.out = (double*)out;
  return launch_status(v2 ? sig->table->fwd2_f64(p, s) : sig->table->fwd_f64(p, s), "fc_tp_fwd");
}


int fc_tp_bwd(const fc_tp_desc* desc, const void* grad_out, const void* in1, const void* in2, const void* weights,
              const int64_t* rowptr, const int64_t* idx_j, int64_t n_out_rows, int64_t n_in1_rows,
              int64_t n_in2_rows, void* grad_in1, void* grad_in2, void* grad_weights, int32_t* status,
              fc_stream_t stream) {
  if (int rc = check_desc(desc)) return rc;
  if (n_out_rows < 0 || n_in1_rows < 0 || n_in2_rows < 0) return fail(FC_ERR_INVALID, "fc_tp_bwd: negative size");
  if (rowptr != nullptr && idx_j == nullptr && n_in2_rows > 0)
    return fail(FC_ERR_INVALID, "fc_tp_bwd: convolution needs idx_j");
  if (rowptr == nullptr && (n_out_rows != n_in1_rows || n_in2_rows != n_in1_rows))
    return fail(FC_ERR_INVALID, "fc_tp_bwd: dense product needs equal row counts");
  const TpSigEntry* sig = find_sig(desc);
  const bool conv = rowptr != nullptr;
  const int esz = desc->dtype == FC_F32 ? 4 : 8;
  const int F = desc->in1_features > desc->in2_features ? desc->in1_features : desc->in2_features;
  const int64_t d1 = (int64_t)(desc->in1_l_max + 1) * (desc->in1_l_max + 1) * desc->in1_features;
  const int64_t d2 = (int64_t)(desc->in2_l_max + 1) * (desc->in2_l_max + 1) * desc->in2_features;
  const int np = sig ? sig->npaths : 0;
  cudaStream_t s = (cudaStream_t)stream;
  // outputs accumulated by atomics start at zero; all others are fully overwritten
  int rc = 0;
  if (grad_in1 && (conv || desc->in1_features == 1 || np == 0)) rc |= zero_fill(grad_in1, n_in1_rows * d1 * esz, s);
  if (grad_in2 && (desc->in2_features == 1 || np == 0)) rc |= zero_fill(grad_in2, n_in2_rows * d2 * esz, s);
  if (grad_weights && (desc->shared_weights || np == 0 || (conv && n_out_rows == 0)))
    rc |= zero_fill(grad_weights, (desc->shared_weights ? 1 : n_in2_rows) * (int64_t)np * F * esz, s);
  if (rc) return launch_status(FC_ERR_LAUNCH, "fc_tp_bwd (zero fill)");
  // no edges: the zero-filled grad_in1 / shared grad_weights are the answer, grad_in2 has no rows
  if (n_out_rows == 0 || np == 0 || (conv && n_in2_rows == 0)) return FC_OK;
  if (!grad_out || !in1 || !in2 || !weights) return fail(FC_ERR_INVALID, "fc_tp_bwd: null tensor");
  const bool v2 = conv2_eligible(desc, conv, in1, weights) && sig->table->bwd2_f32 != nullptr;
  if (desc->dtype == FC_F32) {
    TpBwdParams<float> p;
    fill_common(p, desc, rowptr, idx_j, n_out_rows, n_in1_rows, status);
    p.g_out = (const float*)grad_out; p.in1 = (const float*)in1; p.in2 = (const float*)in2;
    p.w = (const float*)weights;
    p.g_in1 = (float*)grad_in1; p.g_in2 = (float*)grad_in2; p.g_w = (float*)grad_weights;
    if (v2 && pair_eligible(desc, in2) && sig->table->bwd3_f32) return launch_status(sig->table->bwd3_f32(p, s), "fc_tp_bwd");
    if (sig->table->dpbwd_f32 &&
        dense_pair_eligible(desc, conv, grad_weights, {grad_out, in1, in2, weights, grad_in1, grad_in2, grad_weights}))
      return launch_status(sig->table->dpbwd_f32(p, s), "fc_tp_bwd");
    return launch_status(v2 ? sig->table->bwd2_f32(p, s) : sig->table->bwd_f32(p, s), "fc_tp_bwd");
  }
  TpBwdParams<double> p;
  fill_common(p, desc, rowptr, idx_j, n_out_rows, n_in1_rows, status);
  p.g_out = (const double*)grad_out; p.in1 = (const double*)in1; p.in2 = (const double*)in2;
  p.w = (const double*)weights;
  p.g_in1 = (double*)grad_in1; p.g_in2 = (double*)grad_in2; p.g_w = (double*)grad_weights;
  return launch_status(v2 ? sig->table->bwd2_f64(p, s) : sig->table->bwd_f64(p, s), "fc_tp_bwd");
}

int fc_tp_bwd_residual(const fc_tp_desc* desc, const void* grad_out, const void* in1, const void* in2,
                       const void* weights, int64_t n_rows, const void* residual_in1, int64_t residual_in1_ld,
                       int32_t residual_in1_comps, const void* residual_in2, void* grad_in1, void* grad_in2,
                       int32_t* status, fc_stream_t stream) {
  if (int rc = check_desc(desc)) return rc;
  if (n_rows < 0) return fail(FC_ERR_INVALID, "fc_tp_bwd_residual: negative size");
  const TpSigEntry* sig = find_sig(desc);
  if (!dense_pair_eligible(desc, false, nullptr, {grad_out, in1, in2, weights, residual_in1, residual_in2, grad_in1,
                                                  grad_in2}))
    return fail(FC_ERR_UNSUPPORTED, "fc_tp_bwd_residual: float32 dense products of 64 / 128 channels with paths "
                                    "kept and 8-byte aligned rows only");
  const int64_t d1 = (int64_t)(desc->in1_l_max + 1) * (desc->in1_l_max + 1);
  if (residual_in1 && (residual_in1_comps < 0 || residual_in1_comps > d1 ||
                       residual_in1_ld < (int64_t)residual_in1_comps * desc->in1_features || (residual_in1_ld & 1)))
    return fail(FC_ERR_INVALID, "fc_tp_bwd_residual: residual_in1 layout");
  if (n_rows == 0) return FC_OK;
  if (sig == nullptr || sig->npaths == 0 || sig->table->dpbwd_f32 == nullptr)
    return fail(FC_ERR_UNSUPPORTED, "fc_tp_bwd_residual: no dense pair kernel for this signature");
  if (!grad_out || !in1 || !in2 || !weights) return fail(FC_ERR_INVALID, "fc_tp_bwd_residual: null tensor");
  TpBwdParams<float> p;
  fill_common(p, desc, nullptr, nullptr, n_rows, n_rows, status);
  p.g_out = (const float*)grad_out; p.in1 = (const float*)in1; p.in2 = (const float*)in2;
  p.w = (const float*)weights;
  p.g_in1 = (float*)grad_in1; p.g_in2 = (float*)grad_in2; p.g_w = nullptr;
  p.r_in1 = (const float*)residual_in1;
  p.r_in2 = (const float*)residual_in2;
  p.r1_ld = residual_in1_ld;
  p.r1_comps = residual_in1 ? residual_in1_comps : 0;
  const int rc = sig->table->dpbwd_f32(p, (cudaStream_t)stream);
  return rc == FC_ERR_LAUNCH || rc == 0 ? launch_status(rc, "fc_tp_bwd_residual") : rc;
}

int fc_tp_dbwd(const fc_tp_desc* desc, const void* grad_out, const void* in1, const void* in2, const void* weights,
               const void* v_in1, const void* v_in2, const void* v_weights, const int64_t* rowptr,
               const int64_t* idx_j, int64_t n_out_rows, int64_t n_in1_rows, int64_t n_in2_rows, void* d_grad_out,
               void* d_in1, void* d_in2, void* d_weights, int32_t* status, fc_stream_t stream) {
  if (int rc = check_desc(desc)) return rc;
  if (n_out_rows < 0 || n_in1_rows < 0 || n_in2_rows < 0) return fail(FC_ERR_INVALID, "fc_tp_dbwd: negative size");
  if (rowptr != nullptr && idx_j == nullptr && n_in2_rows > 0)
    return fail(FC_ERR_INVALID, "fc_tp_dbwd: convolution needs idx_j");
  if (rowptr == nullptr && (n_out_rows != n_in1_rows || n_in2_rows != n_in1_rows))
    return fail(FC_ERR_INVALID, "fc_tp_dbwd: dense product needs equal row counts");
  const TpSigEntry* sig = find_sig(desc);
  const bool conv = rowptr != nullptr;
  const int esz = desc->dtype == FC_F32 ? 4 : 8;
  const int F = desc->in1_features > desc->in2_features ? desc->in1_features : desc->in2_features;
  const int64_t d1 = (int64_t)(desc->in1_l_max + 1) * (desc->in1_l_max + 1) * desc->in1_features;
  const int64_t d2 = (int64_t)(desc->in2_l_max + 1) * (desc->in2_l_max + 1) * desc->in2_features;
  const int np = sig ? sig->npaths : 0;
  cudaStream_t s = (cudaStream_t)stream;
  int rc = 0;
  if (d_in1 && (conv || desc->in1_features == 1 || np == 0)) rc |= zero_fill(d_in1, n_in1_rows * d1 * esz, s);
  if (d_in2 && (desc->in2_features == 1 || np == 0)) rc |= zero_fill(d_in2, n_in2_rows * d2 * esz, s);
  if (d_weights && (desc->shared_weights || np == 0 || (conv && n_out_rows == 0)))
    rc |= zero_fill(d_weights, (desc->shared_weights ? 1 : n_in2_rows) * (int64_t)np * F * esz, s);
  const bool no_edges = conv && n_in2_rows == 0;
  if (d_grad_out && (np == 0 || no_edges)) rc |= zero_fill(d_grad_out, n_out_rows * out_dim(desc) * esz, s);
  if (rc) return launch_status(FC_ERR_LAUNCH, "fc_tp_dbwd (zero fill)");
  if (n_out_rows == 0 || np == 0 || no_edges) return FC_OK;
  if (!grad_out || !in1 || !in2 || !weights) return fail(FC_ERR_INVALID, "fc_tp_dbwd: null tensor");
  if (desc->dtype == FC_F32) {
    TpDbwdParams<float> p;
    fill_common(p, desc, rowptr, idx_j, n_out_rows, n_in1_rows, status);
    p.g_out = (const float*)grad_out; p.in1 = (const float*)in1; p.in2 = (const float*)in2;
    p.w = (const float*)weights;
    p.v1 = (const float*)v_in1; p.v2 = (const float*)v_in2; p.vw = (const float*)v_weights;
    p.d_g = (float*)d_grad_out; p.d_in1 = (float*)d_in1; p.d_in2 = (float*)d_in2; p.d_w = (float*)d_weights;
    return launch_status(sig->table->dbwd_f32(p, s), "fc_tp_dbwd");
  }
  TpDbwdParams<double> p;
  fill_common(p, desc, rowptr, idx_j, n_out_rows, n_in1_rows, status);
  p.g_out = (const double*)grad_out; p.in1 = (const double*)in1; p.in2 = (const double*)in2;
  p.w = (const double*)weights;
  p.v1 = (const double*)v_in1; p.v2 = (const double*)v_in2; p.vw = (const double*)v_weights;
  p.d_g = (double*)d_grad_out; p.d_in1 = (double*)d_in1; p.d_in2 = (double*)d_in2; p.d_w = (double*)d_weights;
  return launch_status(sig->table->dbwd_f64(p, s), "fc_tp_dbwd");
}

// ------------------------------------------------------------------ irreps

int fc_irreps_fwd(const void* x, int64_t n, int32_t l_max, int32_t dtype, void* out, fc_stream_t stream) {
  if (l_max < 0 || l_max > FC_MAX_L)
    return fail(FC_ERR_UNSUPPORTED, "Irreps supports l_max <= %d, got l_max=%d.", FC_MAX_L, l_max);
  if (n < 0) return fail(FC_ERR_INVALID, "fc_irreps_fwd: negative size");
  if (n == 0) return FC_OK;
  if (!x || !out) return fail(FC_ERR_INVALID, "fc_irreps_fwd: null tensor");
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == FC_F32)
    return launch_status(irreps_fwd_dispatch<float>((const float*)x, (float*)out, n, l_max, s), "fc_irreps_fwd");
  if (dtype == FC_F64)
    return launch_status(irreps_fwd_dispatch<double>((const double*)x, (double*)out, n, l_max, s), "fc_irreps_fwd");
  return fail(FC_ERR_INVALID, "fc_irreps_fwd: bad dtype");
}

int fc_irreps_bwd(const void* grad_out, const void* x, int64_t n, int32_t l_max, int32_t dtype, void* grad_x,
                  fc_stream_t stream) {
  if (l_max < 0 || l_max > FC_MAX_L)
    return fail(FC_ERR_UNSUPPORTED, "Irreps supports l_max <= %d, got l_max=%d.", FC_MAX_L, l_max);
  if (n < 0) return fail(FC_ERR_INVALID, "fc_irreps_bwd: negative size");
  if (n == 0) return FC_OK;
  if (!grad_out || !x || !grad_x) return fail(FC_ERR_INVALID, "fc_irreps_bwd: null tensor");
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == FC_F32)
    return launch_status(
        irreps_bwd_dispatch<float>((const float*)grad_out, (const float*)x, (float*)grad_x, n, l_max, s),
        "fc_irreps_bwd");
  if (dtype == FC_F64)
    return launch_status(
        irreps_bwd_dispatch<double>((const double*)grad_out, (const double*)x, (double*)grad_x, n, l_max, s),
        "fc_irreps_bwd");
  return fail(FC_ERR_INVALID, "fc_irreps_bwd: bad dtype");
}

int fc_irreps_dbwd(const void* grad_out, const void* x, const void* v, int64_t n, int32_t l_max, int32_t dtype,
                   void* d_grad_out, void* d_x, fc_stream_t stream) {
  if (l_max < 0 || l_max > FC_MAX_L)
    return fail(FC_ERR_UNSUPPORTED, "Irreps supports l_max <= %d, got l_max=%d.", FC_MAX_L, l_max);
  if (n < 0) return fail(FC_ERR_INVALID, "fc_irreps_dbwd: negative size");
  if (n == 0) return FC_OK;
  if (!grad_out || !x || !v) return fail(FC_ERR_INVALID, "fc_irreps_dbwd: null tensor");
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == FC_F32)
    return launch_status(irreps_dbwd_dispatch<float>((const float*)grad_out, (const float*)x, (const float*)v,
                                                     (float*)d_grad_out, (float*)d_x, n, l_max, s),
                         "fc_irreps_dbwd");
  if (dtype == FC_F64)
    return launch_status(irreps_dbwd_dispatch<double>((const double*)grad_out, (const double*)x, (const double*)v,
                                                      (double*)d_grad_out, (double*)d_x, n, l_max, s),
                         "fc_irreps_dbwd");
  return fail(FC_ERR_INVALID, "fc_irreps_dbwd: bad dtype");
}

// bf16 storage: one tensor-core launch per rank block (csrc/linear_bf16.cu); columns of y
// outside the active ranks are zeroed.
static int linear_fwd_bf16(const fc_linear_desc* d, const void* x, const void* const* weights, const float* scale,
                           int64_t n, void* out, int* status, cudaStream_t s) {
#ifdef FC_HOST_EMU
  (void)d; (void)x; (void)weights; (void)scale; (void)n; (void)out; (void)status; (void)s;
  return fail(FC_ERR_UNSUPPORTED, "fc_linear_fwd: bf16 maps run on the GPU only");
#else
  int64_t end = 0;
  if (d->n_active > 0) {
    const int l = d->n_active - 1;
    end = d->out_offsets[l] + (int64_t)d->m_values[l] * d->f_out_values[l];
  }
  if (int rc = zero_tail(reinterpret_cast<uint16_t*>(out), n, d->out_dim, end, s)) return rc;
  for (int l = 0; l < d->n_active; ++l) {
    const int rc = lin_bf16_rank(x, d->in_dim, d->in_offsets[l], d->f_in_values[l], d->m_values[l], n, weights[l],
                                 d->f_in_values[l], d->f_out_values[l], scale + l, out, d->out_dim,
                                 d->out_offsets[l], d->f_out_values[l], status, s);
    if (rc == FC_ERR_UNSUPPORTED)
      return fail(FC_ERR_UNSUPPORTED, "fc_linear_fwd (bf16): rank %d is not 16-byte aligned (offsets and widths "
                                      "must be multiples of 8)", l);
    if (rc) return rc;
  }
  return 0;
#endif
}

int fc_linear_fwd(const fc_linear_desc* desc, const void* x, const void* const* weights, const void* scale,
                  int64_t n, void* out, int32_t* status, fc_stream_t stream) {
  if (int rc = check_linear(desc)) return rc;
  if (n < 0) return fail(FC_ERR_INVALID, "fc_linear_fwd: negative size");
  if (n == 0 || desc->out_dim == 0) return FC_OK;
  if (!out || (desc->n_active > 0 && (!x || !scale || !weights)))
    return fail(FC_ERR_INVALID, "fc_linear_fwd: null tensor");
  for (int l = 0; l < desc->n_active; ++l)
    if (!weights[l]) return fail(FC_ERR_INVALID, "fc_linear_fwd: null weight for rank %d", l);
  cudaStream_t s = (cudaStream_t)stream;
  if (desc->dtype == FC_BF16) return launch_status(linear_fwd_bf16(desc, x, weights, (const float*)scale, n, out,
                                                                   reinterpret_cast<int*>(status), s),
                                                   "fc_linear_fwd (bf16)");
  if (desc->dtype == FC_F32)
    return launch_status(linear_fwd_t<float>(desc, (const float*)x, weights, (const float*)scale, n, (float*)out,
                                             reinterpret_cast<int*>(status), s),
                         "fc_linear_fwd");
  return launch_status(linear_fwd_t<double>(desc, (const double*)x, weights, (const double*)scale, n, (double*)out,
                                            reinterpret_cast<int*>(status), s),
                       "fc_linear_fwd");
}

int fc_linear_bwd(const fc_linear_desc* desc, const void* grad_out, const void* x, const void* const* weights,
                  const void* scale, int64_t n, void* grad_x, void* const* grad_weights, int32_t* status,
                  fc_stream_t stream) {
  if (int rc = check_linear(desc)) return rc;
  if (desc->dtype == FC_BF16) return fail(FC_ERR_UNSUPPORTED, "fc_linear_bwd: bf16 maps are forward only");
  if (n < 0) return fail(FC_ERR_INVALID, "fc_linear_bwd: negative size");
  if (desc->n_active > 0 && (!scale || !weights || (n > 0 && (!grad_out || !x))))
    return fail(FC_ERR_INVALID, "fc_linear_bwd: null tensor");
  cudaStream_t s = (cudaStream_t)stream;
  if (desc->dtype == FC_F32)
    return launch_status(linear_bwd_t<float>(desc, (const float*)grad_out, (const float*)x, weights,
                                             (const float*)scale, n, (float*)grad_x, grad_weights,
                                             reinterpret_cast<int*>(status), s),
                         "fc_linear_bwd");
  return launch_status(linear_bwd_t<double>(desc, (const double*)grad_out, (const double*)x, weights,
                                            (const double*)scale, n, (double*)grad_x, grad_weights,
                                            reinterpret_cast<int*>(status), s),
                       "fc_linear_bwd");
}

int fc_linear_dbwd(const fc_linear_desc* desc, const void* grad_out, const void* x, const void* const* weights,
                   const void* v_grad_x, const void* const* v_grad_weights, const void* scale, int64_t n,
                   void* d_grad_out, void* d_x, void* const* d_weights, int32_t* status, fc_stream_t stream) {
  if (int rc = check_linear(desc)) return rc;
  if (desc->dtype == FC_BF16) return fail(FC_ERR_UNSUPPORTED, "fc_linear_dbwd: bf16 maps are forward only");
  if (desc->act != FC_ACT_NONE) return fail(FC_ERR_UNSUPPORTED, "fc_linear_dbwd: no input activation");
  if (n < 0) return fail(FC_ERR_INVALID, "fc_linear_dbwd: negative size");
  if (desc->n_active > 0 && (!scale || !weights || (n > 0 && (!grad_out || !x))))
    return fail(FC_ERR_INVALID, "fc_linear_dbwd: null tensor");
  for (int l = 0; v_grad_weights && l < desc->n_active; ++l)
    if (!v_grad_weights[l]) return fail(FC_ERR_INVALID, "fc_linear_dbwd: null weight tangent for rank %d", l);
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t esz = desc->dtype == FC_F32 ? 4 : 8;
  if (n == 0 || desc->n_active == 0) {
    // no rows (or no active rank): every output is an empty sum
    int rc = 0;
    if (d_grad_out) rc |= zero_fill(d_grad_out, n * desc->out_dim * esz, s);
    if (d_x) rc |= zero_fill(d_x, n * desc->in_dim * esz, s);
    for (int l = 0; d_weights && l < desc->n_active; ++l)
      if (d_weights[l])
        rc |= zero_fill(d_weights[l], (int64_t)desc->f_out_values[l] * desc->f_in_values[l] * esz, s);
    return rc ? launch_status(FC_ERR_LAUNCH, "fc_linear_dbwd (zero fill)") : FC_OK;
  }
  if (desc->dtype == FC_F32)
    return launch_status(linear_dbwd_t<float>(desc, (const float*)grad_out, (const float*)x, weights,
                                              (const float*)v_grad_x, v_grad_weights, (const float*)scale, n,
                                              (float*)d_grad_out, (float*)d_x, d_weights,
                                              reinterpret_cast<int*>(status), s),
                         "fc_linear_dbwd");
  return launch_status(linear_dbwd_t<double>(desc, (const double*)grad_out, (const double*)x, weights,
                                             (const double*)v_grad_x, v_grad_weights, (const double*)scale, n,
                                             (double*)d_grad_out, (double*)d_x, d_weights,
                                             reinterpret_cast<int*>(status), s),
                       "fc_linear_dbwd");
}

// ------------------------------------------------------------------ halo exchange

int fc_halo_pack(const void* x, int64_t n_rows, int64_t row_elems, int32_t dtype, const int64_t* idx,
                 int64_t n_idx, void* buf, int32_t* status, fc_stream_t stream) {
  if (n_rows < 0 || row_elems < 0 || n_idx < 0) return fail(FC_ERR_INVALID, "fc_halo_pack: negative size");
  if (dtype != FC_F32 && dtype != FC_F64) return fail(FC_ERR_INVALID, "fc_halo_pack: dtype must be f32 or f64");
  if (n_idx == 0 || row_elems == 0) return FC_OK;
  if (!idx || !buf || (n_rows > 0 && !x)) return fail(FC_ERR_INVALID, "fc_halo_pack: null tensor");
  cudaStream_t s = (cudaStream_t)stream;
  int* st = reinterpret_cast<int*>(status);
  if (dtype == FC_F32)
    return launch_status(halo_pack_dispatch<float>((const float*)x, n_rows, row_elems, idx, n_idx, (float*)buf, st, s),
                         "fc_halo_pack");
  return launch_status(halo_pack_dispatch<double>((const double*)x, n_rows, row_elems, idx, n_idx, (double*)buf, st,
                                                  s),
                       "fc_halo_pack");
}

int fc_halo_unpack(const void* buf, int64_t n_idx, int64_t row_elems, int32_t dtype, const int64_t* idx, void* x,
                   int64_t n_rows, int32_t accumulate, int32_t* status, fc_stream_t stream) {
  if (n_rows < 0 || row_elems < 0 || n_idx < 0) return fail(FC_ERR_INVALID, "fc_halo_unpack: negative size");
  if (dtype != FC_F32 && dtype != FC_F64) return fail(FC_ERR_INVALID, "fc_halo_unpack: dtype must be f32 or f64");
  if (n_idx == 0 || row_elems == 0) return FC_OK;
  if (!idx || !buf || (n_rows > 0 && !x)) return fail(FC_ERR_INVALID, "fc_halo_unpack: null tensor");
  cudaStream_t s = (cudaStream_t)stream;
  int* st = reinterpret_cast<int*>(status);
  if (dtype == FC_F32)
    return launch_status(halo_unpack_dispatch<float>((const float*)buf, row_elems, idx, n_idx, (float*)x, n_rows,
                                                     accumulate, st, s),
                         "fc_halo_unpack");
  return launch_status(halo_unpack_dispatch<double>((const double*)buf, row_elems, idx, n_idx, (double*)x, n_rows,
                                                    accumulate, st, s),
                       "fc_halo_unpack");
}

// ------------------------------------------------------------------ linear maps, split weights

static int presplit_check(const fc_linear_desc* desc, const void* const* weights, const void* const* split,
                          const char* what) {
  if (int rc = check_linear(desc)) return rc;
  if (desc->dtype != FC_F32) return fail(FC_ERR_UNSUPPORTED, "%s: split weights are for float32 maps", what);
  if (desc->n_active > 0 && (!weights || !split)) return fail(FC_ERR_INVALID, "%s: null weight array", what);
  for (int l = 0; l < desc->n_active; ++l)
    if (!weights[l] || !split[l]) return fail(FC_ERR_INVALID, "%s: null weight for rank %d", what, l);
  return FC_OK;
}

int fc_linear_presplit(const fc_linear_desc* desc, const void* const* weights, int32_t backward,
                       void* const* split, fc_stream_t stream) {
  if (int rc = presplit_check(desc, weights, split, "fc_linear_presplit")) return rc;
  const cudaStream_t s = (cudaStream_t)stream;
  for (int l = 0; l < desc->n_active; ++l) {
    const int fi = desc->f_in_values[l], fo = desc->f_out_values[l];
    // forward B(k, n) = W[n][k] (k = in, n = out); backward B(k, n) = W[k][n] (k = out, n = in)
    const int rc = backward ? lin_presplit((const float*)weights[l], fi, 0, fo, fi, (float*)split[l], s)
                            : lin_presplit((const float*)weights[l], fi, 1, fi, fo, (float*)split[l], s);
    if (rc) return launch_status(rc, "fc_linear_presplit");
  }
  return FC_OK;
}

int fc_linear_fwd_presplit(const fc_linear_desc* desc, const void* x, const void* const* weights,
                           const void* const* split, const void* scale, int64_t n, void* out, int32_t* status,
                           fc_stream_t stream) {
  if (int rc = presplit_check(desc, weights, split, "fc_linear_fwd_presplit")) return rc;
  if (n < 0) return fail(FC_ERR_INVALID, "fc_linear_fwd_presplit: negative size");
  if (n == 0 || desc->out_dim == 0) return FC_OK;
  if (!out || (desc->n_active > 0 && (!x || !scale))) return fail(FC_ERR_INVALID, "fc_linear_fwd_presplit: null tensor");
  return launch_status(linear_fwd_t<float>(desc, (const float*)x, weights, (const float*)scale, n, (float*)out,
                                           reinterpret_cast<int*>(status), (cudaStream_t)stream, split),
                       "fc_linear_fwd_presplit");
}

int fc_linear_bwd_presplit(const fc_linear_desc* desc, const void* grad_out, const void* x,
                           const void* const* weights, const void* const* split, const void* scale, int64_t n,
                           void* grad_x, void* const* grad_weights, int32_t* status, fc_stream_t stream) {
  if (int rc = presplit_check(desc, weights, split, "fc_linear_bwd_presplit")) return rc;
  if (n < 0) return fail(FC_ERR_INVALID, "fc_linear_bwd_presplit: negative size");
  if (desc->n_active > 0 && (!scale || (n > 0 && (!grad_out || !x))))
    return fail(FC_ERR_INVALID, "fc_linear_bwd_presplit: null tensor");
  return launch_status(linear_bwd_t<float>(desc, (const float*)grad_out, (const float*)x, weights,
                                           (const float*)scale, n, (float*)grad_x, grad_weights,
                                           reinterpret_cast<int*>(status), (cudaStream_t)stream, split),
                       "fc_linear_bwd_presplit");
}

// Residual forms (fc_linear_fwd_residual / fc_linear_bwd_residual): the map's GEMM adds
// the residual in its epilogue (LinGemmArgs act 3). TMA path only.
static int linear_residual_t(const fc_linear_desc* d, bool backward, const float* a_rows, const void* const* weights,
                             const void* const* split, const float* scale, int64_t n, const float* residual,
                             float* c, int* status, cudaStream_t s, const char* what) {
  if (int rc = check_linear(d)) return rc;
  if (d->dtype != FC_F32 || d->act != FC_ACT_NONE)
    return fail(FC_ERR_UNSUPPORTED, "%s: float32 maps without an input activation only", what);
  if (n < 0) return fail(FC_ERR_INVALID, "%s: negative size", what);
  const int64_t a_dim = backward ? d->out_dim : d->in_dim, c_dim = backward ? d->in_dim : d->out_dim;
  int64_t prev = 0;
  for (int l = 0; l < d->n_active; ++l) {
    const int64_t off = backward ? d->in_offsets[l] : d->out_offsets[l];
    if (off != prev) return fail(FC_ERR_UNSUPPORTED, "%s: the active ranks must cover the output row", what);
    prev = off + (int64_t)d->m_values[l] * (backward ? d->f_in_values[l] : d->f_out_values[l]);
  }
  if (prev != c_dim) return fail(FC_ERR_UNSUPPORTED, "%s: the active ranks must cover the output row", what);
  if (n == 0 || d->n_active == 0) return FC_OK;
  if (!a_rows || !weights || !scale || !residual || !c) return fail(FC_ERR_INVALID, "%s: null tensor", what);
#ifdef FC_HOST_EMU
  (void)a_dim; (void)split; (void)status; (void)s;
  return fail(FC_ERR_UNSUPPORTED, "%s: tensor-core path only", what);
#else
  LinGemmArgs<float> args[FC_MAX_L + 1];
  for (int l = 0; l < d->n_active; ++l) {
    LinGemmArgs<float>& a = args[l];
    const int64_t a_off = backward ? d->out_offsets[l] : d->in_offsets[l];
    const int64_t c_off = backward ? d->in_offsets[l] : d->out_offsets[l];
    const int ka = backward ? d->f_out_values[l] : d->f_in_values[l];
    const int nc = backward ? d->f_in_values[l] : d->f_out_values[l];
    a.a = LinRows<float>{a_rows, a_dim, a_off, ka, d->m_values[l]};
    a.w = (const float*)weights[l];
    a.ldw = d->f_in_values[l];
    a.trans_b = backward ? 0 : 1;
    a.bsplit = split ? (const float*)split[l] : nullptr;
    a.scale = scale + l;
    a.c = LinRows<float>{c, c_dim, c_off, nc, d->m_values[l]};
    a.R = n * d->m_values[l];
    a.K = ka;
    a.N = nc;
    a.act = 3;
    a.aux = LinRows<float>{residual, c_dim, c_off, nc, d->m_values[l]};
  }
  const bool split3 = d->precision != FC_PREC_TF32;
  int rc = d->n_active > 1 ? lin_gemm_tma_grouped(args, d->n_active, split3, status, s) : 1;
  for (int l = 0; rc == 1 && l < d->n_active; ++l) {
    const int r = lin_gemm_tma(args[l], split3, status, s);
    if (r == 1) return fail(FC_ERR_UNSUPPORTED, "%s: layout not on the tensor-core path (rank %d)", what, l);
    if (r) return r;
    if (l == d->n_active - 1) rc = 0;
  }
  return rc;
#endif
}

int fc_linear_fwd_residual(const fc_linear_desc* desc, const void* x, const void* const* weights,
                           const void* const* split, const void* scale, int64_t n, const void* residual, void* out,
                           int32_t* status, fc_stream_t stream) {
  const int rc = linear_residual_t(desc, false, (const float*)x, weights, split, (const float*)scale, n,
                                   (const float*)residual, (float*)out, reinterpret_cast<int*>(status),
                                   (cudaStream_t)stream, "fc_linear_fwd_residual");
  return rc == FC_ERR_LAUNCH ? launch_status(rc, "fc_linear_fwd_residual") : rc;
}

int fc_linear_bwd_residual(const fc_linear_desc* desc, const void* grad_out, const void* const* weights,
                           const void* const* split, const void* scale, int64_t n, const void* residual,
                           void* grad_x, int32_t* status, fc_stream_t stream) {
  const int rc = linear_residual_t(desc, true, (const float*)grad_out, weights, split, (const float*)scale, n,
                                   (const float*)residual, (float*)grad_x, reinterpret_cast<int*>(status),
                                   (cudaStream_t)stream, "fc_linear_bwd_residual");
  return rc == FC_ERR_LAUNCH ? launch_status(rc, "fc_linear_bwd_residual") : rc;
}

// Convolution forward for callers that cannot allocate device memory (see the header).
int fc_tp_conv_fwd_noalloc(const fc_tp_desc* desc, const void* in1, const void* in2, const void* weights,
                           const int64_t* idx_i, const int64_t* idx_j, int64_t n_nodes, int64_t n_in1_rows,
                           int64_t n_edges, void* out, int32_t* status, fc_stream_t stream) {
  if (int rc = check_desc(desc)) return rc;
  if (n_nodes < 0 || n_in1_rows < 0 || n_edges < 0)
    return fail(FC_ERR_INVALID, "fc_tp_conv_fwd_noalloc: negative size");
  if (n_nodes > kNoAllocMaxNodes)
    return fail(FC_ERR_CAPACITY,
                "fc_tp_conv_fwd_noalloc: %lld receiver nodes exceed the fixed workspace of %lld nodes; use "
                "fc_build_rowptr + fc_tp_fwd with a caller-provided workspace",
                (long long)n_nodes, (long long)kNoAllocMaxNodes);
  if (n_nodes == 0) return FC_OK;
  if (n_edges > 0 && (idx_i == nullptr || idx_j == nullptr))
    return fail(FC_ERR_INVALID, "fc_tp_conv_fwd_noalloc: null index array");
  int64_t* rowptr = nullptr;
  if (int rc = noalloc_rowptr(&rowptr)) return rc;
  // the workspace is fully rewritten by this call, so nothing needs clearing
  if (int rc = fc_build_rowptr(idx_i, n_edges, n_nodes, rowptr, status, stream)) return rc;
  return fc_tp_fwd(desc, in1, in2, weights, rowptr, idx_j, n_nodes, n_in1_rows, n_edges, out, status, stream);
}

// ------------------------------------------------------------------ RMS layer norm

static int rms_check(int l_max, int features, int dtype, int64_t n_rows, const char* what) {
  if (l_max < 0 || l_max > FC_MAX_L)
    return fail(FC_ERR_UNSUPPORTED, "%s: l_max %d outside 0..%d", what, l_max, FC_MAX_L);
  if (features <= 0 || features > 1024)
    return fail(FC_ERR_UNSUPPORTED, "%s: features must be in 1..1024 (got %d)", what, features);
  if (dtype != FC_F32 && dtype != FC_F64) return fail(FC_ERR_INVALID, "%s: dtype must be f32 or f64", what);
  if (n_rows < 0) return fail(FC_ERR_INVALID, "%s: negative row count", what);
  return FC_OK;
}

int fc_rms_norm_fwd(int32_t l_max, int32_t features, int32_t dtype, const void* x, const void* gains,
                    const void* l_weights, double eps, int64_t n_rows, void* y, void* rstd, fc_stream_t stream) {
  if (int rc = rms_check(l_max, features, dtype, n_rows, "fc_rms_norm_fwd")) return rc;
  if (n_rows == 0) return FC_OK;
  if (!x || !gains || !l_weights || !y || !rstd) return fail(FC_ERR_INVALID, "fc_rms_norm_fwd: null pointer");
  const cudaStream_t s = (cudaStream_t)stream;
  if (dtype == FC_F32)
    return launch_status(rms_norm_fwd_dispatch<float>(l_max, (const float*)x, (const float*)gains,
                                                      (const float*)l_weights, (float)eps, features, n_rows,
                                                      (float*)y, (float*)rstd, s),
                         "fc_rms_norm_fwd");
  return launch_status(rms_norm_fwd_dispatch<double>(l_max, (const double*)x, (const double*)gains,
                                                     (const double*)l_weights, eps, features, n_rows, (double*)y,
                                                     (double*)rstd, s),
                       "fc_rms_norm_fwd");
}

int fc_rms_norm_bwd(int32_t l_max, int32_t features, int32_t dtype, const void* grad_y, const void* x,
                    const void* gains, const void* l_weights, const void* rstd, int64_t n_rows, void* grad_x,
                    fc_stream_t stream) {
  if (int rc = rms_check(l_max, features, dtype, n_rows, "fc_rms_norm_bwd")) return rc;
  if (n_rows == 0) return FC_OK;
  if (!grad_y || !x || !gains || !l_weights || !rstd || !grad_x)
    return fail(FC_ERR_INVALID, "fc_rms_norm_bwd: null pointer");
  const cudaStream_t s = (cudaStream_t)stream;
  if (dtype == FC_F32)
    return launch_status(rms_norm_bwd_dispatch<float>(l_max, (const float*)grad_y, (const float*)x,
                                                      (const float*)gains, (const float*)l_weights,
                                                      (const float*)rstd, features, n_rows, (float*)grad_x, s),
                         "fc_rms_norm_bwd");
  return launch_status(rms_norm_bwd_dispatch<double>(l_max, (const double*)grad_y, (const double*)x,
                                                     (const double*)gains, (const double*)l_weights,
                                                     (const double*)rstd, features, n_rows, (double*)grad_x, s),
                       "fc_rms_norm_bwd");
}

// ------------------------------------------------------------------ equivariant gate

int fc_gate_fwd(int32_t l_max, int32_t features, int32_t dtype, const void* values, const void* gates,
                int64_t n_rows, void* y, fc_stream_t stream) {
  if (int rc = rms_check(l_max, features, dtype, n_rows, "fc_gate_fwd")) return rc;
  if (n_rows == 0) return FC_OK;
  if (!values || !gates || !y) return fail(FC_ERR_INVALID, "fc_gate_fwd: null pointer");
  const cudaStream_t s = (cudaStream_t)stream;
  if (dtype == FC_F32)
    return launch_status(gate_fwd_dispatch<float>(l_max, (const float*)values, (const float*)gates, (float*)y,
                                                  features, n_rows, s),
                         "fc_gate_fwd");
  return launch_status(gate_fwd_dispatch<double>(l_max, (const double*)values, (const double*)gates, (double*)y,
                                                 features, n_rows, s),
                       "fc_gate_fwd");
}

int fc_gate_bwd(int32_t l_max, int32_t features, int32_t dtype, const void* grad_y, const void* values,
                const void* gates, int64_t n_rows, void* grad_values, void* grad_gates, fc_stream_t stream) {
  if (int rc = rms_check(l_max, features, dtype, n_rows, "fc_gate_bwd")) return rc;
  if (n_rows == 0) return FC_OK;
  if (!grad_y || !values || !gates) return fail(FC_ERR_INVALID, "fc_gate_bwd: null pointer");
  const cudaStream_t s = (cudaStream_t)stream;
  if (dtype == FC_F32)
    return launch_status(gate_bwd_dispatch<float>(l_max, (const float*)grad_y, (const float*)values,
                                                  (const float*)gates, (float*)grad_values, (float*)grad_gates,
                                                  features, n_rows, s),
                         "fc_gate_bwd");
  return launch_status(gate_bwd_dispatch<double>(l_max, (const double*)grad_y, (const double*)values,
                                                 (const double*)gates, (double*)grad_values, (double*)grad_gates,
                                                 features, n_rows, s),
                       "fc_gate_bwd");
}

// ------------------------------------------------------------------ edge expansion

int fc_edge_expand_fwd(int32_t l_max, int32_t features, int32_t per_rank, int32_t dtype, const void* moments,
                       const void* h, int64_t n_rows, void* out, fc_stream_t stream) {
  if (int rc = rms_check(l_max, features, dtype, n_rows, "fc_edge_expand_fwd")) return rc;
  if (n_rows == 0) return FC_OK;
  if (!moments || !h || !out) return fail(FC_ERR_INVALID, "fc_edge_expand_fwd: null pointer");
  const cudaStream_t s = (cudaStream_t)stream;
  const int pr = per_rank ? 1 : 0;
  if (dtype == FC_F32)
    return launch_status(edge_expand_fwd_dispatch<float>(l_max, (const float*)moments, (const float*)h, features, pr,
                                                         n_rows, (float*)out, s),
                         "fc_edge_expand_fwd");
  return launch_status(edge_expand_fwd_dispatch<double>(l_max, (const double*)moments, (const double*)h, features, pr,
                                                        n_rows, (double*)out, s),
                       "fc_edge_expand_fwd");
}

int fc_edge_expand_bwd(int32_t l_max, int32_t features, int32_t per_rank, int32_t dtype, const void* grad_out,
                       const void* moments, const void* h, int64_t n_rows, void* grad_moments, void* grad_h,
                       fc_stream_t stream) {
  if (int rc = rms_check(l_max, features, dtype, n_rows, "fc_edge_expand_bwd")) return rc;
  if (n_rows == 0) return FC_OK;
  if (!grad_out || !moments || !h) return fail(FC_ERR_INVALID, "fc_edge_expand_bwd: null pointer");
  const cudaStream_t s = (cudaStream_t)stream;
  const int pr = per_rank ? 1 : 0;
  if (dtype == FC_F32)
    return launch_status(edge_expand_bwd_dispatch<float>(l_max, (const float*)grad_out, (const float*)moments,
                                                         (const float*)h, features, pr, n_rows, (float*)grad_moments,
                                                         (float*)grad_h, s),
                         "fc_edge_expand_bwd");
  return launch_status(edge_expand_bwd_dispatch<double>(l_max, (const double*)grad_out, (const double*)moments,
                                                        (const double*)h, features, pr, n_rows,
                                                        (double*)grad_moments, (double*)grad_h, s),
                       "fc_edge_expand_bwd");
}

// ------------------------------------------------------------------ edge geometry

static int geom_check(const fc_edge_geometry_desc* d, int64_t n_nodes, int64_t n_cells, int64_t n_edges,
                      const char* what, GeomParams* p) {
  if (!d) return fail(FC_ERR_INVALID, "%s: null descriptor", what);
  if (d->l_max < 0 || d->l_max > 3) return fail(FC_ERR_UNSUPPORTED, "%s: l_max %d outside 0..3", what, d->l_max);
  if (d->n_radial < 1 || d->n_radial > 64)
    return fail(FC_ERR_UNSUPPORTED, "%s: n_radial %d outside 1..64", what, d->n_radial);
  if (d->poly_order < 2 || d->poly_order > 64)
    return fail(FC_ERR_UNSUPPORTED, "%s: poly_order %d outside 2..64", what, d->poly_order);
  if (d->dtype != FC_F32 && d->dtype != FC_F64) return fail(FC_ERR_INVALID, "%s: dtype must be f32 or f64", what);
  if (!(d->r_max > d->r_min) || !(d->r_cut > 0.0)) return fail(FC_ERR_INVALID, "%s: need r_max > r_min, r_cut > 0", what);
  if (n_nodes < 0 || n_edges < 0 || n_cells < 0) return fail(FC_ERR_INVALID, "%s: negative size", what);
  if (d->use_shifts && n_cells < 1 && n_edges > 0) return fail(FC_ERR_INVALID, "%s: shifts need a cell", what);
  p->l_max = d->l_max; p->n_radial = d->n_radial; p->cosine = d->cosine ? 1 : 0;
  p->poly_order = d->poly_order; p->use_shifts = d->use_shifts ? 1 : 0;
  p->r_min = d->r_min; p->r_max = d->r_max; p->r_cut = d->r_cut;
  p->n_nodes = n_nodes; p->n_edges = n_edges; p->n_cells = n_cells;
  p->vectors_given = 0;
  return FC_OK;
}

int fc_edge_geometry_fwd(const fc_edge_geometry_desc* desc, const void* positions, int64_t n_nodes,
                         const void* cells, int64_t n_cells, const int32_t* shifts, const int64_t* edge_index,
                         const int64_t* batch, int64_t n_edges, void* edge_attrs, void* radial, int32_t* status,
                         fc_stream_t stream) {
  GeomParams p;
  if (int rc = geom_check(desc, n_nodes, n_cells, n_edges, "fc_edge_geometry_fwd", &p)) return rc;
  if (n_edges == 0) return FC_OK;
  if (!positions || !edge_index || !edge_attrs || !radial || (p.use_shifts && (!cells || !shifts)) ||
      (p.use_shifts && n_cells > 1 && !batch))
    return fail(FC_ERR_INVALID, "fc_edge_geometry_fwd: null pointer");
  const cudaStream_t s = (cudaStream_t)stream;
  int* st = reinterpret_cast<int*>(status);
  if (desc->dtype == FC_F32)
    return launch_status(geom_fwd_dispatch<float>(p, (const float*)positions, (const float*)cells, shifts,
                                                  edge_index, batch, (float*)edge_attrs, (float*)radial, st, s),
                         "fc_edge_geometry_fwd");
  return launch_status(geom_fwd_dispatch<double>(p, (const double*)positions, (const double*)cells, shifts,
                                                 edge_index, batch, (double*)edge_attrs, (double*)radial, st, s),
                       "fc_edge_geometry_fwd");
}

int fc_edge_geometry_bwd(const fc_edge_geometry_desc* desc, const void* positions, int64_t n_nodes,
                         const void* cells, int64_t n_cells, const int32_t* shifts, const int64_t* edge_index,
                         const int64_t* batch, int64_t n_edges, const void* grad_attrs, const void* grad_radial,
                         void* grad_positions, void* grad_cells, int32_t* status, fc_stream_t stream) {
  GeomParams p;
  if (int rc = geom_check(desc, n_nodes, n_cells, n_edges, "fc_edge_geometry_bwd", &p)) return rc;
  if (!grad_positions && n_nodes > 0) return fail(FC_ERR_INVALID, "fc_edge_geometry_bwd: null grad_positions");
  const cudaStream_t s = (cudaStream_t)stream;
  const int esz = desc->dtype == FC_F32 ? 4 : 8;
  int rc = 0;
  if (n_nodes > 0) rc |= zero_fill(grad_positions, n_nodes * 3 * esz, s);
  if (grad_cells && n_cells > 0) rc |= zero_fill(grad_cells, n_cells * 9 * esz, s);
  if (rc) return launch_status(FC_ERR_LAUNCH, "fc_edge_geometry_bwd (zero fill)");
  if (n_edges == 0 || (!grad_attrs && !grad_radial)) return FC_OK;
  if (!positions || !edge_index || (p.use_shifts && (!cells || !shifts)) || (p.use_shifts && n_cells > 1 && !batch))
    return fail(FC_ERR_INVALID, "fc_edge_geometry_bwd: null pointer");
  int* st = reinterpret_cast<int*>(status);
  if (desc->dtype == FC_F32)
    return launch_status(geom_bwd_dispatch<float>(p, (const float*)positions, (const float*)cells, shifts, edge_index,
                                                  batch, (const float*)grad_attrs, (const float*)grad_radial,
                                                  (float*)grad_positions, (float*)grad_cells, st, s),
                         "fc_edge_geometry_bwd");
  return launch_status(geom_bwd_dispatch<double>(p, (const double*)positions, (const double*)cells, shifts, edge_index,
                                                 batch, (const double*)grad_attrs, (const double*)grad_radial,
                                                 (double*)grad_positions, (double*)grad_cells, st, s),
                       "fc_edge_geometry_bwd");
}

int fc_edge_geometry_vec_fwd(const fc_edge_geometry_desc* desc, const void* vectors, int64_t n_edges,
                             void* edge_attrs, void* radial, int32_t* status, fc_stream_t stream) {
  GeomParams p;
  if (int rc = geom_check(desc, 0, 0, n_edges, "fc_edge_geometry_vec_fwd", &p)) return rc;
  if (n_edges == 0) return FC_OK;
  if (!vectors || !edge_attrs || !radial) return fail(FC_ERR_INVALID, "fc_edge_geometry_vec_fwd: null pointer");
  p.use_shifts = 0;
  p.vectors_given = 1;
  const cudaStream_t s = (cudaStream_t)stream;
  int* st = reinterpret_cast<int*>(status);
  if (desc->dtype == FC_F32)
    return launch_status(geom_fwd_dispatch<float>(p, (const float*)vectors, nullptr, nullptr, nullptr, nullptr,
                                                  (float*)edge_attrs, (float*)radial, st, s),
                         "fc_edge_geometry_vec_fwd");
  return launch_status(geom_fwd_dispatch<double>(p, (const double*)vectors, nullptr, nullptr, nullptr, nullptr,
                                                 (double*)edge_attrs, (double*)radial, st, s),
                       "fc_edge_geometry_vec_fwd");
}

int fc_edge_geometry_vec_bwd(const fc_edge_geometry_desc* desc, const void* vectors, int64_t n_edges,
                             const void* grad_attrs, const void* grad_radial, void* grad_vectors, int32_t* status,
                             fc_stream_t stream) {
  GeomParams p;
  if (int rc = geom_check(desc, 0, 0, n_edges, "fc_edge_geometry_vec_bwd", &p)) return rc;
  if (n_edges == 0) return FC_OK;
  if (!vectors || !grad_vectors) return fail(FC_ERR_INVALID, "fc_edge_geometry_vec_bwd: null pointer");
  p.use_shifts = 0;
  p.vectors_given = 1;
  const cudaStream_t s = (cudaStream_t)stream;
  if (!grad_attrs && !grad_radial) {
    const int esz = desc->dtype == FC_F32 ? 4 : 8;
    if (zero_fill(grad_vectors, n_edges * 3 * esz, s)) return launch_status(FC_ERR_LAUNCH, "fc_edge_geometry_vec_bwd");
    return FC_OK;
  }
  int* st = reinterpret_cast<int*>(status);
  if (desc->dtype == FC_F32)
    return launch_status(geom_bwd_dispatch<float>(p, (const float*)vectors, nullptr, nullptr, nullptr, nullptr,
                                                  (const float*)grad_attrs, (const float*)grad_radial,
                                                  (float*)grad_vectors, nullptr, st, s),
                         "fc_edge_geometry_vec_bwd");
  return launch_status(geom_bwd_dispatch<double>(p, (const double*)vectors, nullptr, nullptr, nullptr, nullptr,
                                                 (const double*)grad_attrs, (const double*)grad_radial,
                                                 (double*)grad_vectors, nullptr, st, s),
                       "fc_edge_geometry_vec_bwd");
}

// ------------------------------------------------------------------ neighbour list

static int nl_check(const fc_nl_desc* d, int64_t n, const char* what) {
  if (!d) return fail(FC_ERR_INVALID, "%s: null descriptor", what);
  if (n < 0 || n > 0x7fffffffLL) return fail(FC_ERR_INVALID, "%s: atom count %lld outside 0..2^31-1", what,
                                             (long long)n);
  if (!(d->r_max_sq > 0.0)) return fail(FC_ERR_INVALID, "%s: r_max must be positive", what);
  for (int k = 0; k < 3; ++k) {
    if (!(d->lengths[k] > 0.0) || !(d->inv_lengths[k] > 0.0))
      return fail(FC_ERR_INVALID, "%s: cell lengths must be positive", what);
    if (d->bins[k] < 3)
      return fail(FC_ERR_UNSUPPORTED, "%s: %d bins on axis %d; the cell list needs at least 3 (use the host list)",
                  what, d->bins[k], k);
    if (!(d->bin_widths[k] * d->bin_widths[k] >= d->r_max_sq))
      return fail(FC_ERR_INVALID, "%s: bin width below r_max on axis %d", what, k);
  }
  if ((int64_t)d->bins[0] * d->bins[1] * d->bins[2] > (int64_t)1 << 30)
    return fail(FC_ERR_UNSUPPORTED, "%s: too many bins", what);
  return FC_OK;
}

int64_t fc_neighbor_workspace_bytes(const fc_nl_desc* desc, int64_t n_atoms) {
  if (int rc = nl_check(desc, n_atoms, "fc_neighbor_workspace_bytes")) return rc;
  return nl_workspace_bytes(n_atoms, (int64_t)desc->bins[0] * desc->bins[1] * desc->bins[2]);
}

int fc_neighbor_count(const fc_nl_desc* desc, const double* positions, int64_t n_atoms, void* workspace,
                      int64_t* rowptr, int32_t* status, fc_stream_t stream) {
  if (int rc = nl_check(desc, n_atoms, "fc_neighbor_count")) return rc;
  if (!rowptr || (n_atoms > 0 && (!positions || !workspace)))
    return fail(FC_ERR_INVALID, "fc_neighbor_count: null pointer");
#ifdef FC_HOST_EMU
  (void)status; (void)stream;
  return fail(FC_ERR_UNSUPPORTED, "fc_neighbor_count: GPU kernel only");
#else
  if (n_atoms == 0)
    return cudaMemsetAsync(rowptr, 0, sizeof(int64_t), (cudaStream_t)stream) == cudaSuccess
               ? FC_OK
               : fail(FC_ERR_LAUNCH, "fc_neighbor_count: memset failed");
  return launch_status(nl_count(desc, positions, n_atoms, workspace, rowptr, reinterpret_cast<int*>(status),
                                (cudaStream_t)stream),
                       "fc_neighbor_count");
#endif
}

int fc_neighbor_fill(const fc_nl_desc* desc, int64_t n_atoms, const void* workspace, const int64_t* rowptr,
                     int64_t n_edges, int64_t* edge_index, int32_t* shifts, int32_t* status, fc_stream_t stream) {
  if (int rc = nl_check(desc, n_atoms, "fc_neighbor_fill")) return rc;
  if (n_edges < 0) return fail(FC_ERR_INVALID, "fc_neighbor_fill: negative edge count");
  if (n_atoms == 0 || n_edges == 0) return FC_OK;
  if (!workspace || !rowptr || !edge_index || !shifts) return fail(FC_ERR_INVALID, "fc_neighbor_fill: null pointer");
#ifdef FC_HOST_EMU
  (void)status; (void)stream;
  return fail(FC_ERR_UNSUPPORTED, "fc_neighbor_fill: GPU kernel only");
#else
  return launch_status(nl_fill(desc, n_atoms, workspace, rowptr, n_edges, edge_index, shifts,
                               reinterpret_cast<int*>(status), (cudaStream_t)stream),
                       "fc_neighbor_fill");
#endif
}

// Muon Newton-Schulz orthogonalisation (see the header).
int fc_newton_schulz(const void* update, int dtype, int64_t batch, int rows, int cols, const float* coeffs,
                     int steps, const float* polish, int polish_steps, float eps, void* out, int32_t* status,
                     fc_stream_t stream) {
  if (batch < 0 || rows <= 0 || cols <= 0 || steps < 0 || polish_steps < 0)
    return fail(FC_ERR_INVALID, "fc_newton_schulz: invalid sizes");
  if (dtype != FC_F32 && dtype != FC_BF16) return fail(FC_ERR_INVALID, "fc_newton_schulz: dtype must be f32 or bf16");
  if (batch == 0) return FC_OK;
  if (!update || !out || !coeffs || (polish_steps > 0 && !polish))
    return fail(FC_ERR_INVALID, "fc_newton_schulz: null pointer");
  if (rows % 8 != 0 || cols % 8 != 0)
    return fail(FC_ERR_UNSUPPORTED, "fc_newton_schulz: rows and cols must be multiples of 8 (got %d x %d)", rows,
                cols);
#ifdef FC_HOST_EMU
  (void)eps; (void)status; (void)stream;
  return fail(FC_ERR_UNSUPPORTED, "fc_newton_schulz: tensor-core kernel only");
#else
  return launch_status(ns_orthogonalize(update, dtype, batch, rows, cols, coeffs, steps, polish, polish_steps, eps,
                                        out, status, (cudaStream_t)stream),
                       "fc_newton_schulz");
#endif
}

}  // extern "C"
