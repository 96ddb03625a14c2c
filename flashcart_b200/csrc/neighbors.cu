// Periodic neighbour list of an orthorhombic cell on the GPU, in the canonical order of
// flashcart_b200/data/neighbors.py (receiver i ascending, then sender j, then the image
// shift S lexicographically), float64 distance test.
//
//   prepare   one thread per atom: wrapped position pw = p - floor(p * (1/L)) L, the
//             integer wrap, the cell-list bin (bins of width L / nb per axis), bin counts;
//   scan      bin starts (one CTA, chunked exclusive scan);
//   scatter   atoms into bin order;
//   count     one thread per receiver: the 27 neighbouring bins (periodic images
//             -1 / 0 / +1 per axis), |pw_j + img L - pw_i|^2 < r_max^2, self pair excluded;
//   scan      receiver CSR rowptr;
//   fill      the same walk writes (j, S = img - wrap_j + wrap_i) into the receiver's
//             segment, then an insertion sort puts the segment in (j, S) order.
// Every floating-point operation is an explicit round-to-nearest intrinsic (no FMA
// contraction), so the arithmetic is the host list's: pw = p - w*L with w = floor(p * 1/L),
// bin = trunc(pw / (L / nb)), v = (pw_j + img*L) - pw_i, d2 = (v0*v0 + v1*v1) + v2*v2.
#include "fc_base.cuh"

namespace fc {

struct NlLayout {
  double* pw;       // n x 3
  int32_t* wrap;    // n x 3
  int32_t* bid;     // n
  int32_t* sorted;  // n   atoms in bin order
  int32_t* start;   // nbins + 1
  int32_t* fill;    // nbins
};

inline int64_t nl_align(int64_t b) { return (b + 255) & ~int64_t(255); }

int64_t nl_workspace_bytes(int64_t n, int64_t nbins) {
  return nl_align(24 * n) + nl_align(12 * n) + 2 * nl_align(4 * n) + nl_align(4 * (nbins + 1)) + nl_align(4 * nbins);
}

inline NlLayout nl_layout(void* ws, int64_t n, int64_t nbins) {
  uint8_t* p = static_cast<uint8_t*>(ws);
  NlLayout L;
  L.pw = reinterpret_cast<double*>(p);
  p += nl_align(24 * n);
  L.wrap = reinterpret_cast<int32_t*>(p);
  p += nl_align(12 * n);
  L.bid = reinterpret_cast<int32_t*>(p);
  p += nl_align(4 * n);
  L.sorted = reinterpret_cast<int32_t*>(p);
  p += nl_align(4 * n);
  L.start = reinterpret_cast<int32_t*>(p);
  p += nl_align(4 * (nbins + 1));
  L.fill = reinterpret_cast<int32_t*>(p);
  return L;
}

#ifndef FC_HOST_EMU

struct NlGeom {
  double L[3], inv_L[3], width[3], r2;
  int nb[3];
};

__device__ __forceinline__ bool nl_less(int ja, const int* sa, int jb, const int* sb) {
  if (ja != jb) return ja < jb;
  if (sa[0] != sb[0]) return sa[0] < sb[0];
  if (sa[1] != sb[1]) return sa[1] < sb[1];
  return sa[2] < sb[2];
}

__global__ void nl_prepare_kernel(const double* __restrict__ pos, int64_t n, NlGeom g, NlLayout w, int* status) {
  for (int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; a < n; a += (int64_t)gridDim.x * blockDim.x) {
    int b[3];
    for (int k = 0; k < 3; ++k) {
      const double p = pos[3 * a + k];
      const double wr = floor(__dmul_rn(p, g.inv_L[k]));
      const double q = __dsub_rn(p, __dmul_rn(wr, g.L[k]));
      w.pw[3 * a + k] = q;
      w.wrap[3 * a + k] = (int32_t)wr;
      const double t = __ddiv_rn(q, g.width[k]);
      long long bk = 0;
      if (t == t && t > -1.0 && t < 2.0 * g.nb[k]) {
        bk = (long long)t;  // truncation, as the host list's astype(int64)
      } else {
        fc_flag(status, FC_DEV_BAD_INDEX);  // a position that did not wrap into the cell (NaN / inf)
      }
      if (bk > g.nb[k] - 1) bk = g.nb[k] - 1;
      if (bk < 0) bk = 0;
      b[k] = (int)bk;
    }
    const int id = (b[0] * g.nb[1] + b[1]) * g.nb[2] + b[2];
    w.bid[a] = id;
    atomicAdd(&w.start[id], 1);
  }
}

// Exclusive scan of `count` values in place (int32 or int64), one CTA of 1024 threads,
// chunk by chunk with a carry; data[count] receives the total.
template <typename V>
__global__ void nl_scan_kernel(V* data, int64_t count) {
  __shared__ V sh[1024];
  __shared__ V carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < count; base += 1024) {
    const int64_t i = base + threadIdx.x;
    const V v = i < count ? data[i] : V(0);
    sh[threadIdx.x] = v;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {  // Hillis-Steele inclusive scan
      const V t = threadIdx.x >= o ? sh[threadIdx.x - o] : V(0);
      __syncthreads();
      sh[threadIdx.x] += t;
      __syncthreads();
    }
    if (i < count) data[i] = carry + sh[threadIdx.x] - v;
    __syncthreads();
    if (threadIdx.x == 1023) carry += sh[1023];
    __syncthreads();
  }
  if (threadIdx.x == 0) data[count] = carry;
}

__global__ void nl_scatter_kernel(int64_t n, NlLayout w) {
  for (int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; a < n; a += (int64_t)gridDim.x * blockDim.x) {
    const int id = w.bid[a];
    const int slot = atomicAdd(&w.fill[id], 1);
    w.sorted[w.start[id] + slot] = (int32_t)a;
  }
}

// Walk the 27 neighbouring bins of receiver i; visit(j, img) for every pair within r_max.
template <typename Visit>
__device__ __forceinline__ void nl_walk(int64_t i, const NlGeom& g, const NlLayout& w, Visit visit) {
  const double pi0 = w.pw[3 * i], pi1 = w.pw[3 * i + 1], pi2 = w.pw[3 * i + 2];
  const int id = w.bid[i];
  const int b0 = id / (g.nb[1] * g.nb[2]), b1 = (id / g.nb[2]) % g.nb[1], b2 = id % g.nb[2];
  for (int dx = -1; dx <= 1; ++dx)
    for (int dy = -1; dy <= 1; ++dy)
      for (int dz = -1; dz <= 1; ++dz) {
        int c[3] = {b0 + dx, b1 + dy, b2 + dz};
        int img[3];
        for (int k = 0; k < 3; ++k) {
          img[k] = c[k] < 0 ? -1 : (c[k] >= g.nb[k] ? 1 : 0);
          c[k] -= img[k] * g.nb[k];
        }
        const int other = (c[0] * g.nb[1] + c[1]) * g.nb[2] + c[2];
        const double o0 = img[0] ? (img[0] > 0 ? g.L[0] : -g.L[0]) : 0.0;
        const double o1 = img[1] ? (img[1] > 0 ? g.L[1] : -g.L[1]) : 0.0;
        const double o2 = img[2] ? (img[2] > 0 ? g.L[2] : -g.L[2]) : 0.0;
        for (int s = w.start[other]; s < w.start[other + 1]; ++s) {
          const int j = w.sorted[s];
          if (j == i && img[0] == 0 && img[1] == 0 && img[2] == 0) continue;
          const double v0 = __dsub_rn(__dadd_rn(w.pw[3 * j], o0), pi0);
          const double v1 = __dsub_rn(__dadd_rn(w.pw[3 * j + 1], o1), pi1);
          const double v2 = __dsub_rn(__dadd_rn(w.pw[3 * j + 2], o2), pi2);
          const double d2 = __dadd_rn(__dadd_rn(__dmul_rn(v0, v0), __dmul_rn(v1, v1)), __dmul_rn(v2, v2));
          if (d2 < g.r2) visit(j, img);
        }
      }
}

__global__ void nl_count_kernel(int64_t n, NlGeom g, NlLayout w, int64_t* __restrict__ counts) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t c = 0;
    nl_walk(i, g, w, [&](int, const int*) { ++c; });
    counts[i] = c;
  }
}

__global__ void nl_fill_kernel(int64_t n, NlGeom g, NlLayout w, const int64_t* __restrict__ rowptr, int64_t n_edges,
                               int64_t* __restrict__ ei, int32_t* __restrict__ shifts, int* status) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = rowptr[i], e1 = rowptr[i + 1];
    if (e0 < 0 || e1 > n_edges || e1 < e0) {
      fc_flag(status, FC_DEV_BAD_INDEX);
      continue;
    }
    int64_t e = e0;
    const int wi0 = w.wrap[3 * i], wi1 = w.wrap[3 * i + 1], wi2 = w.wrap[3 * i + 2];
    nl_walk(i, g, w, [&](int j, const int* img) {
      if (e >= e1) {
        fc_flag(status, FC_DEV_BAD_INDEX);  // more pairs than the count pass found
        return;
      }
      ei[e] = i;
      ei[n_edges + e] = j;
      shifts[3 * e] = img[0] - w.wrap[3 * j] + wi0;
      shifts[3 * e + 1] = img[1] - w.wrap[3 * j + 1] + wi1;
      shifts[3 * e + 2] = img[2] - w.wrap[3 * j + 2] + wi2;
      ++e;
    });
    // canonical order within the receiver: (j, S0, S1, S2) ascending (insertion sort)
    for (int64_t a = e0 + 1; a < e; ++a) {
      const int ja = (int)ei[n_edges + a];
      const int sa[3] = {shifts[3 * a], shifts[3 * a + 1], shifts[3 * a + 2]};
      int64_t b = a - 1;
      while (b >= e0) {
        const int sb[3] = {shifts[3 * b], shifts[3 * b + 1], shifts[3 * b + 2]};
        if (!nl_less(ja, sa, (int)ei[n_edges + b], sb)) break;
        ei[n_edges + b + 1] = ei[n_edges + b];
        shifts[3 * (b + 1)] = sb[0];
        shifts[3 * (b + 1) + 1] = sb[1];
        shifts[3 * (b + 1) + 2] = sb[2];
        --b;
      }
      ei[n_edges + b + 1] = ja;
      shifts[3 * (b + 1)] = sa[0];
      shifts[3 * (b + 1) + 1] = sa[1];
      shifts[3 * (b + 1) + 2] = sa[2];
    }
  }
}

static NlGeom nl_geom(const fc_nl_desc* d) {
  NlGeom g;
  for (int k = 0; k < 3; ++k) {
    g.L[k] = d->lengths[k];
    g.inv_L[k] = d->inv_lengths[k];
    g.width[k] = d->bin_widths[k];
    g.nb[k] = d->bins[k];
  }
  g.r2 = d->r_max_sq;
  return g;
}

static int nl_grid(int64_t n) {
  const int64_t b = (n + 127) / 128;
  return (int)(b < 1 ? 1 : (b > 148 * 32 ? 148 * 32 : b));
}

int nl_count(const fc_nl_desc* d, const double* pos, int64_t n, void* ws, int64_t* rowptr, int* status,
             cudaStream_t s) {
  const int64_t nbins = (int64_t)d->bins[0] * d->bins[1] * d->bins[2];
  NlLayout w = nl_layout(ws, n, nbins);
  const NlGeom g = nl_geom(d);
  if (cudaMemsetAsync(w.start, 0, sizeof(int32_t) * (nbins + 1), s) != cudaSuccess ||
      cudaMemsetAsync(w.fill, 0, sizeof(int32_t) * nbins, s) != cudaSuccess)
    return FC_ERR_LAUNCH;
  nl_prepare_kernel<<<nl_grid(n), 128, 0, s>>>(pos, n, g, w, status);
  nl_scan_kernel<int32_t><<<1, 1024, 0, s>>>(w.start, nbins);
  nl_scatter_kernel<<<nl_grid(n), 128, 0, s>>>(n, w);
  nl_count_kernel<<<nl_grid(n), 128, 0, s>>>(n, g, w, rowptr);
  nl_scan_kernel<int64_t><<<1, 1024, 0, s>>>(rowptr, n);
  return fc_check_launch();
}

int nl_fill(const fc_nl_desc* d, int64_t n, const void* ws, const int64_t* rowptr, int64_t n_edges,
            int64_t* edge_index, int32_t* shifts, int* status, cudaStream_t s) {
  const int64_t nbins = (int64_t)d->bins[0] * d->bins[1] * d->bins[2];
  NlLayout w = nl_layout(const_cast<void*>(ws), n, nbins);
  nl_fill_kernel<<<nl_grid(n), 128, 0, s>>>(n, nl_geom(d), w, rowptr, n_edges, edge_index, shifts, status);
  return fc_check_launch();
}

#endif  // FC_HOST_EMU

}  // namespace fc
