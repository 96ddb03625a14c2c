// Fused edge geometry of the potential: one pass per edge from positions to the edge
// attributes and the radial features, and its first derivative back to positions and
// cells.
//
// Forward, per edge e = (i receiver, j sender, image shift s):
//   v  = r_j - r_i + s . cell[batch[i]]                        (utils/geometry.py:25-53)
//   r  = |v|,  d = v / max(r, 1e-4)                             (model/flashcart.py:280-284)
//   attrs[e] = T^l(d), l <= l_max, stored STF components        (o3/irreps.py:54-72)
//   radial[e, n] = cheb_n(x) * env(r)                           (nn/radial.py:98-128, 181-245;
//        x = cos(pi t) or 2t - 1, t = (r - r_min) / (r_max - r_min);  the product is the
//        radial-MLP input of InteractionLayer.forward, nn/layers.py:351-356)
//   env(r) = clamp(mask(r < r_cut) * (1 - c1 u^p + c2 u^(p+1) - c3 u^(p+2)), 0, 1), u = r / r_cut
// Backward: the vector-Jacobian product of the same chain (direction normalisation with
// the clamp of torch.clamp_min, Chebyshev derivative by its recurrence, envelope
// derivative, norm), scattered as +g_v into the sender's and -g_v into the receiver's
// position gradient and s (x) g_v into the receiving graph's cell gradient (atomics; runs
// of equal receivers within a warp, and a warp whose edges share one graph, reduce first).
//
// One thread per edge, grid-stride; an index outside [0, n_nodes) flags FC_DEV_BAD_INDEX
// and the edge gives zeros (forward) / no gradient (backward).
//
// Vectors-given mode (fc_edge_geometry_vec_fwd/bwd): the caller supplies v per edge (the
// LAMMPS ML-IAP rij, calculators/lammps_mliap.py:122-170) and the backward writes dE/dv
// per edge, the pair forces that ML-IAP takes (lammps_mliap.py:711-738), with plain
// stores instead of the receiver / sender scatter.
#include "fc_base.cuh"
#include "gen/irreps_poly.cuh"

namespace fc {

template <typename T, int L>
FC_HD FC_INLINE void geom_attrs(T dx, T dy, T dz, T* o) {
  if constexpr (L == 0) irreps_fwd_l0<T>(dx, dy, dz, o);
  else if constexpr (L == 1) irreps_fwd_l1<T>(dx, dy, dz, o);
  else if constexpr (L == 2) irreps_fwd_l2<T>(dx, dy, dz, o);
  else irreps_fwd_l3<T>(dx, dy, dz, o);
}
template <typename T, int L>
FC_HD FC_INLINE void geom_attrs_vjp(T dx, T dy, T dz, const T* g, T* gd) {
  if constexpr (L == 0) irreps_bwd_l0<T>(dx, dy, dz, g, gd);
  else if constexpr (L == 1) irreps_bwd_l1<T>(dx, dy, dz, g, gd);
  else if constexpr (L == 2) irreps_bwd_l2<T>(dx, dy, dz, g, gd);
  else irreps_bwd_l3<T>(dx, dy, dz, g, gd);
}

FC_HD FC_INLINE float fc_cos(float x) { return cosf(x); }
FC_HD FC_INLINE double fc_cos(double x) { return cos(x); }
FC_HD FC_INLINE float fc_sin(float x) { return sinf(x); }
FC_HD FC_INLINE double fc_sin(double x) { return sin(x); }
FC_HD FC_INLINE float fc_sqrt(float x) { return sqrtf(x); }
FC_HD FC_INLINE double fc_sqrt(double x) { return sqrt(x); }

// Edge vector of edge e; false (and zeros) when an index is out of range.
template <typename T>
FC_HD FC_INLINE bool geom_vector(const GeomParams& p, const T* pos, const T* cells, const int32_t* shifts,
                                 const int64_t* ei, const int64_t* batch, int64_t e, T* v, int64_t* ij_b) {
  if (p.vectors_given) {  // v supplied per edge (LAMMPS rij): no atoms, shifts or cells
    for (int c = 0; c < 3; ++c) v[c] = pos[3 * e + c];
    ij_b[0] = ij_b[1] = e; ij_b[2] = 0;
    return true;
  }
  const int64_t i = ei[e], j = ei[p.n_edges + e];
  if (i < 0 || i >= p.n_nodes || j < 0 || j >= p.n_nodes) {
    v[0] = v[1] = v[2] = T(0);
    return false;
  }
  int64_t b = 0;
  if (p.use_shifts && p.n_cells > 1) {
    b = batch[i];
    if (b < 0 || b >= p.n_cells) {
      v[0] = v[1] = v[2] = T(0);
      return false;
    }
  }
  ij_b[0] = i; ij_b[1] = j; ij_b[2] = b;
  for (int c = 0; c < 3; ++c) v[c] = pos[3 * j + c] - pos[3 * i + c];
  if (p.use_shifts) {
    const T s0 = T(shifts[3 * e]), s1 = T(shifts[3 * e + 1]), s2 = T(shifts[3 * e + 2]);
    const T* cl = cells + 9 * b;
    for (int c = 0; c < 3; ++c) v[c] = v[c] + (s0 * cl[c] + s1 * cl[3 + c] + s2 * cl[6 + c]);
  }
  return true;
}

// Envelope and its derivative with respect to r (torch.clamp passes the gradient on the
// closed interval [0, 1]).
template <typename T>
FC_HD FC_INLINE void geom_envelope(const GeomParams& p, T r, T* env, T* denv) {
  const T rc = T(p.r_cut);
  const int po = p.poly_order;
  const T c1 = T((po + 1.0) * (po + 2.0) / 2.0), c2 = T(po * (po + 2.0)), c3 = T(po * (po + 1.0) / 2.0);
  const T d = r < T(0) ? T(0) : r;
  const T u = d / rc;
  T tpm1 = T(1);
  for (int k = 0; k < po - 1; ++k) tpm1 = tpm1 * u;
  const T tp = tpm1 * u, tp1 = tp * u, tp2 = tp1 * u;
  const T e = T(1) - c1 * tp + c2 * tp1 - c3 * tp2;
  const T mask = d < rc ? T(1) : T(0);
  const T em = e * mask;
  *env = em < T(0) ? T(0) : (em > T(1) ? T(1) : em);
  const T de = (-c1 * T(po) * tpm1 + c2 * T(po + 1) * tp - c3 * T(po + 2) * tp1) / rc;
  *denv = (em >= T(0) && em <= T(1)) ? mask * de : T(0);
}

template <typename T, int L>
FC_HD FC_INLINE void geom_fwd_one(const GeomParams& p, const T* pos, const T* cells, const int32_t* shifts,
                                  const int64_t* ei, const int64_t* batch, T* attrs, T* radial, int* status,
                                  int64_t e) {
  constexpr int D = (L + 1) * (L + 1);
  T v[3];
  int64_t ijb[3];
  const bool ok = geom_vector<T>(p, pos, cells, shifts, ei, batch, e, v, ijb);
  if (!ok) {
    fc_flag(status, FC_DEV_BAD_INDEX);
    for (int k = 0; k < D; ++k) attrs[e * D + k] = T(0);
    for (int n = 0; n < p.n_radial; ++n) radial[e * p.n_radial + n] = T(0);
    return;
  }
  const T r = fc_sqrt(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
  const T c = r < T(1.0e-4) ? T(1.0e-4) : r;
  T o[D];
  geom_attrs<T, L>(v[0] / c, v[1] / c, v[2] / c, o);
  for (int k = 0; k < D; ++k) attrs[e * D + k] = o[k];
  T env, denv;
  geom_envelope<T>(p, r, &env, &denv);
  const T t = (r - T(p.r_min)) / (T(p.r_max) - T(p.r_min));
  const T x = p.cosine ? fc_cos(t * T(3.14159265358979323846)) : T(2) * t - T(1);
  T* out = radial + e * p.n_radial;
  T tm2 = T(1), tm1 = x;
  out[0] = tm2 * env;
  if (p.n_radial > 1) out[1] = tm1 * env;
  for (int n = 2; n < p.n_radial; ++n) {
    const T tn = T(2) * x * tm1 - tm2;
    out[n] = tn * env;
    tm2 = tm1;
    tm1 = tn;
  }
}

// g_v of edge e (and its indices); false for a skipped edge.
template <typename T, int L>
FC_HD FC_INLINE bool geom_bwd_one(const GeomParams& p, const T* pos, const T* cells, const int32_t* shifts,
                                  const int64_t* ei, const int64_t* batch, const T* g_attrs, const T* g_radial,
                                  int* status, int64_t e, T* gv, int64_t* ijb) {
  constexpr int D = (L + 1) * (L + 1);
  T v[3];
  if (!geom_vector<T>(p, pos, cells, shifts, ei, batch, e, v, ijb)) {
    fc_flag(status, FC_DEV_BAD_INDEX);
    return false;
  }
  const T r = fc_sqrt(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
  const bool clamped = r < T(1.0e-4);
  const T c = clamped ? T(1.0e-4) : r;
  const T d0 = v[0] / c, d1 = v[1] / c, d2 = v[2] / c;
  T gd[3] = {T(0), T(0), T(0)};
  if (g_attrs) {
    T ga[D];
    for (int k = 0; k < D; ++k) ga[k] = g_attrs[e * D + k];
    geom_attrs_vjp<T, L>(d0, d1, d2, ga, gd);
  }
  // radial features: g_r = sum_n g_n (cheb_n' x' env + cheb_n env')
  T g_r = T(0);
  if (g_radial) {
    T env, denv;
    geom_envelope<T>(p, r, &env, &denv);
    const T span = T(p.r_max) - T(p.r_min);
    const T t = (r - T(p.r_min)) / span;
    const T pi = T(3.14159265358979323846);
    const T x = p.cosine ? fc_cos(t * pi) : T(2) * t - T(1);
    const T dx = p.cosine ? -pi * fc_sin(t * pi) / span : T(2) / span;
    const T* gr = g_radial + e * p.n_radial;
    T tm2 = T(1), tm1 = x, dm2 = T(0), dm1 = T(1);
    T s_val = gr[0] * tm2, s_der = T(0);
    if (p.n_radial > 1) {
      s_val += gr[1] * tm1;
      s_der += gr[1] * dm1;
    }
    for (int n = 2; n < p.n_radial; ++n) {
      const T tn = T(2) * x * tm1 - tm2;
      const T dn = T(2) * tm1 + T(2) * x * dm1 - dm2;
      s_val += gr[n] * tn;
      s_der += gr[n] * dn;
      tm2 = tm1; tm1 = tn;
      dm2 = dm1; dm1 = dn;
    }
    g_r = s_der * dx * env + s_val * denv;
  }
  // direction d = v / max(r, eps): dd/dv = I / c, dd/dr = -v / c^2 where r >= eps
  if (!clamped) g_r -= (gd[0] * v[0] + gd[1] * v[1] + gd[2] * v[2]) / (c * c);
  const T inv_r = r > T(0) ? T(1) / r : T(0);
  for (int k = 0; k < 3; ++k) gv[k] = gd[k] / c + g_r * v[k] * inv_r;
  return true;
}

#ifndef FC_HOST_EMU
template <typename T, int L>
__global__ void __launch_bounds__(256) geom_fwd_kernel(GeomParams p, const T* pos, const T* cells,
                                                       const int32_t* shifts, const int64_t* ei, const int64_t* batch,
                                                       T* attrs, T* radial, int* status) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < p.n_edges; e += (int64_t)gridDim.x * blockDim.x)
    geom_fwd_one<T, L>(p, pos, cells, shifts, ei, batch, attrs, radial, status, e);
}

template <typename T, int L>
__global__ void __launch_bounds__(256) geom_bwd_kernel(GeomParams p, const T* pos, const T* cells,
                                                       const int32_t* shifts, const int64_t* ei, const int64_t* batch,
                                                       const T* g_attrs, const T* g_radial, T* g_pos, T* g_cells,
                                                       int* status) {
  if (p.vectors_given) {  // gradient per edge vector: one plain store per edge, no scatter
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < p.n_edges;
         e += (int64_t)gridDim.x * blockDim.x) {
      T gv[3] = {T(0), T(0), T(0)};
      int64_t ijb[3];
      geom_bwd_one<T, L>(p, pos, cells, shifts, ei, batch, g_attrs, g_radial, status, e, gv, ijb);
      for (int k = 0; k < 3; ++k) g_pos[3 * e + k] = gv[k];
    }
    return;
  }
  const int lane = threadIdx.x & 31;
  // one cell: every edge adds into the same nine cell-gradient values, so each thread
  // keeps its sum in registers and the CTA reduces once at the end (per-warp atomics on
  // the same nine addresses serialise in L2)
  const bool one_cell = g_cells != nullptr && p.use_shifts && p.n_cells == 1;
  T gc_own[9];
  for (int k = 0; k < 9; ++k) gc_own[k] = T(0);
  for (int64_t base = blockIdx.x * (int64_t)blockDim.x; base < p.n_edges; base += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = base + threadIdx.x;
    T gv[3] = {T(0), T(0), T(0)};
    int64_t ijb[3] = {0, 0, -1};
    bool ok = false;
    if (e < p.n_edges) ok = geom_bwd_one<T, L>(p, pos, cells, shifts, ei, batch, g_attrs, g_radial, status, e, gv, ijb);
    if (ok)
      for (int k = 0; k < 3; ++k) atomicAdd(g_pos + 3 * ijb[1] + k, gv[k]);
    // receiver side: edges normally come sorted by receiver, so the lanes of a warp share
    // few receivers. A segmented suffix sum over runs of consecutive lanes with equal
    // receivers leaves each run's total in its first lane, which issues the run's three
    // atomics (a receiver that reappears after another one starts a new run).
    {
      const long long key = ok ? (long long)ijb[0] : -1 - (long long)lane;
      const long long prev = __shfl_up_sync(0xffffffffu, key, 1);
      const bool head = lane == 0 || prev != key;
      const unsigned heads = __ballot_sync(0xffffffffu, head);
      const unsigned later = lane == 31 ? 0u : heads & ~((2u << lane) - 1u);
      const int run_end = later ? __ffs(later) - 1 : 32;  // first lane of the next run
      T acc[3] = {ok ? -gv[0] : T(0), ok ? -gv[1] : T(0), ok ? -gv[2] : T(0)};
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        T y[3];
        for (int k = 0; k < 3; ++k) y[k] = __shfl_down_sync(0xffffffffu, acc[k], off);
        if (lane + off < run_end)
          for (int k = 0; k < 3; ++k) acc[k] += y[k];
      }
      if (ok && head)
        for (int k = 0; k < 3; ++k) atomicAdd(g_pos + 3 * key + k, acc[k]);
    }
    if (one_cell) {
      if (ok)
        for (int a = 0; a < 3; ++a)
          for (int c = 0; c < 3; ++c) gc_own[3 * a + c] += T(shifts[3 * e + a]) * gv[c];
    } else if (g_cells && p.use_shifts) {
      // s (x) g_v into the receiving graph's cell gradient; one graph per warp -> warp sum
      T gc[9];
      T s[3] = {T(0), T(0), T(0)};
      if (ok)
        for (int a = 0; a < 3; ++a) s[a] = T(shifts[3 * e + a]);
      for (int a = 0; a < 3; ++a)
        for (int c = 0; c < 3; ++c) gc[3 * a + c] = s[a] * gv[c];
      const long long b = ok ? (long long)ijb[2] : -1;
      const long long b0 = __shfl_sync(0xffffffffu, b, 0);
      const bool uniform = __all_sync(0xffffffffu, b == b0 || b < 0);
      if (uniform) {
        for (int k = 0; k < 9; ++k) gc[k] = fc_warp_sum(gc[k]);
        if (lane == 0 && b0 >= 0)
          for (int k = 0; k < 9; ++k) atomicAdd(g_cells + 9 * b0 + k, gc[k]);
        if (b0 < 0) {  // lane 0's edge was skipped: take the warp's graph from a valid lane
          const unsigned any = __ballot_sync(0xffffffffu, b >= 0);
          if (any) {
            const int src = __ffs(any) - 1;
            const long long bb = __shfl_sync(0xffffffffu, b, src);
            if (lane == 0)
              for (int k = 0; k < 9; ++k) atomicAdd(g_cells + 9 * bb + k, gc[k]);
          }
        }
      } else if (b >= 0) {
        for (int k = 0; k < 9; ++k) atomicAdd(g_cells + 9 * b + k, gc[k]);
      }
    }
  }
  if (one_cell) {
    __shared__ T red[9][8];  // blockDim <= 256: 8 warps
    for (int k = 0; k < 9; ++k) {
      const T v = fc_warp_sum(gc_own[k]);
      if (lane == 0) red[k][threadIdx.x >> 5] = v;
    }
    __syncthreads();
    if (threadIdx.x < 9) {
      T v = T(0);
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += red[threadIdx.x][w];
      atomicAdd(g_cells + threadIdx.x, v);
    }
  }
}

static unsigned geom_grid(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return (unsigned)(b < 148 * 32 ? (b < 1 ? 1 : b) : 148 * 32);
}
#endif

template <typename T, int L>
int geom_fwd_l(const GeomParams& p, const T* pos, const T* cells, const int32_t* shifts, const int64_t* ei,
               const int64_t* batch, T* attrs, T* radial, int* status, cudaStream_t s) {
#ifndef FC_HOST_EMU
  geom_fwd_kernel<T, L><<<geom_grid(p.n_edges), 256, 0, s>>>(p, pos, cells, shifts, ei, batch, attrs, radial, status);
  return fc_check_launch();
#else
  (void)s;
  for (int64_t e = 0; e < p.n_edges; ++e) geom_fwd_one<T, L>(p, pos, cells, shifts, ei, batch, attrs, radial, status, e);
  return 0;
#endif
}

template <typename T, int L>
int geom_bwd_l(const GeomParams& p, const T* pos, const T* cells, const int32_t* shifts, const int64_t* ei,
               const int64_t* batch, const T* g_attrs, const T* g_radial, T* g_pos, T* g_cells, int* status,
               cudaStream_t s) {
#ifndef FC_HOST_EMU
  const int64_t want = (p.n_edges + 255) / 256;
  const unsigned grid = (unsigned)(want < 148 * 8 ? (want < 1 ? 1 : want) : 148 * 8);
  geom_bwd_kernel<T, L><<<grid, 256, 0, s>>>(p, pos, cells, shifts, ei, batch, g_attrs, g_radial, g_pos, g_cells,
                                             status);
  return fc_check_launch();
#else
  (void)s;
  for (int64_t e = 0; e < p.n_edges; ++e) {
    T gv[3];
    int64_t ijb[3];
    if (!geom_bwd_one<T, L>(p, pos, cells, shifts, ei, batch, g_attrs, g_radial, status, e, gv, ijb)) continue;
    if (p.vectors_given) {
      for (int k = 0; k < 3; ++k) g_pos[3 * e + k] = gv[k];
      continue;
    }
    for (int k = 0; k < 3; ++k) {
      g_pos[3 * ijb[1] + k] += gv[k];
      g_pos[3 * ijb[0] + k] -= gv[k];
    }
    if (g_cells && p.use_shifts)
      for (int a = 0; a < 3; ++a)
        for (int c = 0; c < 3; ++c) g_cells[9 * ijb[2] + 3 * a + c] += T(shifts[3 * e + a]) * gv[c];
  }
  return 0;
#endif
}

template <typename T>
int geom_fwd_dispatch(const GeomParams& p, const T* pos, const T* cells, const int32_t* shifts, const int64_t* ei,
                      const int64_t* batch, T* attrs, T* radial, int* status, cudaStream_t s) {
  switch (p.l_max) {
    case 0: return geom_fwd_l<T, 0>(p, pos, cells, shifts, ei, batch, attrs, radial, status, s);
    case 1: return geom_fwd_l<T, 1>(p, pos, cells, shifts, ei, batch, attrs, radial, status, s);
    case 2: return geom_fwd_l<T, 2>(p, pos, cells, shifts, ei, batch, attrs, radial, status, s);
    case 3: return geom_fwd_l<T, 3>(p, pos, cells, shifts, ei, batch, attrs, radial, status, s);
  }
  return FC_ERR_UNSUPPORTED;
}

template <typename T>
int geom_bwd_dispatch(const GeomParams& p, const T* pos, const T* cells, const int32_t* shifts, const int64_t* ei,
                      const int64_t* batch, const T* g_attrs, const T* g_radial, T* g_pos, T* g_cells, int* status,
                      cudaStream_t s) {
  switch (p.l_max) {
    case 0: return geom_bwd_l<T, 0>(p, pos, cells, shifts, ei, batch, g_attrs, g_radial, g_pos, g_cells, status, s);
    case 1: return geom_bwd_l<T, 1>(p, pos, cells, shifts, ei, batch, g_attrs, g_radial, g_pos, g_cells, status, s);
    case 2: return geom_bwd_l<T, 2>(p, pos, cells, shifts, ei, batch, g_attrs, g_radial, g_pos, g_cells, status, s);
    case 3: return geom_bwd_l<T, 3>(p, pos, cells, shifts, ei, batch, g_attrs, g_radial, g_pos, g_cells, status, s);
  }
  return FC_ERR_UNSUPPORTED;
}

template int geom_fwd_dispatch<float>(const GeomParams&, const float*, const float*, const int32_t*, const int64_t*,
                                      const int64_t*, float*, float*, int*, cudaStream_t);
template int geom_fwd_dispatch<double>(const GeomParams&, const double*, const double*, const int32_t*,
                                       const int64_t*, const int64_t*, double*, double*, int*, cudaStream_t);
template int geom_bwd_dispatch<float>(const GeomParams&, const float*, const float*, const int32_t*, const int64_t*,
                                      const int64_t*, const float*, const float*, float*, float*, int*, cudaStream_t);
template int geom_bwd_dispatch<double>(const GeomParams&, const double*, const double*, const int32_t*,
                                       const int64_t*, const int64_t*, const double*, const double*, double*, double*,
                                       int*, cudaStream_t);

}  // namespace fc
