"""Channel-pair kernels for the dense node-level products (float32).

Emitted into each signature file next to the generic bodies of
:mod:`flashcart_b200.codegen.emit`, for the case of the product layers
(``nn/layers.py:768-1018`` of the reference: ``TensorProduct`` of two node-feature
tensors): no edges (``rowptr == NULL``, output row = in1 row = in2 row), both inputs with
the same ``F`` channels (64 or 128), paths not reduced, weights per row or shared by all
rows (the element-agnostic products; their backward takes this kernel only when no
weight gradient is requested, since a shared weight gradient is a reduction over rows).

Each thread owns two adjacent channels ``2t, 2t+1`` of one row (``F/2`` threads per
row, several rows per 128-thread CTA). Loads and stores are 8-byte ``float2`` vectors and
the arithmetic runs as packed ``f32x2`` multiply-adds (``__ffma2_rn``), half the issue
slots of the one-channel-per-thread bodies (measured on the product layers' shapes,
27,648 rows, C = 128: forward (3,3)->3 0.40 -> 0.33 ms, (3,3)->0 0.12 -> 0.09 ms; backward
(3,3)->3 0.70 -> 0.69 ms, (3,3)->0 0.26 -> 0.17 ms). With no edge loop there is nothing to
accumulate across edges: the forward stores each output component as soon as its path
is done, and the backward loads the output gradient of a path when the path needs it,
so the register footprint is the inputs plus (backward) their gradients.

The arithmetic of a path is the one the generic bodies use (the same exact tensors of
:mod:`flashcart_b200.codegen.stf`); only the grouping of the float32 sums differs.
"""

from __future__ import annotations

from typing import List, Sequence, Tuple

from flashcart_b200.codegen import stf
from flashcart_b200.codegen.emit_pair import _chain, _lin_pairs

BLOCK = 128
# CTAs per SM the backward's register allocation must allow. The backward holds the inputs
# and their gradients (4 x D float2 values per thread); uncapped it takes 254 registers (2
# CTAs per SM). Measured on the (3,3)->3 product at 27,648 rows, C = 128: 0.87 ms at 2
# CTAs, 0.69 ms at 3 (168 registers), 0.74 ms at 4 (128 registers, more local spills);
# the one-channel-per-thread body took 0.70 ms. Issuing each path's weight and gradient
# loads one path ahead of their use made the backward slower (0.53 -> 0.59 ms with shared
# weights): the extra live registers cost more than the hidden latency.
BWD_MIN_CTAS = 3


def _q(r: int, i: int) -> int:
    return r * r + i


def _m_expr(K, a: int, i: int, r2: int) -> str:
    """sum_j K[a][i][j] x2[j] of the path as a packed expression ("" when zero)."""
    e = _lin_pairs([(K[a][i][j], f"x2[{_q(r2, j)}]") for j in range(2 * r2 + 1)])
    return "" if e == "p2(0.0f)" else e


def _n_expr(K, a: int, j: int, r1: int) -> str:
    """sum_i K[a][i][j] x1[i] of the path as a packed expression ("" when zero)."""
    e = _lin_pairs([(K[a][i][j], f"x1[{_q(r1, i)}]") for i in range(2 * r1 + 1)])
    return "" if e == "p2(0.0f)" else e


def emit(sig, store_offsets: List[Tuple[int, int]]) -> str:
    L: List[str] = []
    w = L.append
    w("// ---- dense channel-pair products (float32): F/2 threads per row, two channels per thread")
    w("#ifndef FC_DP_BWD_MIN_CTAS")
    w(f"#define FC_DP_BWD_MIN_CTAS {BWD_MIN_CTAS}")
    w("#endif")
    # ---------------- forward
    w(f"__global__ void __launch_bounds__({BLOCK}) dpfwd_kernel(TpParams<float> P) {{")
    w("  const int F = P.F, tpr = F >> 1;")
    w(f"  const int64_t row = (int64_t)blockIdx.x * ({BLOCK} / tpr) + threadIdx.x / tpr;")
    w("  if (row >= P.n_rows) return;")
    w("  const int c = 2 * (int)(threadIdx.x % tpr);")
    w("  const float* __restrict__ a1 = P.in1 + row * (int64_t)(D1 * F) + c;")
    w("  const float* __restrict__ a2 = P.in2 + row * (int64_t)(D2 * F) + c;")
    w("  const float* __restrict__ wr = P.w + (P.shared_w ? 0 : row * (int64_t)(NP * F)) + c;")
    w("  float* __restrict__ o = P.out + row * (int64_t)(OUT_COMPS * F) + c;")
    w("  float2 x1[D1], x2[D2];")
    w("#pragma unroll")
    w("  for (int q = 0; q < D1; ++q) x1[q] = ldg2(a1 + q * F);")
    w("#pragma unroll")
    w("  for (int q = 0; q < D2; ++q) x2[q] = ldg2(a2 + q * F);")
    for p, (r1, r2, o) in enumerate(sig.paths):
        K = stf.oriented_path_tensor(r1, r2, o)
        w(f"  {{ // path {p}: ({r1},{r2})->{o}")
        w(f"    const float2 wp = ldg2(wr + {p} * F);")
        for a in range(2 * o + 1):
            pairs = []
            for i in range(2 * r1 + 1):
                m = _m_expr(K, a, i, r2)
                if m:
                    pairs.append((f"x1[{_q(r1, i)}]", m))
            k = sig.base[p] + a
            t = _chain(pairs)
            w(f"    st2(o + {store_offsets[k][0]} * F, pmul(wp, {t}));")
        w("  }")
    w("}")
    # ---------------- backward
    w(f"__global__ void __launch_bounds__({BLOCK}, FC_DP_BWD_MIN_CTAS) dpbwd_kernel(TpBwdParams<float> P) {{")
    w("  const int F = P.F, tpr = F >> 1;")
    w(f"  const int64_t row = (int64_t)blockIdx.x * ({BLOCK} / tpr) + threadIdx.x / tpr;")
    w("  if (row >= P.n_rows) return;")
    w("  const bool NEED_1 = P.g_in1 != nullptr, NEED_2 = P.g_in2 != nullptr, NEED_W = P.g_w != nullptr;")
    w("  const int c = 2 * (int)(threadIdx.x % tpr);")
    w("  const float* __restrict__ a1 = P.in1 + row * (int64_t)(D1 * F) + c;")
    w("  const float* __restrict__ a2 = P.in2 + row * (int64_t)(D2 * F) + c;")
    w("  const float* __restrict__ wr = P.w + (P.shared_w ? 0 : row * (int64_t)(NP * F)) + c;")
    w("  const float* __restrict__ go = P.g_out + row * (int64_t)(OUT_COMPS * F) + c;")
    w("  float* __restrict__ gwr = NEED_W ? P.g_w + row * (int64_t)(NP * F) + c : nullptr;")
    w("  float2 x1[D1], x2[D2], gx1[D1], gx2[D2];")
    w("#pragma unroll")
    w("  for (int q = 0; q < D1; ++q) { x1[q] = ldg2(a1 + q * F); gx1[q] = p2(0.0f); }")
    w("#pragma unroll")
    w("  for (int q = 0; q < D2; ++q) { x2[q] = ldg2(a2 + q * F); gx2[q] = p2(0.0f); }")
    for p, (r1, r2, o) in enumerate(sig.paths):
        K = stf.oriented_path_tensor(r1, r2, o)
        w(f"  {{ // path {p}: ({r1},{r2})->{o}")
        w(f"    const float2 wp = ldg2(wr + {p} * F);")
        for a in range(2 * o + 1):
            k = sig.base[p] + a
            w(f"    const float2 g{a} = ldg2(go + {store_offsets[k][0]} * F);")
        hs = []
        for i in range(2 * r1 + 1):
            pairs = []
            for a in range(2 * o + 1):
                m = _m_expr(K, a, i, r2)
                if m:
                    pairs.append((f"g{a}", m))
            if pairs:
                w(f"    const float2 h{i} = {_chain(pairs)};")
                hs.append(i)
        if hs:
            gw = _chain([(f"x1[{_q(r1, i)}]", f"h{i}") for i in hs])
            w(f"    if (NEED_W) st2(gwr + {p} * F, {gw});")
            w("    if (NEED_1) {")
            for i in hs:
                q = _q(r1, i)
                w(f"      gx1[{q}] = pfma(wp, h{i}, gx1[{q}]);")
            w("    }")
        else:
            w(f"    if (NEED_W) st2(gwr + {p} * F, p2(0.0f));")
        body2 = []
        for j in range(2 * r2 + 1):
            pairs = []
            for a in range(2 * o + 1):
                n = _n_expr(K, a, j, r1)
                if n:
                    pairs.append((f"g{a}", n))
            if pairs:
                q = _q(r2, j)
                body2.append(f"      gx2[{q}] = pfma(wp, {_chain(pairs)}, gx2[{q}]);")
        if body2:
            w("    if (NEED_2) {")
            L.extend(body2)
            w("    }")
        w("  }")
    w("  if (NEED_1) {")
    w("    float* t1 = P.g_in1 + row * (int64_t)(D1 * F) + c;")
    w("    if (P.r_in1) {  // residual of the leading components (plain loads: it may alias an output)")
    w("      const float* r1 = P.r_in1 + row * P.r1_ld + c;")
    w("#pragma unroll")
    w("      for (int q = 0; q < D1; ++q)")
    w("        if (q < P.r1_comps) gx1[q] = padd(gx1[q], ld2(r1 + q * F));")
    w("    }")
    w("#pragma unroll")
    w("    for (int q = 0; q < D1; ++q) st2(t1 + q * F, gx1[q]);")
    w("  }")
    w("  if (NEED_2) {")
    w("    float* t2 = P.g_in2 + row * (int64_t)(D2 * F) + c;")
    w("    if (P.r_in2) {")
    w("      const float* r2 = P.r_in2 + row * (int64_t)(D2 * F) + c;")
    w("#pragma unroll")
    w("      for (int q = 0; q < D2; ++q) gx2[q] = padd(gx2[q], ld2(r2 + q * F));")
    w("    }")
    w("#pragma unroll")
    w("    for (int q = 0; q < D2; ++q) st2(t2 + q * F, gx2[q]);")
    w("  }")
    w("}")
    # ---------------- launchers
    for kind, params in (("fwd", "TpParams"), ("bwd", "TpBwdParams")):
        w(f"inline int launch_dp{kind}(const {params}<float>& P, cudaStream_t s) {{")
        w("  if (P.n_rows == 0) return 0;")
        w("  if (P.F != 64 && P.F != 128) return FC_ERR_UNSUPPORTED;")
        w(f"  const int64_t rows_per_cta = {BLOCK} / (P.F >> 1);")
        w("  const int64_t grid = (P.n_rows + rows_per_cta - 1) / rows_per_cta;")
        w("  if (grid > 0x7fffffffLL) return FC_ERR_UNSUPPORTED;")
        w(f"  dp{kind}_kernel<<<(unsigned)grid, {BLOCK}, 0, s>>>(P);")
        w("  return fc_check_launch();")
        w("}")
    return "\n".join(L) + "\n"
