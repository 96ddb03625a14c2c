"""Channel-pair convolution kernels (float32) for edge attributes shared by all channels.

Emitted into each signature file next to :mod:`flashcart_b200.codegen.emit_conv` and
used for the same case (the interaction layer's receiver-CSR convolution:
``in2_features == 1``, ``in1_features == F``, per-edge weights, paths not reduced) when
the data are float32 and F is 64 or 128 (F/2 consumer threads: one or two warps).

Why pairs. The per-edge arithmetic of one channel is a few hundred FP32 multiply-adds;
the kernels are bound by instruction issue, not by HBM, and a large share of the issued
instructions is per-edge overhead that does not depend on the channel (edge-matrix
loads, barrier waits, index and address work, the reduction of the in2 gradient over
the channels). Each consumer thread therefore owns two adjacent channels ``2t, 2t+1``:

* the arithmetic of both channels runs as packed ``f32x2`` multiply-adds (one issue slot
  for two FP32 FMAs, ``__ffma2_rn``), so the FMA pipes, not the issue slot, set the pace;
* loads and stores of both channels are 8-byte vectors (``float2``), the in1-gradient
  scatter is one ``red.global.add.v2.f32`` per component;
* the channel-independent per-edge work (edge-matrix reads, the wait on the prefetch
  slot, the sender index, the warp reduction of the in2 gradient) is shared by the two.

CTA = one receiver row. ``F/2`` consumer threads plus one producer warp:

* the producer warp reads the receiver's sender indices 32 at a time (one coalesced
  load), and for each edge waits until its ring slot is free, writes the sender index
  into the slot header and issues 1-D bulk async copies (``cp.async.bulk``, global ->
  this CTA's shared memory, no multicast) of the sender's in1 components of the path
  group and of the edge's path weights; the copies complete on the slot's mbarrier. It
  never waits for the consumers' arithmetic, only for slot releases, so the gathers run
  up to RING edges ahead;
* the consumers walk the edges in chunks of EC: the edge matrices
  ``M_p[a, i] = sum_j K_p[a, i, j] x2_j`` of the chunk are computed cooperatively into
  shared memory (plain floats, each path's entries 16-byte aligned, so that one 16-byte
  broadcast load gives four entries), then per edge every consumer thread waits for the slot, reads the sender
  index from the slot header and does the path-group arithmetic for its two channels.
  Consumers synchronise among themselves with a named barrier; the producer is never
  part of a CTA-wide barrier after the roles split.

Every wait is bounded (FC_DEV_TIMEOUT and a CTA abort flag on expiry); an aborted CTA's
producer waits for its in-flight copies before it exits. Data errors (sender index out
of range) are flagged in the status word and the edge is skipped.
"""

from __future__ import annotations

from fractions import Fraction
from typing import List, Sequence, Tuple

from flashcart_b200.codegen import stf
from flashcart_b200.codegen.emit_conv import GroupSlots, make_groups, _q

NPART = 8     # edge-matrix work split per edge (EC x NPART work items per chunk)
BUDGET = 32   # accumulator pairs per path group when a signature is split
# Per path group: large groups (more than SMALL_NACC accumulator pairs) are limited by how
# many CTAs fit an SM, so they take a small footprint -- chunks of 8 edges, 4 ring slots,
# the backward's output-gradient pairs in shared memory (each thread reads back only its
# own values) and a register cap (P3MinBlocks); small groups keep 16-edge chunks, 6 slots
# and their gradients in registers. Measured on the (3,3)->3 and (0,3)->3 convolutions at
# C = 128, 1.49 M edges: (3,3)->3 backward 21.8 -> 14.0 ms with the small footprint, while
# (0,3)->3 is fastest with the large one (1.38 vs 1.93 ms).
SMALL_NACC = 16
STAGE_X2 = True  # the producer stages each chunk's in2 rows (in2 rows of 4 or 16 floats)
G_SMEM = None  # None: per group as above; True / False force it (experiments)
EC = None
RING = None


def group_cfg(gs) -> dict:
    big = gs.nacc > SMALL_NACC
    return {"big": big,
            "ec": EC if EC is not None else (8 if big else 16),
            "ring": RING if RING is not None else (4 if big else 6),
            "gsmem": G_SMEM if G_SMEM is not None else big}


def _cf(fr: Fraction) -> str:
    return f"p2({float(fr)!r}f)"


def _lin_pairs(terms: Sequence[Tuple[Fraction, str]]) -> str:
    """Packed linear combination sum c_k * v_k of float2 operands (constant coefficients)."""
    terms = [(c, v) for c, v in terms if c != 0]
    if not terms:
        return "p2(0.0f)"
    c0, v0 = terms[0]
    if c0 == 1:
        e = v0
    else:
        e = f"pmul({_cf(c0)}, {v0})"
    for c, v in terms[1:]:
        if c == 1:
            e = f"padd({e}, {v})"
        else:
            e = f"pfma({_cf(c)}, {v}, {e})"
    return e


# Sums of more than CHAIN_SPLIT products split into two independent fma chains. Measured
# on the (3,3)->3 convolution at C = 128: a split at 3 or 5 terms made the backward 1-4%
# slower (13.8 ms unsplit, 14.4 ms at 3), so sums stay single chains.
CHAIN_SPLIT = 99


def _chain1(pairs: Sequence[Tuple[str, str]], init: str = "") -> str:
    e = init
    for a, b in pairs:
        e = f"pmul({a}, {b})" if not e else f"pfma({a}, {b}, {e})"
    return e or "p2(0.0f)"


def _chain(pairs: Sequence[Tuple[str, str]], init: str = "") -> str:
    """sum a_k * b_k (+ init) of float2 operands. A long sum is split into two independent
    fma chains (even / odd terms) joined by one add, so consecutive multiply-adds do not all
    wait for each other (the packed FMA has a multi-cycle latency and few warps per
    scheduler hide it)."""
    pairs = list(pairs)
    if len(pairs) <= CHAIN_SPLIT:
        return _chain1(pairs, init)
    return f"padd({_chain(pairs[0::2], init)}, {_chain(pairs[1::2])})"


# Edge matrices in shared memory as plain floats: each path's entries start on a 16-byte
# boundary, so one 16-byte broadcast load carries four entries and the packed f32x2
# operands are formed in registers. The pair kernels are bound by these shared-memory
# broadcasts; against the earlier layout of duplicated pairs (two entries per 16-byte load),
# measured on the 27,648-atom water box (C = 128): (3,3)->3 forward 5.81 -> 5.13 ms, backward
# 13.72 -> 12.84 ms, (0,3)->3 backward 1.62 -> 1.57 ms, four-channel forward 0.73 -> 0.71 ms.
# The shared-memory carve-up keeps NMP pairs per edge (2 * NMP >= NMF floats).


def scalar_offsets(gs: GroupSlots):
    """Per path: float offset of its first entry (multiple of 4); per edge: total floats."""
    off, pos = {}, 0
    for p in gs.paths:
        s0, s1 = gs.range[p]
        off[p] = pos
        pos += (s1 - s0 + 3) // 4 * 4
    return off, max(pos, 4)


def _phase1(gs: GroupSlots, ind: str) -> List[str]:
    off, _ = scalar_offsets(gs)
    where = {}
    for p in gs.paths:
        s0, s1 = gs.range[p]
        for sl in range(s0, s1):
            where[sl] = off[p] + sl - s0
    L = [f"{ind}switch (part) {{"]
    per = (gs.nm + NPART - 1) // NPART
    for part in range(NPART):
        L.append(f"{ind}  case {part}:")
        for sl in range(part * per, min(gs.nm, (part + 1) * per)):
            if gs.slots[sl] is not None and sl in where:
                L.append(f"{ind}    mf[{where[sl]}] = {gs.m_expr(sl)};")
        L.append(f"{ind}    break;")
    L.append(f"{ind}}}")
    return L


def _path_mload(gs: GroupSlots, p: int, ind: str) -> List[str]:
    """Edge-matrix entries of one path: 16-byte shared loads of four entries each."""
    off, _ = scalar_offsets(gs)
    s0, s1 = gs.range[p]
    n = s1 - s0
    L = [f"{ind}float2 mv[{max(n, 1)}];"]
    for k in range((n + 3) // 4):
        L.append(f"{ind}{{ const float4 q = *reinterpret_cast<const float4*>(mf + {off[p] + 4 * k});")
        for j, comp in enumerate("xyzw"):
            if 4 * k + j < n:
                L.append(f"{ind}  mv[{4 * k + j}] = p2(q.{comp});")
        L.append(f"{ind}}}")
    return L


def _fwd_body(gs: GroupSlots, ind: str) -> List[str]:
    sig = gs.sig
    L = []
    acc_base = 0
    for p in gs.paths:
        r1, r2, o = sig.paths[p]
        s0 = gs.range[p][0]
        L.append(f"{ind}{{ // path {p}: ({r1},{r2})->{o}")
        L.extend(_path_mload(gs, p, ind + "  "))
        L.append(f"{ind}  const float2 wp = ld2(sw + {gs.w_pos[p]} * F);")
        for a in range(2 * o + 1):
            pairs = [(f"mv[{gs.index[(p, a, i)] - s0}]", f"x1[{_q(r1, i) - gs.x_lo}]") for i in range(2 * r1 + 1)
                     if (p, a, i) in gs.index]
            t = _chain(pairs)
            L.append(f"{ind}  acc[{acc_base + a}] = pfma(wp, {t}, acc[{acc_base + a}]);")
        L.append(f"{ind}}}")
        acc_base += 2 * o + 1
    return L


def _bwd_body(gs: GroupSlots, ind: str, d2p: int) -> List[str]:
    """Backward of one edge for the thread's channel pair; the first contribution to a
    gradient register assigns it."""
    sig = gs.sig
    L = []
    base = 0
    set1, set2 = set(), set()

    def acc(name: str, k: int, a: str, b: str, seen: set) -> str:
        if k in seen:
            return f"{name}[{k}] = pfma({a}, {b}, {name}[{k}]);"
        seen.add(k)
        return f"{name}[{k}] = pmul({a}, {b});"

    for p in gs.paths:
        r1, r2, o = sig.paths[p]
        K = stf.oriented_path_tensor(r1, r2, o)
        s0 = gs.range[p][0]
        L.append(f"{ind}{{ // path {p}: ({r1},{r2})->{o}")
        L.extend(_path_mload(gs, p, ind + "  "))
        L.append(f"{ind}  const float2 wp = ld2(sw + {gs.w_pos[p]} * F);")
        if gs.gsmem:
            for a in range(2 * o + 1):
                L.append(f"{ind}  const float2 ga{base + a} = gb[{base + a} * NC + t];")
        gname = (lambda k: f"ga{k}") if gs.gsmem else (lambda k: f"g[{k}]")
        hs = []
        for i in range(2 * r1 + 1):
            pairs = [(gname(base + a), f"mv[{gs.index[(p, a, i)] - s0}]") for a in range(2 * o + 1)
                     if (p, a, i) in gs.index]
            if pairs:
                L.append(f"{ind}  const float2 h{i} = {_chain(pairs)};")
                hs.append(i)
        gw = _chain([(f"x1[{_q(r1, i) - gs.x_lo}]", f"h{i}") for i in hs])
        L.append(f"{ind}  if (NEED_W) st2(gwr + {p} * F, {gw});")
        if hs:
            L.append(f"{ind}  if (NEED_1) {{")
            for i in hs:
                L.append(f"{ind}    " + acc("gx1", _q(r1, i) - gs.x_lo, "wp", f"h{i}", set1))
            L.append(f"{ind}  }}")
        body2 = []
        for j in range(2 * r2 + 1):
            pairs = []
            for a in range(2 * o + 1):
                n = _lin_pairs([(K[a][i][j], f"x1[{_q(r1, i) - gs.x_lo}]") for i in range(2 * r1 + 1)])
                if n != "p2(0.0f)":
                    pairs.append((gname(base + a), n))
            if pairs:
                body2.append(f"{ind}    " + acc("gx2", _q(r2, j), "wp", _chain(pairs), set2))
        if body2:
            L.append(f"{ind}  if (NEED_2) {{")
            L.extend(body2)
            L.append(f"{ind}  }}")
        L.append(f"{ind}}}")
        base += 2 * o + 1
    for q in range(gs.x_n):
        if q not in set1:
            L.append(f"{ind}gx1[{q}] = p2(0.0f);")
    for q in range(d2p):
        if q not in set2:
            L.append(f"{ind}gx2[{q}] = p2(0.0f);")
    return L


def _setup(gs: GroupSlots, extra_floats: str, ind: str, channels_per_thread: int = 2) -> List[str]:
    """Shared-memory carve-up: M pairs | ring slots | [extra] | slot headers | mbarriers."""
    nc_shift = {2: 1, 4: 2}[channels_per_thread]
    return [
        f"{ind}using T = float;",
        f"{ind}constexpr int XLO = {gs.x_lo}, XN = {gs.x_n}, NW = {len(gs.paths)}, NMP = {gs.nmp};",
        f"{ind}const int F = P.F, NC = F >> {nc_shift}, t = threadIdx.x, lane = t & 31;",
        f"{ind}const int64_t row = blockIdx.x;",
        f"{ind}float2* m2 = reinterpret_cast<float2*>(smem);",
        f"{ind}float* ring = reinterpret_cast<float*>(m2 + NMP * {gs.ec});",
        f"{ind}const int SLOT = (XN + NW) * F;",
        f"{ind}float* extra = ring + {gs.ring} * SLOT;",
        f"{ind}float* xbuf = extra + {extra_floats};  // [2][EC][D2] in2 rows of the chunks (staged)",
        f"{ind}int64_t* sj = reinterpret_cast<int64_t*>(xbuf + {2 * gs.ec * gs.sig.d2 if gs.stage else 0});",
        f"{ind}uint64_t* full = reinterpret_cast<uint64_t*>(sj + {gs.ring});",
        f"{ind}uint64_t* empty = full + {gs.ring};",
        f"{ind}uint64_t* xfull = empty + {gs.ring};",
        f"{ind}uint64_t* xempty = xfull + 2;",
        f"{ind}volatile int* abort_flag = reinterpret_cast<volatile int*>(xempty + 2);",
        f"{ind}const int64_t e0 = P.rowptr[row], ne_all = P.rowptr[row + 1] - e0;",
        f"{ind}if (t == 0) {{",
        f"{ind}  for (int s = 0; s < {gs.ring}; ++s) {{ fc_mbar_init(&full[s], 1); fc_mbar_init(&empty[s], NC >> 5); }}",
        f"{ind}  for (int b = 0; b < 2; ++b) {{ fc_mbar_init(&xfull[b], 1); fc_mbar_init(&xempty[b], 1); }}",
        f"{ind}  *abort_flag = 0;",
        f"{ind}  fc_mbar_init_fence();",
        f"{ind}}}",
        f"{ind}__syncthreads();",
    ]


def _producer(gs: GroupSlots, ind: str) -> List[str]:
    """The producer warp: sender indices 32 at a time, then per edge wait for the slot,
    header + bulk copies; at the end, an aborted CTA waits for its copies in flight."""
    L = [f"{ind}if (t >= NC) {{",
         f"{ind}  const int pl = t - NC;",
         f"{ind}  int64_t issued = 0, xissued = 0;",
         f"{ind}  for (int64_t base = 0; base < ne_all; base += 32) {{",
         f"{ind}    const int64_t jv = base + pl < ne_all ? P.idx_j[e0 + base + pl] : 0;",
         f"{ind}    const int nb = (int)min((int64_t)32, ne_all - base);",
         f"{ind}    for (int k = 0; k < nb; ++k) {{",
         f"{ind}      const int64_t j = __shfl_sync(0xffffffffu, jv, k);",
         f"{ind}      if (pl == 0 && !*abort_flag) {{",
         f"{ind}        const int64_t kk = base + k;"]
    if gs.stage:
        # the in2 rows of a chunk, one bulk copy, issued with the chunk's first edge
        L += [f"{ind}        if (kk % {gs.ec} == 0) {{",
              f"{ind}          const int64_t c = kk / {gs.ec};",
              f"{ind}          const int b = (int)(c & 1);",
              f"{ind}          if (c < 2 || fc_mbar_wait(&xempty[b], (uint32_t)((c / 2 - 1) & 1), abort_flag, P.status)) {{",
              f"{ind}            const int nec = (int)min((int64_t){gs.ec}, ne_all - kk);",
              f"{ind}            fc_mbar_arrive_tx(&xfull[b], (uint32_t)(nec * D2 * 4));",
              f"{ind}            fc_bulk_g2s(xbuf + b * {gs.ec * gs.sig.d2}, P.in2 + (e0 + kk) * (int64_t)D2, (uint32_t)(nec * D2 * 4), &xfull[b]);",
              f"{ind}            xissued = c + 1;",
              f"{ind}          }}",
              f"{ind}        }}"]
    L += [f"{ind}        const int s = (int)(kk % {gs.ring});",
         f"{ind}        if (kk < {gs.ring} || fc_mbar_wait(&empty[s], (uint32_t)((kk / {gs.ring} - 1) & 1), abort_flag, P.status)) {{",
         f"{ind}          const bool ok = (uint64_t)j < (uint64_t)P.n_in1;",
         f"{ind}          if (!ok) fc_flag(P.status, FC_DEV_BAD_INDEX);",
         f"{ind}          sj[s] = ok ? j : -1;",
         f"{ind}          float* dst = ring + s * SLOT;",
         f"{ind}          fc_mbar_arrive_tx(&full[s], (uint32_t)(((ok ? XN : 0) + NW) * F * 4));",
         f"{ind}          if (ok) fc_bulk_g2s(dst, P.in1 + j * (int64_t)(D1 * F) + XLO * F, (uint32_t)(XN * F * 4), &full[s]);",
         f"{ind}          const float* wrow = P.w + (e0 + kk) * (int64_t)(NP * F);"]
    for (p0, n, r) in gs.w_runs:
        L.append(f"{ind}          fc_bulk_g2s(dst + (XN + {r}) * F, wrow + {p0} * F, (uint32_t)({n} * F * 4), &full[s]);")
    L += [f"{ind}          issued = kk + 1;",
          f"{ind}        }}",
          f"{ind}      }}",
          f"{ind}      __syncwarp();",
          f"{ind}    }}",
          f"{ind}  }}",
          f"{ind}  if (pl == 0 && *abort_flag) {{",
          f"{ind}    for (int64_t kk = issued > {gs.ring} ? issued - {gs.ring} : 0; kk < issued; ++kk)",
          f"{ind}      for (long long it = 0; it < FC_RING_WAIT_LIMIT; ++it)",
          f"{ind}        if (fc_mbar_test(&full[kk % {gs.ring}], (uint32_t)((kk / {gs.ring}) & 1))) break;",
          f"{ind}    for (int64_t c = xissued > 2 ? xissued - 2 : 0; c < xissued; ++c)",
          f"{ind}      for (long long it = 0; it < FC_RING_WAIT_LIMIT; ++it)",
          f"{ind}        if (fc_mbar_test(&xfull[c & 1], (uint32_t)((c >> 1) & 1))) break;",
          f"{ind}  }}",
          f"{ind}  return;",
          f"{ind}}}"]
    return L


def _phase1_loop(gs: GroupSlots, ind: str) -> List[str]:
    if gs.stage:
        load = [f"{ind}    const T* a2 = xbuf + (cidx & 1) * {gs.ec * gs.sig.d2} + le * D2;",
                f"{ind}    for (int q = 0; q < D2; ++q) x2[q] = xok ? a2[q] : T(0);"]
        head = [f"{ind}const int64_t cidx = eb / {gs.ec};",
                f"{ind}const bool xok = fc_mbar_wait(&xfull[cidx & 1], (uint32_t)((cidx >> 1) & 1), abort_flag, P.status);"]
        tail = [f"{ind}if (t == 0) fc_mbar_arrive(&xempty[cidx & 1]);"]
    else:
        load = [f"{ind}    const T* __restrict__ a2 = P.in2 + (e0 + eb + le) * (int64_t)D2;",
                f"{ind}    for (int q = 0; q < D2; ++q) x2[q] = fc_ldg(a2 + q);"]
        head, tail = [], []
    return [*head,
            f"{ind}for (int u = t; u < {gs.ec * NPART}; u += NC) {{",
            f"{ind}  const int le = u % {gs.ec}, part = u / {gs.ec};",
            f"{ind}  if (le < ne) {{",
            f"{ind}    T x2[D2];",
            *load,
            f"{ind}    float* mf = reinterpret_cast<float*>(m2) + le * NMF;",
            *_phase1(gs, ind + "    "),
            f"{ind}  }}",
            f"{ind}}}",
            f"{ind}fc_named_sync(1, NC);",
            *tail]


def _edge_begin(gs: GroupSlots, ind: str) -> List[str]:
    return [f"{ind}const int64_t kk = eb + k;",
            f"{ind}const int s = (int)(kk % {gs.ring});",
            f"{ind}const bool landed = fc_mbar_wait(&full[s], (uint32_t)((kk / {gs.ring}) & 1), abort_flag, P.status);",
            f"{ind}const int64_t j = landed ? sj[s] : -1;"]


def _edge_end(ind: str) -> List[str]:
    return [f"{ind}__syncwarp();",
            f"{ind}if (lane == 0) fc_mbar_arrive(&empty[s]);"]


def emit(sig, store_offsets: List[Tuple[int, int]]) -> str:
    groups = [GroupSlots(sig, g) for g in make_groups(sig, BUDGET)]
    for gs in groups:
        for k, v in group_cfg(gs).items():
            setattr(gs, k, v)
        gs.stage = STAGE_X2 and sig.d2 % 4 == 0  # 16-byte in2 rows: bulk-copied by the producer
    d2p = 1
    while d2p < sig.d2:
        d2p *= 2
    acc_out = {}
    k = 0
    for p, (r1, r2, o) in enumerate(sig.paths):
        for a in range(2 * o + 1):
            acc_out[(p, a)] = store_offsets[k][0]
            k += 1
    L = []
    w = L.append
    w(f"// ---- channel-pair convolution (float32): {len(groups)} path groups, producer warp")
    w(f"constexpr int P3_GROUPS = {len(groups)};")
    for kind in ("fwd", "bwd"):
        w(f"inline size_t {kind}3_smem(int g, int F) {{")
        w("  switch (g) {")
        for gi, gs in enumerate(groups):
            extra = gs.ec * d2p if kind == "bwd" else 0
            gextra = f" + {gs.nacc} * F" if (kind == "bwd" and gs.gsmem) else ""
            xb = 2 * gs.ec * gs.sig.d2 if gs.stage else 0
            w(f"    case {gi}: return (size_t){gs.nmp * gs.ec} * 8 + (size_t)({gs.ring} * ({gs.x_n} + {len(gs.paths)}) * F"
              f" + {extra + xb}{gextra}) * 4 + {gs.ring * 8 + 2 * gs.ring * 8 + 4 * 8 + 16};")
        w("  }")
        w("  return 0;")
        w("}")
    # ---------------- forward
    for gi, gs in enumerate(groups):
        w(f"__device__ __forceinline__ void fwd3_g{gi}(const TpParams<float>& P, unsigned char* smem) {{")
        L.extend(_setup(gs, "0", "  "))
        w(f"  constexpr int NMF = {scalar_offsets(gs)[1]};  // edge-matrix floats per edge (scalar layout)")
        L.extend(_producer(gs, "  "))
        w(f"  float2 acc[{gs.nacc}];")
        w(f"  for (int q = 0; q < {gs.nacc}; ++q) acc[q] = p2(0.0f);")
        w(f"  for (int64_t eb = 0; eb < ne_all; eb += {gs.ec}) {{")
        w(f"    const int ne = (int)min((int64_t){gs.ec}, ne_all - eb);")
        L.extend(_phase1_loop(gs, "    "))
        w("    for (int k = 0; k < ne; ++k) {")
        L.extend(_edge_begin(gs, "      "))
        w("      if (j >= 0) {")
        w("        const float* sx = ring + s * SLOT + 2 * t;")
        w("        float2 x1[XN];")
        w("        for (int q = 0; q < XN; ++q) x1[q] = ld2(sx + q * F);")
        w("        const float* sw = sx + XN * F;")
        w("        const float* mf = reinterpret_cast<const float*>(m2) + k * NMF;")
        L.extend(_fwd_body(gs, "        "))
        w("      }")
        L.extend(_edge_end("      "))
        w("    }")
        w("    fc_named_sync(1, NC);")
        w("  }")
        w("  float* __restrict__ o = P.out + row * (int64_t)(OUT_COMPS * F) + 2 * t;")
        k = 0
        for p in gs.paths:
            o_ = sig.paths[p][2]
            for a in range(2 * o_ + 1):
                w(f"  st2(o + {acc_out[(p, a)]} * F, acc[{k}]);")
                k += 1
        w("}")
    w("template <int G> struct P3Big;")
    for gi, gs in enumerate(groups):
        w(f"template <> struct P3Big<{gi}> {{ static constexpr bool value = {'true' if gs.big else 'false'}; }};")
    w("template <int G, int NT>")
    w("__global__ void __launch_bounds__(NT, P3MinBlocks<NT, P3Big<G>::value>::fwd) fwd3_kernel(TpParams<float> P) {")
    w("  extern __shared__ __align__(16) unsigned char fc_smem_raw[];")
    for gi in range(len(groups)):
        w(f"  if constexpr (G == {gi}) fwd3_g{gi}(P, fc_smem_raw);")
    w("}")
    # ---------------- backward
    for gi, gs in enumerate(groups):
        w("template <int NM>")
        w(f"__device__ __forceinline__ void bwd3_g{gi}(const TpBwdParams<float>& P, unsigned char* smem, bool multi) {{")
        w("  // NM: requested gradients as a compile-time mask (1 in1, 2 in2, 4 weights), 0 = read the pointers")
        w("  const bool NEED_1 = NM ? (NM & 1) != 0 : P.g_in1 != nullptr;")
        w("  const bool NEED_2 = NM ? (NM & 2) != 0 : P.g_in2 != nullptr;")
        w("  const bool NEED_W = NM ? (NM & 4) != 0 : P.g_w != nullptr;")
        L.extend(_setup(gs, f"{gs.ec * d2p}" + (f" + {gs.nacc} * F" if gs.gsmem else ""), "  "))
        w(f"  constexpr int NMF = {scalar_offsets(gs)[1]};  // edge-matrix floats per edge (scalar layout)")
        L.extend(_producer(gs, "  "))
        w("  float* gsm = extra;  // [EC][D2P] grad_in2 partial sums")
        if gs.gsmem:
            w(f"  float2* gb = reinterpret_cast<float2*>(gsm + {gs.ec * d2p});  // [NACC][NC] this thread's g pairs")
        else:
            w(f"  float2 g[{gs.nacc}];")
        w("  {")
        w("    const float* __restrict__ go = P.g_out + row * (int64_t)(OUT_COMPS * F) + 2 * t;")
        k = 0
        for p in gs.paths:
            o_ = sig.paths[p][2]
            for a in range(2 * o_ + 1):
                if gs.gsmem:
                    w(f"    gb[{k} * NC + t] = ldg2(go + {acc_out[(p, a)]} * F);")
                else:
                    w(f"    g[{k}] = ldg2(go + {acc_out[(p, a)]} * F);")
                k += 1
        w("  }")
        w(f"  for (int64_t eb = 0; eb < ne_all; eb += {gs.ec}) {{")
        w(f"    const int ne = (int)min((int64_t){gs.ec}, ne_all - eb);")
        w(f"    for (int u = t; u < {gs.ec * d2p}; u += NC) gsm[u] = 0.0f;")
        L.extend(_phase1_loop(gs, "    "))
        w("    for (int k = 0; k < ne; ++k) {")
        L.extend(_edge_begin(gs, "      "))
        w("      if (j >= 0) {")
        w("        const int64_t e = e0 + kk;")
        w("        const float* sx = ring + s * SLOT + 2 * t;")
        w("        float2 x1[XN], gx1[XN];")
        w(f"        float2 gx2[{d2p}];")
        w("        for (int q = 0; q < XN; ++q) x1[q] = ld2(sx + q * F);")
        w("        const float* sw = sx + XN * F;")
        w("        float* __restrict__ gwr = NEED_W ? P.g_w + e * (int64_t)(NP * F) + 2 * t : nullptr;")
        w("        const float* mf = reinterpret_cast<const float*>(m2) + k * NMF;")
        L.extend(_bwd_body(gs, "        ", d2p))
        w("        if (NEED_1) {")
        w("          float* __restrict__ t1 = P.g_in1 + j * (int64_t)(D1 * F) + XLO * F + 2 * t;")
        w("          for (int q = 0; q < XN; ++q) red2(t1 + q * F, gx1[q]);")
        w("        }")
        w("        if (NEED_2) {")
        w(f"          float v[{d2p}];")
        w(f"          for (int q = 0; q < {d2p}; ++q) v[q] = gx2[q].x + gx2[q].y;")
        w(f"          const int comp = fc_warp_transpose_reduce<float, {d2p}>(v);")
        w(f"          if ((lane & {32 // d2p - 1}) == 0 && comp < D2) atomicAdd(gsm + k * {d2p} + comp, v[0]);")
        w("        }")
        w("      }")
        L.extend(_edge_end("      "))
        w("    }")
        w("    fc_named_sync(1, NC);")
        w("    if (NEED_2) {")
        w("      for (int u = t; u < ne * D2; u += NC) {")
        w("        const int k = u / D2, q = u % D2;")
        w("        float* dst = P.g_in2 + (e0 + eb + k) * (int64_t)D2 + q;")
        w(f"        const float v = gsm[k * {d2p} + q];")
        w("        if (multi) atomicAdd(dst, v); else *dst = v;")
        w("      }")
        w("    }")
        w("    fc_named_sync(1, NC);")
        w("  }")
        w("}")
    w("template <int G, int NM, int NT>")
    w("__global__ void __launch_bounds__(NT, P3MinBlocks<NT, P3Big<G>::value>::bwd) bwd3_kernel(TpBwdParams<float> P) {")
    w("  extern __shared__ __align__(16) unsigned char fc_smem_raw[];")
    for gi in range(len(groups)):
        w(f"  if constexpr (G == {gi}) bwd3_g{gi}<NM>(P, fc_smem_raw, P3_GROUPS > 1);")
    w("}")
    # ---------------- launchers
    w("template <int G, int NT>")
    w("int launch_fwd3_nt(const TpParams<float>& P, size_t smem, cudaStream_t s) {")
    w("  if (smem > 48 * 1024 && cudaFuncSetAttribute(fwd3_kernel<G, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, "
      "(int)smem) != cudaSuccess) return FC_ERR_LAUNCH;")
    w("  fwd3_kernel<G, NT><<<(unsigned)P.n_rows, NT, smem, s>>>(P);")
    w("  return fc_check_launch();")
    w("}")
    w("template <int G>")
    w("int launch_fwd3_group(const TpParams<float>& P, cudaStream_t s) {")
    w("  const size_t smem = fwd3_smem(G, P.F);")
    w("  if (smem > 227 * 1024) return FC_ERR_UNSUPPORTED;")
    w("  switch (P.F) {")
    w("    case 64: return launch_fwd3_nt<G, 64>(P, smem, s);")
    w("    case 128: return launch_fwd3_nt<G, 96>(P, smem, s);")
    w("  }")
    w("  return FC_ERR_UNSUPPORTED;")
    w("}")
    w("template <int G, int NM, int NT>")
    w("int launch_bwd3_nt(const TpBwdParams<float>& P, size_t smem, cudaStream_t s) {")
    w("  if (smem > 48 * 1024 && cudaFuncSetAttribute(bwd3_kernel<G, NM, NT>, "
      "cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return FC_ERR_LAUNCH;")
    w("  bwd3_kernel<G, NM, NT><<<(unsigned)P.n_rows, NT, smem, s>>>(P);")
    w("  return fc_check_launch();")
    w("}")
    w("template <int G, int NM>")
    w("int launch_bwd3_variant(const TpBwdParams<float>& P, size_t smem, cudaStream_t s) {")
    w("  switch (P.F) {")
    w("    case 64: return launch_bwd3_nt<G, NM, 64>(P, smem, s);")
    w("    case 128: return launch_bwd3_nt<G, NM, 96>(P, smem, s);")
    w("  }")
    w("  return FC_ERR_UNSUPPORTED;")
    w("}")
    w("template <int G>")
    w("int launch_bwd3_group(const TpBwdParams<float>& P, cudaStream_t s) {")
    w("  const size_t smem = bwd3_smem(G, P.F);")
    w("  if (smem > 227 * 1024) return FC_ERR_UNSUPPORTED;")
    w("  const int nm = (P.g_in1 ? 1 : 0) | (P.g_in2 ? 2 : 0) | (P.g_w ? 4 : 0);")
    w("  if (nm == 7) return launch_bwd3_variant<G, 7>(P, smem, s);")
    w("  if (nm == 6) return launch_bwd3_variant<G, 6>(P, smem, s);")
    w("  return launch_bwd3_variant<G, 0>(P, smem, s);")
    w("}")
    for kind, params in (("fwd", "TpParams"), ("bwd", "TpBwdParams")):
        w(f"inline int launch_{kind}3(const {params}<float>& P, cudaStream_t s) {{")
        w("  if (P.n_rows == 0) return 0;")
        w("  if (P.n_rows > 0x7fffffffLL || (P.F != 64 && P.F != 128)) return FC_ERR_UNSUPPORTED;")
        for gi in range(len(groups)):
            w(f"  if (int rc = launch_{kind}3_group<{gi}>(P, s)) return rc;")
        w("  return 0;")
        w("}")
    return "\n".join(L) + "\n"


# ---------------------------------------------------------------------------------------
# Four-channel forward (F = 128): one consumer warp per receiver, each thread owning the
# channels 4t .. 4t+3 as two packed pairs. Every 16-byte broadcast of an edge-matrix pair
# then feeds four channels instead of two, so the edge matrices are read from shared
# memory by one warp per receiver instead of two (the forward's shared-memory wavefronts
# are mostly these broadcasts); sender rows and weights come as 16-byte loads. A thread
# holds two register copies of its accumulators, so it is emitted only for signatures
# whose paths fit one group of at most BUDGET4 accumulator pairs. Measured at C = 128 on
# the 1.49 M-edge benchmark graph: (0,3)->3 (one group of 16) 0.89 -> 0.73 ms; (3,3)->3
# split into eight such groups instead of the pair kernel's three took 8.6 ms against 5.8
# (each group walks the edges and gathers its sender rows again, at half the consumer
# warps per SM), so larger signatures keep the pair kernel.
BUDGET4 = 16
FWD4_MIN_CTAS = 5


def make_groups4(sig) -> List[List[int]]:
    order = sorted(range(len(sig.paths)), key=lambda p: (-sig.paths[p][0], p))
    groups, cur, used = [], [], 0
    for p in order:
        n = 2 * sig.paths[p][2] + 1
        if cur and (used + n > BUDGET4 or sig.paths[cur[-1]][0] != sig.paths[p][0]):
            groups.append(sorted(cur))
            cur, used = [], 0
        cur.append(p)
        used += n
    if cur:
        groups.append(sorted(cur))
    nacc = lambda g: sum(2 * sig.paths[p][2] + 1 for p in g)
    while len(groups) > 1 and nacc(groups[-1]) + nacc(groups[-2]) <= BUDGET4:
        last = groups.pop()
        groups[-1] = sorted(groups[-1] + last)
    return groups


def _fwd4_body(gs: GroupSlots, ind: str) -> List[str]:
    sig = gs.sig
    L = []
    acc_base = 0
    for p in gs.paths:
        r1, r2, o = sig.paths[p]
        s0 = gs.range[p][0]
        L.append(f"{ind}{{ // path {p}: ({r1},{r2})->{o}")
        L.extend(_path_mload(gs, p, ind + "  "))
        L.append(f"{ind}  float2 wpa, wpb;")
        L.append(f"{ind}  ld4p(sw + {gs.w_pos[p]} * F, wpa, wpb);")
        for a in range(2 * o + 1):
            for h in ("a", "b"):
                pairs = [(f"mv[{gs.index[(p, a, i)] - s0}]", f"x1{h}[{_q(r1, i) - gs.x_lo}]")
                         for i in range(2 * r1 + 1) if (p, a, i) in gs.index]
                L.append(f"{ind}  acc{h}[{acc_base + a}] = pfma(wp{h}, {_chain(pairs)}, acc{h}[{acc_base + a}]);")
        L.append(f"{ind}}}")
        acc_base += 2 * o + 1
    return L


def has_fwd4(sig) -> bool:
    return len(make_groups4(sig)) == 1


def emit_fwd4(sig, store_offsets: List[Tuple[int, int]]) -> str:
    if not has_fwd4(sig):
        return ""
    groups = [GroupSlots(sig, g) for g in make_groups4(sig)]
    for gs in groups:
        gs.big, gs.ec, gs.ring, gs.gsmem = True, 8, 4, False
        gs.stage = STAGE_X2 and sig.d2 % 4 == 0
    acc_out = {}
    k = 0
    for p, (r1, r2, o) in enumerate(sig.paths):
        for a in range(2 * o + 1):
            acc_out[(p, a)] = store_offsets[k][0]
            k += 1
    L = []
    w = L.append
    w(f"// ---- four-channel convolution forward (float32, F = 128): {len(groups)} path groups")
    w("#ifndef FC_P4_FWD_MINB")
    w(f"#define FC_P4_FWD_MINB {FWD4_MIN_CTAS}")
    w("#endif")
    w(f"constexpr int P4_GROUPS = {len(groups)};")
    w("inline size_t fwd4_smem(int g, int F) {")
    w("  switch (g) {")
    for gi, gs in enumerate(groups):
        xb = 2 * gs.ec * gs.sig.d2 if gs.stage else 0
        w(f"    case {gi}: return (size_t){gs.nmp * gs.ec} * 8 + (size_t)({gs.ring} * ({gs.x_n} + {len(gs.paths)}) * F"
          f" + {xb}) * 4 + {gs.ring * 8 + 2 * gs.ring * 8 + 4 * 8 + 16};")
    w("  }")
    w("  return 0;")
    w("}")
    for gi, gs in enumerate(groups):
        w(f"__device__ __forceinline__ void fwd4_g{gi}(const TpParams<float>& P, unsigned char* smem) {{")
        L.extend(_setup(gs, "0", "  ", channels_per_thread=4))
        w(f"  constexpr int NMF = {scalar_offsets(gs)[1]};  // edge-matrix floats per edge (scalar layout)")
        L.extend(_producer(gs, "  "))
        w(f"  float2 acca[{gs.nacc}], accb[{gs.nacc}];")
        w(f"  for (int q = 0; q < {gs.nacc}; ++q) {{ acca[q] = p2(0.0f); accb[q] = p2(0.0f); }}")
        w(f"  for (int64_t eb = 0; eb < ne_all; eb += {gs.ec}) {{")
        w(f"    const int ne = (int)min((int64_t){gs.ec}, ne_all - eb);")
        L.extend(_phase1_loop(gs, "    "))
        w("    for (int k = 0; k < ne; ++k) {")
        L.extend(_edge_begin(gs, "      "))
        w("      if (j >= 0) {")
        w("        const float* sx = ring + s * SLOT + 4 * t;")
        w("        float2 x1a[XN], x1b[XN];")
        w("        for (int q = 0; q < XN; ++q) ld4p(sx + q * F, x1a[q], x1b[q]);")
        w("        const float* sw = sx + XN * F;")
        w("        const float* mf = reinterpret_cast<const float*>(m2) + k * NMF;")
        L.extend(_fwd4_body(gs, "        "))
        w("      }")
        L.extend(_edge_end("      "))
        w("    }")
        w("    fc_named_sync(1, NC);")
        w("  }")
        w("  float* __restrict__ o = P.out + row * (int64_t)(OUT_COMPS * F) + 4 * t;")
        k = 0
        for p in gs.paths:
            o_ = sig.paths[p][2]
            for a in range(2 * o_ + 1):
                w(f"  st4p(o + {acc_out[(p, a)]} * F, acca[{k}], accb[{k}]);")
                k += 1
        w("}")
    w("template <int G>")
    w("__global__ void __launch_bounds__(64, FC_P4_FWD_MINB) fwd4_kernel(TpParams<float> P) {")
    w("  extern __shared__ __align__(16) unsigned char fc_smem_raw[];")
    for gi in range(len(groups)):
        w(f"  if constexpr (G == {gi}) fwd4_g{gi}(P, fc_smem_raw);")
    w("}")
    w("template <int G>")
    w("int launch_fwd4_group(const TpParams<float>& P, cudaStream_t s) {")
    w("  const size_t smem = fwd4_smem(G, P.F);")
    w("  if (smem > 227 * 1024) return FC_ERR_UNSUPPORTED;")
    w("  if (smem > 48 * 1024 && cudaFuncSetAttribute(fwd4_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, "
      "(int)smem) != cudaSuccess) return FC_ERR_LAUNCH;")
    w("  fwd4_kernel<G><<<(unsigned)P.n_rows, 64, smem, s>>>(P);")
    w("  return fc_check_launch();")
    w("}")
    w("inline int launch_fwd4(const TpParams<float>& P, cudaStream_t s) {")
    w("  if (P.n_rows == 0) return 0;")
    w("  if (P.n_rows > 0x7fffffffLL || P.F != 128) return FC_ERR_UNSUPPORTED;")
    for gi in range(len(groups)):
        w(f"  if (int rc = launch_fwd4_group<{gi}>(P, s)) return rc;")
    w("  return 0;")
    w("}")
    return "\n".join(L) + "\n"
