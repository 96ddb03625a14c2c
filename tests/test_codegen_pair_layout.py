"""Shared-memory layout of the edge matrices in the channel-pair convolution kernels
(``codegen/emit_pair.py``), checked on the generator for every signature and every path
group the kernels are emitted for (no GPU).

Each edge's matrices ``M_p[a, i]`` are written by the cooperative phase-1 code as plain
floats and read back per path with 16-byte loads of four entries. The kernels are only
correct if (1) each path's first entry sits on a 16-byte boundary (the float4 loads),
(2) every entry the arithmetic reads was written, at a position of its own, and the reads
of one path never pick up another path's entries, and (3) an edge's floats fit the
per-edge stride of the shared-memory carve-up (NMP pairs = 2 * NMP floats).
"""

import re

import pytest

from flashcart_b200.codegen import emit, emit_pair
from flashcart_b200.codegen.emit_conv import GroupSlots, make_groups


def _groups():
    for sig in emit.all_signatures():
        for g in make_groups(sig, emit_pair.BUDGET):
            yield sig, "pair", GroupSlots(sig, g)
        if emit_pair.has_fwd4(sig):
            for g in emit_pair.make_groups4(sig):
                yield sig, "four", GroupSlots(sig, g)


CASES = list(_groups())


def test_every_signature_has_pair_groups():
    assert len(CASES) > len(emit.all_signatures())


@pytest.mark.parametrize("sig,kind,gs", CASES, ids=[f"{s.name}-{k}-{','.join(map(str, g.paths))}"
                                                    for s, k, g in CASES])
def test_scalar_edge_matrix_layout(sig, kind, gs):
    off, nmf = emit_pair.scalar_offsets(gs)
    assert nmf % 4 == 0 and nmf <= 2 * gs.nmp
    assert all(off[p] % 4 == 0 for p in gs.paths)

    # what phase 1 writes: position -> slot (each position written once)
    written = {}
    text = "\n".join(emit_pair._phase1(gs, ""))
    for pos, expr in re.findall(r"mf\[(\d+)\] = (.+);", text):
        pos = int(pos)
        assert pos not in written and 0 <= pos < nmf
        written[pos] = expr
    assert len(written) == sum(1 for s in gs.slots if s is not None)

    # what each path's loads read, and which mv register each float lands in
    owner = {}
    for p in gs.paths:
        s0, s1 = gs.range[p]
        text = "\n".join(emit_pair._path_mload(gs, p, ""))
        base = None
        for line in text.splitlines():
            m = re.search(r"mf \+ (\d+)\)", line)
            if m:
                base = int(m.group(1))
                assert base % 4 == 0
                continue
            m = re.search(r"mv\[(\d+)\] = p2\(q\.([xyzw])\)", line)
            if m:
                k, comp = int(m.group(1)), "xyzw".index(m.group(2))
                pos = base + comp
                slot = s0 + k
                assert pos in written, f"path {p} reads float {pos} that phase 1 never writes"
                assert owner.setdefault(pos, p) == p, f"float {pos} read by paths {owner[pos]} and {p}"
                # the float holds this slot's entry: the same expression phase 1 writes for it
                if gs.slots[slot] is not None:
                    assert written[pos] == gs.m_expr(slot)
        # every nonzero entry of the path is read
        assert {pos for pos, q in owner.items() if q == p} == {
            off[p] + s - s0 for s in range(s0, s1) if gs.slots[s] is not None}
