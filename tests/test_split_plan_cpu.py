"""The GEMM's split-tail plan (svdq_linear_gemm_plan, host only) walked the way the kernel walks
it (a Python mirror of its unit walker in csrc/linear_gemm.cu): every K iteration of every tile is
computed exactly once; each pair hands at most one partial to an owner, and that is the pair's
first tail unit; an owner's unit is its pair's last, and its helpers are the following pairs."""
from __future__ import annotations

import ctypes

import pytest


def _plan(tiles, iters, max_pairs, ws=True):
    from krea2_svdquant_b200 import _lib, build
    build.build()
    out = (ctypes.c_int * 4)()
    _lib.call("svdq_linear_gemm_plan", tiles, iters, max_pairs, 1 if ws else 0, out)
    return tuple(out)


def _units(pair, pairs, dp_tiles, tail_len, tail_total, iters):
    """Mirror of walk_init / walk_next: (tile, k0, k1) in the order the pair runs them."""
    out = []
    j = 0
    while pair + j * pairs < dp_tiles:
        out.append((pair + j * pairs, 0, iters))
        j += 1
    if tail_total > 0:
        g = min(pair * tail_len, tail_total)
        gend = min(g + tail_len, tail_total)
        while g < gend:
            tt = g // iters
            k0 = g - tt * iters
            k1 = min(iters, k0 + gend - g)
            out.append((dp_tiles + tt, k0, k1))
            g += k1 - k0
    return out


CASES = [(102, 97, 74), (408, 97, 74), (408, 257, 74), (1024, 97, 74), (1088, 97, 74), (1, 97, 74),
         (1, 17, 74), (6, 10, 74), (4, 98, 74), (48, 97, 74), (96, 97, 74), (3, 9, 74), (500, 40, 70),
         (7, 300, 8), (0, 97, 74)]


@pytest.mark.parametrize("tiles,iters,max_pairs", CASES)
def test_plan_covers_every_iteration_once(tiles, iters, max_pairs):
    pairs, dp_tiles, tail_len, tail_total = _plan(tiles, iters, max_pairs)
    assert 0 <= pairs <= max(max_pairs, 0)
    if tiles == 0:
        return
    assert pairs >= 1
    if tail_total == 0:
        assert dp_tiles == tiles and pairs == min(tiles, max_pairs)
    else:
        assert tail_total == (tiles - dp_tiles) * iters and dp_tiles % max_pairs == 0
        assert 8 <= tail_len < iters and tail_len >= -(-iters // 4)
        assert (tiles - dp_tiles) * 20 <= max_pairs * 11
    seen = {}
    owner_of = {}
    for p in range(pairs):
        units = _units(p, pairs, dp_tiles, tail_len, tail_total, iters)
        contrib = [i for i, (_, k0, _) in enumerate(units) if k0 > 0]
        assert len(contrib) <= 1 and (not contrib or units[contrib[0]][0] >= dp_tiles)
        if contrib:  # the pair's first tail unit
            assert all(t < dp_tiles for t, _, _ in units[:contrib[0]])
        for i, (t, k0, k1) in enumerate(units):
            assert k0 < k1
            for k in range(k0, k1):
                assert (t, k) not in seen
                seen[(t, k)] = p
            if k0 == 0 and k1 < iters:
                assert i == len(units) - 1, "an owner's unit is its pair's last"
                tile_end = (t - dp_tiles + 1) * iters
                helpers = [c for c in range(p + 1, pairs) if c * tail_len < tile_end]
                owner_of[t] = (p, helpers)
    assert len(seen) == tiles * iters
    # each split tile: its owner's helpers are exactly the pairs holding its other iterations
    for t, (p, helpers) in owner_of.items():
        others = sorted({seen[(t, k)] for k in range(iters)} - {p})
        assert others == helpers


def test_plan_thresholds():
    # a last wave above 11/20 of the pairs stays whole; without a workspace nothing splits
    assert _plan(1088, 97, 74)[3] == 0          # ff.gate / ff.up: 52 of 74
    assert _plan(1024, 97, 74)[3] == 0          # config 2: 62 of 74
    assert _plan(102, 97, 74)[3] == 28 * 97     # to_k / to_v
    assert _plan(102, 97, 74, ws=False)[3] == 0
    assert _plan(1, 4, 74)[3] == 0              # too few K iterations to cut
