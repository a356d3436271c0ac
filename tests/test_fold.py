"""CPU tests of folded row-block shards: the launch geometry of
kernels/geometry.cuh compiled as plain C++ (tests/geometry_check.cpp) and
checked by brute force, and bench.rank_segments.

A folded launch stores two row blocks of one matrix one after the other
(local rows >= split_row sit split_shift rows further down the matrix); the
row-resident kernels pair rows inside it, so a rank that holds a block and
its mirror gets row pairs of rows + 1 causal elements each."""
from __future__ import annotations

import os
import random
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KERNELS = os.path.join(ROOT, "gb200-sm100a-tma-fused-causal-attention-softmax_b200", "csrc", "kernels")
sys.path.insert(0, ROOT)


@pytest.fixture(scope="module")
def geometry_check(tmp_path_factory):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("g++ not available")
    exe = str(tmp_path_factory.mktemp("geom") / "geometry_check")
    subprocess.run([cxx, "-O2", "-std=c++17", "-D__host__=", "-D__device__=",
                    "-D__forceinline__=inline", "-I", KERNELS,
                    os.path.join(ROOT, "tests", "geometry_check.cpp"), "-o", exe], check=True)

    def run(geoms):
        text = "".join(f"{r} {c} {o} {s} {h}\n" for r, c, o, s, h in geoms)
        out = subprocess.run([exe], input=text, capture_output=True, text=True, check=True).stdout
        rows = [tuple(int(x) for x in line.split()) for line in out.splitlines()]
        assert len(rows) == len(geoms)
        return rows

    return run


def test_geometry_random(geometry_check):
    rng = random.Random(11)
    geoms = []
    for _ in range(3000):
        rows = rng.randint(1, 70)
        cols = rng.randint(1, 90)
        off = rng.randint(0, 100)
        split = rng.choice([0, rng.randint(0, rows - 1)])
        shift = 0 if split == 0 else rng.randint(0, 60)
        geoms.append((rows, cols, off, split, shift))
    for g, (n_tri, units, bound, max_nv, lo, hi, ok) in zip(geoms, geometry_check(geoms)):
        assert ok == 1, g
        assert max_nv <= bound <= max_nv + 2, (g, bound, max_nv)


def test_geometry_unsplit_bound_unchanged(geometry_check):
    """Without a fold, the stage bound is the closed form of one row block:
    a pair holds 2*row_offset + n_tri + 1 elements."""
    rng = random.Random(5)
    geoms = [(rng.randint(1, 5000), rng.randint(1, 5000), rng.randint(0, 6000), 0, 0) for _ in range(500)]
    geoms += [(4096, 4096, 0, 0, 0), (8192, 8192, 0, 0, 0), (32768, 32768, 0, 0, 0), (1000, 1037, 0, 0, 0)]
    for (rows, cols, off, _, _), (n_tri, units, bound, *_rest) in zip(geoms, geometry_check(geoms)):
        n_pairs = n_tri // 2
        want = 0
        if n_pairs:
            want = max(want, (2 * off + n_tri + 1 + 7) // 8 + 1)
        if n_tri & 1:
            want = max(want, (off + n_pairs + 1 + 7) // 8)
        if rows > n_tri:
            want = max(want, (cols + 7) // 8)
        assert bound == want, (rows, cols, off)


def fold_geometry(rows, cols, parts, rank):
    import bench

    segs = bench.rank_segments(rows, cols, parts, rank)
    (a, n), rest = segs[0], segs[1:]
    if not rest:
        return (n, cols, a, 0, 0)
    b, m = rest[0]
    return (n + m, cols, a, n, b - (a + n))


@pytest.mark.parametrize("parts", [2, 3, 4, 8])
def test_fold_pairs_carry_whole_matrix_units(geometry_check, parts):
    sizes = [(64, 64), (1000, 1037), (1001, 1001), (4096, 4096), (8192, 8192), (32768, 32768)]
    geoms = [fold_geometry(r, c, parts, k) for r, c in sizes for k in range(parts)]
    res = geometry_check(geoms)
    i = 0
    for rows, cols in sizes:
        for k in range(parts):
            g, (n_tri, units, bound, max_nv, lo, hi, ok) = geoms[i], res[i]
            i += 1
            assert ok == 1, g
            # Every pair holds rows + 1 elements (rows for the rank that holds
            # the last row of a square matrix, which is a full-width single).
            assert rows <= lo <= hi <= rows + 1, (rows, k, lo, hi)
            assert bound <= (rows + 1 + 7) // 8 + 1


@pytest.mark.parametrize("rows,cols", [(64, 64), (1000, 1037), (1001, 1001), (32768, 32768), (4096, 32)])
@pytest.mark.parametrize("parts", [1, 2, 3, 4, 8])
def test_rank_segments_cover_rows_once(rows, cols, parts):
    import bench

    seen = [0] * rows
    costs = []
    for k in range(parts):
        segs = bench.rank_segments(rows, cols, parts, k)
        assert 1 <= len(segs) <= 2
        if len(segs) == 2:
            (a, n), (b, m) = segs
            assert b >= a + n  # the second block starts after the first
        cost = 0
        for a, n in segs:
            assert n > 0
            for r in range(a, a + n):
                seen[r] += 1
                cost += 2 * min(r + 1, cols) + 2 * cols
        costs.append(cost)
    assert seen == [1] * rows
    if rows <= cols:
        # Equal shards up to the rounding of rows // 2 over the ranks.
        per_row = 2 * (rows + 1) + 4 * cols
        assert max(costs) - min(costs) <= 2 * per_row * 2
