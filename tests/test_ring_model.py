"""Index arithmetic of the online and cluster kernels, modelled on the CPU.

The kernels walk their rows and their shared-memory ring without dividing:
a row cursor (matrix b, row i) that advances by (step // rows, step % rows)
with one carry (`RowCursor`, csrc/kernels/geometry.cuh), and a ring position
(stage, phase parity) advanced one use at a time (`RingPos`,
csrc/kernels/common.cuh). Three places derive barrier phases from that
position instead of from the use index: the producer's wait for a stage's
previous use, the end-of-loop flush of the rows still held by the cluster
kernel's stages, and the wait for loads in flight after an abort. These
tests replay those rules and compare them with the division-based formulas
(use r of the ring lives in stage r % S, phase parity (r // S) & 1) over many
ring depths and use counts.
"""
import os
import random
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KERNELS = os.path.join(ROOT, "gb200-sm100a-tma-fused-causal-attention-softmax_b200", "csrc", "kernels")


class RingPos:
    def __init__(self):
        self.s, self.ph = 0, 0

    def next(self, S):
        self.s += 1
        if self.s == S:
            self.s, self.ph = 0, self.ph ^ 1

    def copy(self):
        c = RingPos()
        c.s, c.ph = self.s, self.ph
        return c


def ring_at(n, S):
    pos = RingPos()
    for _ in range(n):
        pos.next(S)
    return pos


@pytest.mark.parametrize("S", [1, 2, 3, 4, 7, 8, 14, 32])
def test_position_and_previous_phase_match_division(S):
    pos = RingPos()
    for r in range(5 * S + 3):
        assert (pos.s, pos.ph) == (r % S, (r // S) & 1)
        if r >= S:
            # The producer waits for the stage's previous use: phase parity
            # ((r // S) - 1) & 1, which the kernels take as pos.ph ^ 1.
            assert pos.ph ^ 1 == ((r // S) - 1) & 1
        pos.next(S)


@pytest.mark.parametrize("S", [1, 2, 3, 5, 8, 13])
def test_abort_tail_waits_cover_the_last_uses(S):
    # After an abort at use j (not issued), the kernels wait, for each stage
    # k, for the phase of its last use d = (pos.s - 1 - k) mod S back, if
    # that use exists: parity pos.ph for k < pos.s, else pos.ph ^ 1.
    for j in range(0, 4 * S + 2):
        pos = ring_at(j, S)
        got = set()
        for k in range(S):
            d = (pos.s - 1 - k + S) % S
            if j - 1 - d < 0:
                continue
            got.add((k, pos.ph if k < pos.s else pos.ph ^ 1))
        want = {(r % S, (r // S) & 1) for r in range(max(0, j - S), j)}
        assert got == want, (S, j)


@pytest.mark.parametrize("S", [1, 2, 3, 4, 8])
def test_cluster_flush_stores_every_held_row_once(S):
    # After j rows, the stages from position j on hold rows j - S .. j - 1
    # (those >= 0); each is released in the phase before its position's.
    for j in range(0, 4 * S + 2):
        pos = ring_at(j, S)
        f = pos.copy()
        got = []
        for k in range(S):
            if j + k >= S:
                got.append((f.s, f.ph ^ 1))
            f.next(S)
        want = [(jj % S, ((jj // S) - 1) & 1) for jj in range(j, j + S) if jj - S >= 0]
        assert got == want, (S, j)
        # The stages named are exactly those of rows j - S .. j - 1.
        assert sorted(s for s, _ in got) == sorted((r % S) for r in range(max(0, j - S), j))


class RowCursor:
    def __init__(self, rows, first, step):
        self.rows = rows
        self.b, self.i = first // rows, first % rows
        self.step_b, self.step_i = step // rows, step % rows

    def next(self):
        # The kernels form i + step_i in 32 unsigned bits: both are below
        # rows < 2^31, so the sum stays below 2^32.
        self.b += self.step_b
        n = self.i + self.step_i
        assert n < 2 ** 32
        if n >= self.rows:
            n -= self.rows
            self.b += 1
        self.i = n


def test_row_cursor_walks_the_flat_rows():
    rng = random.Random(7)
    cases = [(4096, 444, 3), (32768, 444, 3), (1, 888, 5), (7, 148, 40), (100, 100, 3), (4095, 8192, 4)]
    cases += [(rng.randint(1, 5000), rng.randint(1, 3000), rng.randint(1, 9)) for _ in range(200)]
    for rows, grid, batch in cases:
        total = rows * batch
        for first in {0, 1, grid // 2, grid - 1}:
            if first >= grid:
                continue
            cur = RowCursor(rows, first, grid)
            seen = []
            while cur.b < batch:  # inside the launch exactly while the matrix index is
                seen.append(cur.b * rows + cur.i)
                assert 0 <= cur.i < rows
                cur.next()
            assert seen == list(range(first, total, grid)), (rows, grid, batch, first)


@pytest.fixture(scope="module")
def cursor_check(tmp_path_factory):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("g++ not available")
    exe = str(tmp_path_factory.mktemp("cursor") / "cursor_check")
    subprocess.run([cxx, "-O2", "-std=c++17", "-D__host__=", "-D__device__=",
                    "-D__forceinline__=inline", "-I", KERNELS,
                    os.path.join(ROOT, "tests", "cursor_check.cpp"), "-o", exe], check=True)

    def run(cases):
        text = "".join(f"{r} {b} {s}\n" for r, b, s in cases)
        out = subprocess.run([exe], input=text, capture_output=True, text=True, check=True).stdout
        res = [tuple(int(x) for x in line.split()) for line in out.splitlines()]
        assert len(res) == len(cases)
        return res

    return run


def test_row_cursor_of_the_kernels_up_to_the_largest_row_count(cursor_check):
    # The header's own RowCursor, compiled as C++: small shapes with the step
    # above and below the row count, and matrices of up to 2^31 - 1 rows (the
    # largest the ABI accepts), where a signed 32-bit i + step_i would
    # overflow within the last `step` rows of every matrix.
    rng = random.Random(5)
    cases = [(4096, 3, 444), (7, 5, 148), (1, 9, 888), (100, 3, 100), (32768, 2, 3552),
             (2 ** 31 - 1, 2, 888), (2 ** 31 - 700, 2, 888), (2 ** 31 - 1, 1, 148 * 7)]
    cases += [(rng.randint(1, 5000), rng.randint(1, 6), rng.randint(1, 3000)) for _ in range(300)]
    for (rows, batch, step), (visits, ok) in zip(cases, cursor_check(cases)):
        assert ok == 1, (rows, batch, step)
        assert visits > 0
