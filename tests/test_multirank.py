"""Multi-rank host path on CPU (gloo, world_size 2): the sharding bench.py uses.

Each rank regenerates only its shard (heads via first_batch, row blocks via
first_row), computes it with the oracle standing in for the device kernel
(row_offset = absolute first row), and the shards gathered on rank 0 must equal
the unsharded result bit for bit. Also checks the max-over-ranks timing
reduction and that row blocks are balanced by causal cost.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q):
    import bench
    import causal_softmax as cs
    import oracle_ctypes as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # Row blocks of one matrix (the single-matrix workloads).
        rows, cols = 300, 260
        pitch = cs.padded_pitch(cols)
        a, b = bench.row_blocks(rows, cols, world)[rank]
        x = cs.generate(3, 2, batch=1, rows=b - a, cols=cols, first_row=a)[0]
        y = O.softmax_strided(x.ravel(), 1, 0, b - a, cols, pitch, a, 1.0).reshape(b - a, pitch)
        parts = [None] * world
        dist.all_gather_object(parts, (a, b, y))
        # Folded shards (a row block and its mirror, stored one after the
        # other), laid out as bench.py lays out a rank's buffer.
        fr, fc = 301, 320  # folding needs rows <= cols; an odd count leaves a middle row
        fp = cs.padded_pitch(fc)
        segs = bench.rank_segments(fr, fc, world, rank)
        xf = np.concatenate([cs.generate(3, 2, batch=1, rows=n, cols=fc, first_row=s0)[0]
                             for s0, n in segs])
        yf = np.concatenate([O.softmax_strided(xf[o:o + n].ravel(), 1, 0, n, fc, fp, s0, 1.0)
                             .reshape(n, fp)
                             for (s0, n), o in zip(segs, np.cumsum([0] + [n for _, n in segs]))])
        fparts = [None] * world
        dist.all_gather_object(fparts, yf)
        # Heads (the batched workload), split as bench.py splits them.
        heads, hr = 6, 40
        hp = cs.padded_pitch(hr)
        first, per = bench.head_range(heads, world, rank)
        xh = cs.generate(4, 3, batch=per, rows=hr, cols=hr, first_batch=first)
        yh = O.softmax_strided(xh.ravel(), per, hr * hp, hr, hr, hp, 0, 0.0883883).reshape(per, hr, hp)
        hparts = [None] * world
        dist.all_gather_object(hparts, yh)
        # Max over ranks, as bench.py reduces its step times.
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put((parts, fparts, hparts, float(t.item())))
    finally:
        dist.destroy_process_group()


def test_sharded_results_equal_unsharded():
    import bench
    import causal_softmax as cs
    import oracle_ctypes as O

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    parts, fparts, hparts, tmax = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert tmax == float(world)

    rows, cols = 300, 260
    pitch = cs.padded_pitch(cols)
    x = cs.generate(3, 2, batch=1, rows=rows, cols=cols)[0]
    full = O.softmax_strided(x.ravel(), 1, 0, rows, cols, pitch, 0, 1.0).reshape(rows, pitch)
    assert [p[0] for p in parts] == [0, parts[0][1]] and parts[-1][1] == rows
    assert np.array_equal(np.concatenate([p[2] for p in parts]), full)
    # Folded shards put back at their rows give the same matrix.
    fr, fc = 301, 320
    fp = cs.padded_pitch(fc)
    xf = cs.generate(3, 2, batch=1, rows=fr, cols=fc)[0]
    ffull = O.softmax_strided(xf.ravel(), 1, 0, fr, fc, fp, 0, 1.0).reshape(fr, fp)
    assembled = np.full_like(ffull, 0xFFFF)
    for r in range(world):
        o = 0
        for s0, n in bench.rank_segments(fr, fc, world, r):
            assembled[s0:s0 + n] = fparts[r][o:o + n]
            o += n
        assert o == len(fparts[r])
    assert len(bench.rank_segments(fr, fc, world, 0)) == 2  # rank 0's shard is folded
    assert np.array_equal(assembled, ffull)

    heads, hr = 6, 40
    hp = cs.padded_pitch(hr)
    xh = cs.generate(4, 3, batch=heads, rows=hr, cols=hr)
    fh = O.softmax_strided(xh.ravel(), heads, hr * hp, hr, hr, hp, 0, 0.0883883).reshape(heads, hr, hp)
    assert np.array_equal(np.concatenate(hparts), fh)


def test_row_blocks_balance_causal_cost():
    import bench

    for rows, cols, parts in [(4096, 4096, 2), (4096, 4096, 8), (32768, 32768, 8), (1000, 1037, 4),
                              (4096, 32, 8), (8, 100, 8), (9, 100, 8), (3, 3, 2)]:
        blocks = bench.row_blocks(rows, cols, parts)
        assert len(blocks) == parts and blocks[0][0] == 0 and blocks[-1][1] == rows
        assert all(b[0] < b[1] for b in blocks), (rows, cols, parts, blocks)  # no empty shard
        assert all(blocks[i][1] == blocks[i + 1][0] for i in range(parts - 1))
        cost = lambda a, b: sum(2 * min(r + 1, cols) + 2 * cols for r in range(a, b))
        costs = [cost(a, b) for a, b in blocks]
        row_cost = 2 * cols + 2 * min(rows, cols)
        if rows >= 8 * parts:
            assert max(costs) - min(costs) <= 2 * row_cost, (rows, cols, parts, costs)


def test_shards_never_empty_and_fold_falls_back():
    import bench

    # Fewer rows than ranks: a clear error instead of empty shards.
    with pytest.raises(ValueError, match="every rank needs a row"):
        bench.row_blocks(7, 100, 8)
    # Too few rows to give every rank a block and its mirror: contiguous blocks.
    for rows, cols, parts in [(8, 100, 8), (15, 100, 8), (3, 3, 2)]:
        assert not bench.can_fold(rows, cols, parts)
        segs = [bench.rank_segments(rows, cols, parts, r) for r in range(parts)]
        assert all(len(s) == 1 and s[0][1] > 0 for s in segs), segs
        assert sum(s[0][1] for s in segs) == rows
    # Enough rows: folded, every segment non-empty, all rows covered once.
    for rows, cols, parts in [(16, 100, 8), (4096, 4096, 8), (301, 320, 2), (32768, 32768, 8)]:
        assert bench.can_fold(rows, cols, parts)
        seen = np.zeros(rows, np.int32)
        for r in range(parts):
            for a, n in bench.rank_segments(rows, cols, parts, r):
                assert n > 0
                seen[a:a + n] += 1
        assert np.all(seen == 1)


def test_head_split_matches_job():
    import bench

    for heads, world in [(256, 1), (256, 2), (256, 4), (256, 8), (6, 4), (7, 3)]:
        ranges = [bench.head_range(heads, world, r) for r in range(world)]
        assert sum(n for _, n in ranges) == heads
        assert all(ranges[r][0] + ranges[r][1] == ranges[r + 1][0] for r in range(world - 1))
        assert max(n for _, n in ranges) - min(n for _, n in ranges) <= 1
    with pytest.raises(ValueError):
        bench.head_range(2, 4, 0)
    # The batched workload: strong scaling keeps the job at 256 heads, N = 1
    # is the whole batch, and --weak gives every rank its own 256.
    w = bench.WORKLOADS["c4"]
    for world in (1, 2, 4, 8):
        first, n, segs, scaling, job = bench.rank_share(w, world, world - 1, False, False)
        assert (scaling, job, n, first) == ("strong", 256, 256 // world, 256 - 256 // world)
        first, n, segs, scaling, job = bench.rank_share(w, world, world - 1, True, False)
        assert (scaling, job, n, first) == ("weak", 256 * world, 256, 256 * (world - 1))
