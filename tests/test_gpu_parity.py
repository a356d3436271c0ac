"""GPU parity tests: every kernel, called through the C ABI, against the CPU oracle.

Shapes and patterns follow the reference's hardware suites
(gpu/src/driver.rs:250-331: QUICK x {zeros, spikes, random} at scale 0.125, and
MORE x all seven patterns x scales {0, 0.125, 0.5, 1, 1e30}), plus the five
benchmark configurations and the row-block / batch layouts this library adds.
Outputs start filled with the 0xfb00 sentinel (gpu/src/driver.rs:78-79), so a
missing store shows up as a mask or element violation.

Tolerances (see gpu_helpers): masked == 0x0000 bit-exact; unmasked within
2 FP16 ulp or 2e-3 absolute of the FP64 oracle rounded to half; |row sum - 1|
<= 2e-3; and the reference verifier (0.003 + 0.003*w, row sum 0.02) accepts.
"""
import numpy as np
import pytest
import torch

import causal_softmax as cs
import oracle_ctypes as O
from gpu_helpers import (KERNELS, SENTINEL, check, from_dev, pattern_input, run, sentinel_like,
                         supported, to_dev)

pytestmark = pytest.mark.gpu

# gpu/src/driver.rs:250-265
QUICK = [(1, 1), (1, 8), (2, 17), (3, 31), (4, 32), (5, 33), (7, 64), (8, 127), (9, 256),
         (10, 257), (13, 513), (17, 1024), (33, 9), (64, 65)]
# gpu/src/driver.rs:266-285
MORE = [(1, 129), (2, 255), (3, 256), (4, 257), (5, 511), (6, 512), (7, 513), (8, 1025),
        (15, 2048), (16, 16), (31, 31), (32, 32), (33, 33), (64, 128), (65, 256), (127, 512),
        (129, 8192), (257, 257)]
STRESS_SCALES = [0.0, 0.125, 0.5, 1.0, 1.0e30]


@pytest.fixture(scope="module", autouse=True)
def device():
    import build

    build.build_library()
    assert torch.cuda.is_available()
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, "these kernels are built for sm_100a only"
    yield


@pytest.mark.parametrize("kernel", KERNELS)
def test_gpu_tests_quick(kernel):
    n = 0
    for rows, cols in QUICK:
        if not supported(kernel, cols):
            continue
        for pattern in ("zeros", "spikes", "random"):
            x = pattern_input(rows, cols, pattern)
            got = run(kernel, x, cols=cols, scale=0.125)
            check(got, x, cols=cols, scale=0.125, what=f"{kernel} {rows}x{cols} {pattern}")
            n += 1
    assert n > 0


@pytest.mark.parametrize("kernel", KERNELS)
def test_gpu_stress(kernel):
    for rows, cols in MORE:
        if not supported(kernel, cols):
            continue
        for pattern in cs.PATTERNS:
            x = pattern_input(rows, cols, pattern)
            for scale in STRESS_SCALES:
                got = run(kernel, x, cols=cols, scale=scale)
                check(got, x, cols=cols, scale=scale, what=f"{kernel} {rows}x{cols} {pattern} {scale}")


@pytest.mark.parametrize("kernel", ["baseline", "tma", "pipeline", "online"])
def test_tall_wide_and_ragged_shapes(kernel):
    # Rows past the diagonal (M > N), a single row, and widths straddling every
    # vector / warp / tile boundary of the kernels (8, 256, 512, 4096 columns).
    for rows, cols in [(300, 64), (1000, 40), (1, 4096), (2, 8191), (40, 4097), (513, 511),
                       (4100, 33), (97, 4104)]:
        x = cs.generate(2, 1, batch=1, rows=rows, cols=cols)[0]
        for scale in (0.0, 0.0883883, 1.0):
            got = run(kernel, x, cols=cols, scale=scale)
            check(got, x, cols=cols, scale=scale, what=f"{kernel} {rows}x{cols} {scale}")


def test_reference_online_model_shapes_all_kernels():
    # reference/src/online.rs:79-100 shapes and scales, every kernel.
    for rows, cols in [(1, 1), (7, 17), (9, 129), (65, 257), (137, 259), (257, 513)]:
        dense = np.array([O.h(((i * 7919 % 251) - 125.0) * 0.125) for i in range(rows * cols)],
                         np.uint16)
        x = O.pad(dense, rows, cols).reshape(rows, cs.padded_pitch(cols))
        for kernel in KERNELS:
            if not supported(kernel, cols):
                continue
            for scale in (0.0, 0.001, 0.125, 1.0, 10.0):
                got = run(kernel, x, cols=cols, scale=scale)
                check(got, x, cols=cols, scale=scale, what=f"{kernel} {rows}x{cols} {scale}")
                if scale == 0.0:
                    # Zero scale is an exact uniform distribution (online.rs:116-120).
                    g = got.reshape(rows, -1)
                    for r in range(rows):
                        v = min(r + 1, cols)
                        assert np.all(g[r, :v] == O.h(1.0 / v)), (kernel, r)


@pytest.mark.parametrize("kernel", ["baseline", "tma", "pipeline", "online"])
def test_config1_4096(kernel):
    x = cs.generate(1, 0, batch=1, rows=4096, cols=4096)[0]
    got = run(kernel, x, cols=4096, scale=1 / np.sqrt(128))
    rep = check(got, x, cols=4096, scale=float(np.float32(1 / np.sqrt(128))), what=f"C1 {kernel}")
    assert rep["max_ulp_vs_f32_spec"] <= 2


@pytest.mark.parametrize("kernel", KERNELS)
def test_config2_odd_and_narrow(kernel):
    for rows, cols, pitch in [(1000, 1037, 1040), (4096, 32, 32)]:
        if not supported(kernel, cols):
            continue
        x = cs.generate(2, 1, batch=1, rows=rows, cols=cols, pitch=pitch)[0]
        for scale in (0.0, 0.0883883, 1.0):
            got = run(kernel, x, cols=cols, scale=scale)
            check(got, x, cols=cols, scale=scale, what=f"C2 {kernel} {rows}x{cols} {scale}")
            assert np.all(got[:, cols:] == 0)  # padding written zero


@pytest.mark.parametrize("kernel", ["baseline", "tma", "pipeline", "online"])
def test_config3_8192_stress(kernel):
    x = cs.generate(3, 2, batch=1, rows=8192, cols=8192)[0]
    got = run(kernel, x, cols=8192, scale=1.0)
    check(got, x, cols=8192, scale=1.0, what=f"C3 {kernel}")


def gpu_structure(y: torch.Tensor, cols: int, row_offset: int = 0, chunk: int = 2048) -> dict:
    """Size-independent properties on the device: masked entries are 0x0000,
    valid ones finite and non-negative, |row sum - 1| <= 2e-3 (f64 sums)."""
    y3 = y if y.dim() == 3 else y.unsqueeze(0)
    batch, rows, pitch = y3.shape
    col = torch.arange(pitch, device=y.device)
    worst, bad_mask, bad_val = 0.0, 0, 0
    for b in range(batch):
        for r0 in range(0, rows, chunk):
            blk = y3[b, r0:r0 + chunk]
            n = blk.shape[0]
            valid = torch.clamp(torch.arange(r0, r0 + n, device=y.device) + row_offset + 1, max=cols)
            masked = col[None, :] >= valid[:, None]
            bits = blk.view(torch.int16)
            bad_mask += int(((bits != 0) & masked).sum())
            neg_or_inf = (bits < 0) | ((bits & 0x7C00) == 0x7C00)
            bad_val += int((neg_or_inf & ~masked).sum())
            sums = blk.double().sum(dim=1)
            worst = max(worst, float((sums - 1.0).abs().max()))
    return {"mask": bad_mask, "values": bad_val, "max_rowsum_err": worst}


def test_config4_batched_multihead():
    # 8 x 32 x 4096^2 = 256 matrices, 8 GiB in + 8 GiB out.
    free, _ = torch.cuda.mem_get_info()
    if free < 20 * 2**30:
        pytest.skip("needs 20 GiB of free device memory")
    batch, L = 256, 4096
    scale = float(np.float32(1 / np.sqrt(128)))
    x = torch.empty((batch, L, L), dtype=torch.int16)
    cs.generate(4, 3, batch=batch, rows=L, cols=L, out=x.numpy().view(np.uint16))
    d_in = x.cuda().view(torch.float16)
    d_out = sentinel_like(d_in)
    with cs.Plan.for_tensors(d_in, d_out, cols=L) as plan:
        plan.launch("auto", scale)
        assert plan.status() == (0, 0)
    rep = gpu_structure(d_out, L)
    assert rep["mask"] == 0 and rep["values"] == 0 and rep["max_rowsum_err"] <= 2e-3, rep
    # Full oracle check on 32 matrices spread over the batch (every 8th, from
    # both ends), and batch invariance on three of them (a single-matrix
    # launch gives the same bits as that matrix inside the batched launch).
    for b in sorted(set(range(0, batch, 8)) | {batch - 1}):
        xb = x[b].numpy().view(np.uint16)
        gb = from_dev(d_out[b])
        check(gb, xb, cols=L, scale=scale, what=f"C4 matrix {b}")
        if b in (0, 136, 255):
            assert np.array_equal(run("auto", xb, cols=L, scale=scale), gb)


def test_config5_long_context():
    L = 32768
    free, _ = torch.cuda.mem_get_info()
    if free < 8 * 2**30:
        pytest.skip("needs 8 GiB of free device memory")
    scale = float(np.float32(1 / np.sqrt(128)))
    x = cs.generate(5, 4, batch=1, rows=L, cols=L)[0]
    d_in = to_dev(x)
    for kernel in ("auto", "online"):
        d_out = sentinel_like(d_in)
        with cs.Plan.for_tensors(d_in, d_out, cols=L) as plan:
            plan.launch(kernel, scale)
            assert plan.status() == (0, 0)
        rep = gpu_structure(d_out, L)
        assert rep["mask"] == 0 and rep["values"] == 0 and rep["max_rowsum_err"] <= 2e-3, rep
        got = from_dev(d_out)
        # Every row against the FP64 oracle, in blocks of 2048 rows.
        for r0 in range(0, L, 2048):
            check(got[r0:r0 + 2048], x[r0:r0 + 2048], cols=L, scale=scale, row_offset=r0,
                  what=f"C5 {kernel} rows {r0}+2048")
        del d_out
        torch.cuda.empty_cache()


@pytest.mark.parametrize("kernel", ["baseline", "tma", "pipeline", "online"])
def test_row_block_shards_match_full_matrix(kernel):
    # Row blocks launched with their absolute row offset reproduce the full
    # matrix (the multi-GPU sharding contract): each block passes the oracle
    # check on its absolute rows, and agrees with the full launch within one
    # FP16 ulp. Kernels whose per-row work split does not depend on the launch
    # geometry (baseline, online) agree bit for bit; the row-resident kernel
    # pairs rows per launch, which can move a row sum's last f32 bit.
    rows = cols = 4096
    scale = float(np.float32(1 / np.sqrt(128)))
    x = cs.generate(1, 0, batch=1, rows=rows, cols=cols)[0]
    full = run(kernel, x, cols=cols, scale=scale)
    for a, b in [(0, 1000), (1000, 2501), (2501, 4096)]:
        part = run(kernel, x[a:b], cols=cols, scale=scale, row_offset=a)
        check(part, x[a:b], cols=cols, scale=scale, row_offset=a, what=f"{kernel} rows {a}:{b}")
        diff = np.abs(part.astype(np.int32) - full[a:b].astype(np.int32))
        assert diff.max() <= 1, (kernel, a, b)
        if kernel in ("baseline", "online"):
            assert diff.max() == 0, (kernel, a, b)


def run_folded(kernel: str, x: np.ndarray, segs, *, cols: int, scale: float, tuning=None) -> np.ndarray:
    """One launch over a folded shard: x holds the segments' rows one after
    the other; the plan maps them with row_offset and cs_plan_set_row_split."""
    d_in = to_dev(x)
    d_out = sentinel_like(d_in)
    with cs.Plan.for_tensors(d_in, d_out, cols=cols, row_offset=segs[0][0]) as plan:
        if len(segs) > 1:
            plan.set_row_split(segs[0][1], segs[1][0])
        if tuning:
            plan.set_tuning(*tuning)
        plan.launch(kernel, scale)
        rc, status = plan.status()
        assert rc == 0 and status == 0, (rc, status)
    torch.cuda.synchronize()
    return from_dev(d_out)


FOLD_CASES = [(4096, 4096, 4), (1001, 1001, 3), (300, 20000, 2), (4096, 4096, 8)]


@pytest.mark.parametrize("kernel", ["baseline", "tma", "pipeline", "online", "auto"])
def test_folded_shards_match_full_matrix(kernel):
    # A rank's folded shard (row block [a, b) and its mirror, stored one after
    # the other) reproduces those rows of the full launch: each segment passes
    # the oracle check on its absolute rows and agrees with the full matrix
    # within one FP16 ulp (bit for bit for the kernels whose per-row work does
    # not depend on how rows are grouped into units).
    import bench

    for rows, cols, parts in FOLD_CASES:
        scale = float(np.float32(1 / np.sqrt(128)))
        x = cs.generate(1, 0, batch=1, rows=rows, cols=cols)[0]
        full = run(kernel, x, cols=cols, scale=scale)
        for r in range(parts):
            segs = bench.rank_segments(rows, cols, parts, r)
            xl = np.concatenate([x[a:a + n] for a, n in segs])
            got = run_folded(kernel, xl, segs, cols=cols, scale=scale)
            o = 0
            for a, n in segs:
                what = f"{kernel} {rows}x{cols} rank {r}/{parts} rows {a}:{a + n}"
                check(got[o:o + n], x[a:a + n], cols=cols, scale=scale, row_offset=a, what=what)
                diff = np.abs(got[o:o + n].astype(np.int32) - full[a:a + n].astype(np.int32))
                assert diff.max() <= (0 if kernel in ("baseline", "online") else 1), what
                o += n


@pytest.mark.parametrize("variant", range(8))
def test_folded_shards_every_row_resident_variant(variant):
    import bench

    for rows, cols, parts in [(2000, 2000, 4), (300, 20000, 2)]:
        x = cs.generate(2, 5, batch=1, rows=rows, cols=cols)[0]
        for r in range(parts):
            segs = bench.rank_segments(rows, cols, parts, r)
            xl = np.concatenate([x[a:a + n] for a, n in segs])
            try:
                got = run_folded("pipeline", xl, segs, cols=cols, scale=0.0883883,
                                 tuning=(16 + variant, 0, -1, -1))
            except cs.CausalSoftmaxError as e:
                assert e.code == cs.ERR_CODE["UNSUPPORTED"] and variant != 7, e
                continue
            o = 0
            for a, n in segs:
                check(got[o:o + n], x[a:a + n], cols=cols, scale=0.0883883, row_offset=a,
                      what=f"variant {variant} {rows}x{cols} rank {r} rows {a}:{a + n}")
                o += n


def test_folded_narrow_rows_and_split_errors():
    import bench

    # The warp path (cols <= 32) under a fold.
    x = cs.generate(2, 1, batch=1, rows=32, cols=32)[0]
    for r in range(2):
        segs = bench.rank_segments(32, 32, 2, r)
        xl = np.concatenate([x[a:a + n] for a, n in segs])
        for kernel in ("warp", "auto"):
            got = run_folded(kernel, xl, segs, cols=32, scale=0.5)
            o = 0
            for a, n in segs:
                check(got[o:o + n], x[a:a + n], cols=32, scale=0.5, row_offset=a, what=f"{kernel} rank {r}")
                o += n
    # Argument checks of cs_plan_set_row_split.
    E = cs.ERR_CODE
    d_in = torch.zeros((64, 64), dtype=torch.float16, device="cuda")
    d_out = torch.zeros_like(d_in)
    L = cs.lib()
    with cs.Plan.for_tensors(d_in, d_out, cols=64, row_offset=10) as plan:
        h = plan._h
        assert L.cs_plan_set_row_split(h, 64, 200) == E["ARG"]   # no rows left for the second block
        assert L.cs_plan_set_row_split(h, -1, 200) == E["ARG"]
        assert L.cs_plan_set_row_split(h, 16, 25) == E["ARG"]    # overlaps the first block (ends at 26)
        assert L.cs_plan_set_row_split(h, 16, 2**31 - 40) == E["ARG"]  # past 32-bit rows
        assert L.cs_plan_set_row_split(None, 16, 26) == E["NULL"]
        assert L.cs_plan_set_row_split(h, 16, 26) == 0           # contiguous: same as no split
        assert L.cs_plan_set_row_split(h, 0, 0) == 0             # back to one block


def test_deterministic_and_kernels_agree():
    rows, cols = 777, 1500
    x = cs.generate(2, 1, batch=1, rows=rows, cols=cols)[0]
    outs = {}
    for k in ("baseline", "tma", "pipeline", "online"):
        a = run(k, x, cols=cols, scale=1.0)
        assert np.array_equal(a, run(k, x, cols=cols, scale=1.0)), k
        outs[k] = a
    # Same causal math in every kernel: outputs within 1 FP16 ulp of each other.
    base = outs["tma"].astype(np.int32)
    for k, v in outs.items():
        assert np.max(np.abs(v.astype(np.int32) - base)) <= 1, k
    assert np.array_equal(outs["tma"], outs["pipeline"])


@pytest.mark.parametrize("tuning", [(2, 2, 0, 0), (2, 4, 1, 1), (4, 3, 1, 0), (4, 2, 0, 1),
                                    (8, 2, 0, 1), (8, 3, 1, 0), (8, 4, 1, 1)])
def test_row_resident_tuning_variants(tuning):
    for rows, cols in [(4096, 4096), (300, 2000), (1000, 40)]:
        x = cs.generate(1, 0, batch=1, rows=rows, cols=cols)[0]
        for kernel in ("tma", "pipeline"):
            got = run(kernel, x, cols=cols, scale=0.125, tuning=tuning)
            check(got, x, cols=cols, scale=0.125, what=f"{kernel} {tuning} {rows}x{cols}")


@pytest.mark.parametrize("variant", range(8))
def test_every_compiled_row_resident_variant(variant):
    # Tuning vec 16 + i forces compiled variant i (V and register budget;
    # variant 7 keeps rows in shared memory).
    for rows, cols in [(2000, 2000), (6000, 6001), (300, 20000)]:
        x = cs.generate(2, 5, batch=1, rows=rows, cols=cols)[0]
        for kernel in ("tma", "pipeline"):
            try:
                got = run(kernel, x, cols=cols, scale=0.0883883, tuning=(16 + variant, 0, -1, -1))
            except cs.CausalSoftmaxError as e:
                # Register-resident variants have a widest unit; variant 7 has none here.
                assert e.code == cs.ERR_CODE["UNSUPPORTED"] and variant != 7, e
                continue
            check(got, x, cols=cols, scale=0.0883883, what=f"{kernel} variant {variant} {rows}x{cols}")


@pytest.mark.parametrize("cols", [2048, 20000])
def test_repeated_launches_are_fast_and_exact(cols):
    # 100 back-to-back launches of one plan finish quickly (no launch waits
    # out a bounded wait; the dynamic schedule's counters are reset by every
    # launch), and the last output is still exact. 20000 columns select the
    # shared-memory variant, which claims its units dynamically.
    rows = 2048 if cols == 2048 else 600
    x = cs.generate(1, 7, batch=1, rows=rows, cols=cols)[0]
    d_in = to_dev(x)
    for kernel in ("tma", "pipeline"):
        d_out = sentinel_like(d_in)
        with cs.Plan.for_tensors(d_in, d_out, cols=cols) as plan:
            plan.launch(kernel, 0.125)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(100):
                plan.launch(kernel, 0.125)
            b.record()
            torch.cuda.synchronize()
            assert plan.status() == (0, 0)
            assert a.elapsed_time(b) < 500.0, (kernel, a.elapsed_time(b))
        check(from_dev(d_out), x, cols=cols, scale=0.125, what=f"repeated {kernel} {rows}x{cols}")


@pytest.mark.parametrize("variant", [None, 1, 5, 6, 7])
def test_l2_prefetch_depth_changes_no_bit(variant):
    # The row-resident kernel pulls the rows of each CTA's first units into
    # L2 before it waits for the previous kernel: whatever the depth, the
    # launch reads its inputs after that wait, so the output bits are those
    # of the shallowest prefetch, for consecutive launches of one plan whose
    # input the previous kernel in the stream has just rewritten.
    for rows, cols, batch, off in [(4096, 4096, 1, 0), (700, 700, 3, 0), (301, 5000, 2, 4000)]:
        x = cs.generate(2, 9, batch=batch, rows=rows, cols=cols, first_row=off)
        d_in = to_dev(x)
        outs = []
        for depth in (0, 3, 4, 64):
            d_out = sentinel_like(d_in)
            with cs.Plan.for_tensors(d_in, d_out, cols=cols, row_offset=off) as plan:
                if variant is not None:
                    try:
                        plan.set_tuning(16 + variant, 0, -1, -1)
                        plan.describe("pipeline")
                    except cs.CausalSoftmaxError as e:
                        assert e.code == cs.ERR_CODE["UNSUPPORTED"], e
                        break
                plan.set_prefetch(depth)
                for _ in range(2):
                    d_in.view(torch.int16).bitwise_not_()  # the input changes right before the launch
                    plan.launch("pipeline", 0.0883883)
                assert plan.status() == (0, 0)
            outs.append(from_dev(d_out))
        if not outs:
            continue
        what = f"variant {variant} {batch}x{rows}x{cols}+{off}"
        for b in range(batch):
            check(outs[0][b], x[b], cols=cols, scale=0.0883883, row_offset=off, what=what)
        for o in outs[1:]:
            assert np.array_equal(o, outs[0]), what


def test_chained_launches_read_the_previous_output():
    # Launch B reads what launch A (just before it on the stream) writes.
    # B starts while A finishes (programmatic dependent launch) and prefetches
    # its input rows into L2 before it waits for A; its loads come after the
    # wait, so B must see A's final output: softmax applied twice, with the
    # same bits as two launches separated by a device synchronisation.
    for rows, cols, kernel, tuning in [(4096, 4096, "pipeline", None), (2048, 2048, "tma", None),
                                       (1000, 1037, "pipeline", (23, 0, -1, -1)), (600, 20000, "auto", None)]:
        pitch = cs.padded_pitch(cols)
        x = cs.generate(1, 12, batch=1, rows=rows, cols=cols, pitch=pitch)[0]
        d_in = to_dev(x)
        mids = [sentinel_like(d_in) for _ in range(2)]
        outs = [sentinel_like(d_in) for _ in range(2)]
        for i, chained in enumerate((True, False)):
            with cs.Plan.for_tensors(d_in, mids[i], cols=cols) as a, \
                    cs.Plan.for_tensors(mids[i], outs[i], cols=cols) as b:
                for p in (a, b):
                    if tuning:
                        p.set_tuning(*tuning)
                    p.set_prefetch(64)
                for _ in range(3):
                    a.launch(kernel, 0.5)
                    if not chained:
                        torch.cuda.synchronize()
                    b.launch(kernel, 0.5)
                    if not chained:
                        torch.cuda.synchronize()
                assert a.status() == (0, 0) and b.status() == (0, 0)
        got, want = from_dev(outs[0]), from_dev(outs[1])
        assert np.array_equal(got, want), (rows, cols, kernel, int(np.count_nonzero(got != want)))
        check(from_dev(mids[0]), x, cols=cols, scale=0.5, what=f"chained first pass {rows}x{cols}")


def test_prefetch_arguments():
    E = cs.ERR_CODE
    d_in = torch.zeros((64, 64), dtype=torch.float16, device="cuda")
    d_out = torch.zeros_like(d_in)
    L = cs.lib()
    with cs.Plan.for_tensors(d_in, d_out, cols=64) as plan:
        assert L.cs_plan_set_prefetch(plan._h, -2) == E["ARG"]
        assert L.cs_plan_set_prefetch(plan._h, 1025) == E["ARG"]
        assert L.cs_plan_set_prefetch(None, 1) == E["NULL"]
        assert L.cs_plan_set_prefetch(plan._h, -1) == 0
        assert L.cs_plan_set_prefetch(plan._h, 1024) == 0


def test_unpaired_fallback_when_a_pair_does_not_fit():
    # Forcing 2 vectors per thread caps a unit at 30 warps x 64 vectors: row
    # pairs of ~24000 columns do not fit, single rows (~1500 vectors) do, so
    # the planner drops pairing.
    rows, cols, off = 40, 12288, 12000
    x = cs.generate(5, 4, batch=1, rows=rows, cols=cols, first_row=off)[0]
    d_in = to_dev(x)
    d_out = sentinel_like(d_in)
    with cs.Plan.for_tensors(d_in, d_out, cols=cols, row_offset=off) as plan:
        plan.set_tuning(2, 0, -1, -1)
        info = plan.describe("tma")
        assert info["vec_per_thread"] == 2 and info["units"] == rows  # one unit per row
        for kernel in ("tma", "pipeline"):
            plan.launch(kernel, 0.0883883)
            assert plan.status() == (0, 0)
            check(from_dev(d_out), x, cols=cols, scale=0.0883883, row_offset=off, what=kernel)


def test_online_very_long_rows():
    # Rows far beyond the row-resident kernel (which holds a pair of up to
    # ~56K columns): one 100000-column row, and 64 rows of ~70000 columns in
    # a batch of two, with the automatic ring (the whole row resident in
    # shared memory) and with rings too short for it (two fetches per row).
    for rows, cols, off, batch in [(1, 100000, 99999, 1), (64, 70000, 69936, 2)]:
        x = cs.generate(5, 4, batch=batch, rows=rows, cols=cols, first_row=off)
        # Automatic; 8 KB tiles, two fetches or the row resident; the
        # 1024-thread shape with 16 KB tiles, resident and two fetches.
        for tuning in (None, (0, 4, -1, -1), (0, 27, -1, -1), (1, 13, -1, -1), (1, 4, -1, -1)):
            got = run("online", x if batch > 1 else x[0], cols=cols, scale=0.0883883, row_offset=off,
                      tuning=tuning)
            g = got.reshape(batch, rows, -1)
            for b in range(batch):
                check(g[b], x[b], cols=cols, scale=0.0883883, row_offset=off,
                      what=f"online {batch}x{rows}x{cols}+{off} tuning {tuning}")
        assert cs.resolve_kernel("auto", off + rows, cols) == "online" or cols <= 56000


@pytest.mark.parametrize("stages", [0, 3])
def test_cluster_resident_online_kernel(stages):
    # Tuning vec 3 runs `online` on the cluster kernel: each row dealt in 2 KB
    # blocks over the 2, 4 or 8 CTAs of a thread-block cluster, the partial
    # (max, sum) exchanged through distributed shared memory. Cluster sizes
    # 2/4/8 (row widths of up to 48, 96 and 192 blocks), odd pitch, batches,
    # row offsets, zero scale, rows shorter than one block of some CTAs.
    cases = [(300, 4096, 0, 1, 0.0883883), (64, 12000, 20000, 2, 1.0), (1000, 1037, 0, 1, 0.0883883),
             (33, 100000, 99967, 1, 0.0883883), (700, 700, 0, 3, 0.5), (40, 20000, 0, 1, 0.0),
             (16, 70000, 69984, 2, 0.125)]
    for rows, cols, off, batch, scale in cases:
        x = cs.generate(5, 4, batch=batch, rows=rows, cols=cols, first_row=off)
        got = run("online", x if batch > 1 else x[0], cols=cols, scale=scale, row_offset=off,
                  tuning=(3, stages, -1, -1))
        g = got.reshape(batch, rows, -1)
        for b in range(batch):
            check(g[b], x[b], cols=cols, scale=scale, row_offset=off,
                  what=f"cluster online {batch}x{rows}x{cols}+{off} scale {scale} S={stages}")
    # The launch is a cluster launch of the online kernel.
    d_in = to_dev(cs.generate(5, 4, batch=1, rows=8, cols=100000, first_row=99992)[0])
    d_out = sentinel_like(d_in)
    with cs.Plan.for_tensors(d_in, d_out, cols=100000, row_offset=99992) as plan:
        plan.set_tuning(3, stages, -1, -1)
        info = plan.describe("online")
        assert info["kernel_name"] == "online" and info["vec_per_thread"] == 3
        assert info["grid"] % 8 == 0  # 98 blocks per row: clusters of 8


def test_online_ring_depths_and_long_rows():
    # Rows longer than the ring take the two-fetch path.
    for stages in (2, 3, 8, 16):
        for rows, cols in [(40, 20000), (3, 70000), (600, 4100)]:
            x = cs.generate(5, 4, batch=1, rows=rows, cols=cols)[0]
            got = run("online", x, cols=cols, scale=0.0883883, tuning=(0, stages, -1, -1))
            check(got, x, cols=cols, scale=0.0883883, what=f"online S={stages} {rows}x{cols}")
            # The same rows as the tail of a taller matrix (row offset).
            got = run("online", x, cols=cols, scale=0.0883883, row_offset=5000,
                      tuning=(0, stages, -1, -1))
            check(got, x, cols=cols, scale=0.0883883, row_offset=5000, what=f"online offset S={stages}")


def test_batched_layout_with_gaps():
    # batch_stride larger than rows * pitch (a view into a bigger buffer).
    batch, rows, cols = 5, 100, 203
    pitch = cs.padded_pitch(cols)
    gap = 8 * 7
    stride = rows * pitch + gap
    flat = np.zeros(batch * stride, np.uint16)
    x = cs.generate(2, 1, batch=batch, rows=rows, cols=cols)
    for b in range(batch):
        flat[b * stride:b * stride + rows * pitch] = x[b].ravel()
    d_in = to_dev(flat)
    d_out = sentinel_like(d_in)
    for kernel in ("baseline", "tma", "pipeline", "online"):
        d_out.view(torch.int16).fill_(int(np.uint16(SENTINEL).view(np.int16)))
        with cs.Plan(d_in.data_ptr(), d_out.data_ptr(), rows=rows, cols=cols, pitch=pitch,
                     batch=batch, batch_stride=stride) as plan:
            plan.launch(kernel, 0.7)
            assert plan.status() == (0, 0)
        got = from_dev(d_out)
        for b in range(batch):
            blk = got[b * stride:b * stride + rows * pitch].reshape(rows, pitch)
            check(blk, x[b], cols=cols, scale=0.7, what=f"gaps {kernel} {b}")
            if b + 1 < batch:  # the gap between matrices is untouched
                assert np.all(got[b * stride + rows * pitch:(b + 1) * stride] == SENTINEL)


def test_one_shot_entry_points_match_plans():
    rows, cols = 513, 700
    pitch = cs.padded_pitch(cols)
    x = cs.generate(1, 0, batch=2, rows=rows, cols=cols)
    d_in = to_dev(x)
    y = cs.softmax(d_in, cols=cols, scale=0.3)
    torch.cuda.synchronize()
    got = from_dev(y)
    for b in range(2):
        assert np.array_equal(got[b], run("auto", x[b], cols=cols, scale=0.3))
    y1 = torch.empty_like(d_in[0])
    rc = cs.lib().cs_softmax(cs.TMA, d_in[0].data_ptr(), y1.data_ptr(), rows, cols, pitch, 0.3,
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert np.array_equal(from_dev(y1), got[0])


def test_session_paths():
    with cs.Session(0) as s:
        s.probe()  # gpu/src/driver.rs:44-59
        # prepare / launch / result with the sentinel and padding check.
        rows, cols = 123, 77
        dense = cs.make_input(rows, cols, "random", 0x13579BDF)
        out = np.zeros_like(dense)
        for kernel in ("baseline", "tma", "pipeline", "online"):
            s.prepare(dense, rows, cols)
            s.launch(kernel, 0.125)
            s.result(out)
            want = O.causal_softmax(dense, rows, cols, 0.125)[1]
            name, acc = O.verify(out, want, rows, cols)
            assert name == "ok", (kernel, name, acc.index)
        # End to end from host buffers: equals the device path bit for bit,
        # including the masked tails the host threads zero (the output starts
        # as the 0xfb00 sentinel), for whole matrices and row blocks.
        for batch, rows, cols, off in [(7, 300, 301, 0), (3, 700, 1037, 0), (2, 500, 600, 350),
                                       (1, 40, 20, 100), (4, 600, 32, 0), (1, 3000, 3001, 7)]:
            xin = cs.generate(4, 3, batch=batch, rows=rows, cols=cols, pitch=cols, first_row=off)
            hout = np.full_like(xin, SENTINEL)
            s.softmax_host(xin.ravel(), hout.reshape(-1), batch=batch, rows=rows, cols=cols, scale=0.2,
                           row_offset=off)
            for b in range(batch):
                dev = run("auto", O.pad(xin[b].ravel(), rows, cols).reshape(rows, -1), cols=cols,
                          scale=0.2, row_offset=off)
                assert np.array_equal(O.unpad(dev.ravel(), rows, cols), hout[b].ravel()), (rows, cols, off, b)


@pytest.mark.parametrize("kernel,tuning", [("tma", None), ("pipeline", None), ("online", None),
                                           ("tma", (23, 0, -1, -1)), ("pipeline", (23, 0, -1, -1)),
                                           ("online", (3, 0, -1, -1))])
def test_bounded_wait_reports_timeout_and_context_survives(kernel, tuning):
    # The producer issues no copies, so every consumer wait must run out after
    # 1 ms; the kernel returns, the host reads CS_ERR_TIMEOUT, and the next
    # normal launch on the same context is correct. Tuning 23 selects the
    # row-resident variant whose rows stay in shared memory.
    rows, cols = 64, 300
    x = cs.generate(2, 1, batch=1, rows=rows, cols=cols)[0]
    d_in = to_dev(x)
    d_out = sentinel_like(d_in)
    with cs.Plan.for_tensors(d_in, d_out, cols=cols) as plan:
        if tuning:
            plan.set_tuning(*tuning)
        plan.launch_debug(kernel, 1.0, cs.DEBUG_SKIP_LOADS, 1_000_000)
        rc, status = plan.status()
        assert rc == cs.ERR_CODE["TIMEOUT"] and status & cs.STATUS_TIMEOUT
        plan.launch(kernel, 1.0)
        assert plan.status() == (0, 0)
    check(from_dev(d_out), x, cols=cols, scale=1.0, what=f"after timeout {kernel}")


def test_argument_errors():
    E = cs.ERR_CODE
    x = torch.zeros((64, 64), dtype=torch.float16, device="cuda")
    y = torch.zeros_like(x)
    L = cs.lib()
    st = torch.cuda.current_stream().cuda_stream
    assert L.cs_softmax(cs.WARP, x.data_ptr(), y.data_ptr(), 64, 33, 64, 1.0, st) == E["WARP_COLS"]
    assert L.cs_softmax(cs.TMA, x.data_ptr() + 2, y.data_ptr(), 8, 8, 8, 1.0, st) == E["ALIGNMENT"]
    assert L.cs_softmax(cs.TMA, x.data_ptr(), x.data_ptr(), 8, 8, 8, 1.0, st) == E["ARG"]
    assert L.cs_softmax(cs.TMA, x.data_ptr(), y.data_ptr(), 8, 8, 8, -1.0, st) == E["BAD_SCALE"]
    assert L.cs_softmax(cs.TMA, x.data_ptr(), y.data_ptr(), 8, 9, 12, 1.0, st) == E["PITCH"]
    assert L.cs_softmax(cs.TMA, None, y.data_ptr(), 8, 8, 8, 1.0, st) == E["NULL"]
    assert L.cs_softmax(9, x.data_ptr(), y.data_ptr(), 8, 8, 8, 1.0, st) == E["BAD_KERNEL"]
    assert L.cs_softmax(cs.TMA, x.data_ptr(), y.data_ptr(), 0, 8, 8, 1.0, st) == E["EMPTY"]
    torch.cuda.synchronize()
