"""CPU tests of the C-ABI library: it loads, exports every declared symbol, and
its GPU-independent host surface matches the reference host crate.

Each host test restates a test of host/src/lib.rs:409-584 (cited) against the
C++ mirror exported by libcausal_softmax.so. No kernel is launched here.
"""
import ctypes
import math
import os
import re

import numpy as np
import pytest

import causal_softmax as cs
import oracle_ctypes as O
import patterns_ref


@pytest.fixture(scope="module", autouse=True)
def built():
    import build

    build.build_library()
    yield


def declared_functions() -> set[str]:
    names = set()
    for path in cs.HEADER_PATHS:
        text = open(path).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(cs_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(cs.LIB_PATH)
    missing = [n for n in sorted(declared_functions()) if not hasattr(L, n)]
    assert not missing, missing
    assert len(declared_functions()) >= 40
    assert cs.lib().cs_abi_version() == 1


def test_strerror_and_kernel_names():
    L = cs.lib()
    for code in list(cs.ERR) + [0]:
        assert L.cs_strerror(code)
    assert L.cs_strerror(-5).decode() == "warp specialization requires cols<=32"
    # host/src/lib.rs:22-42
    for name, k in cs.KERNELS.items():
        assert L.cs_kernel_name(k).decode() == name
        assert L.cs_kernel_parse(name.encode()) == k
    assert L.cs_kernel_parse(b"wrong") == cs.ERR_CODE["BAD_KERNEL"]
    assert L.cs_kernel_name(99) is None


def test_status_word_mapping():
    # Every status read (plan, session, no-alloc) maps the device word through
    # cs_status_error: kernels only ever set the timeout bit; any other bit is
    # reserved and reported as CS_ERR_STATUS rather than silently ignored.
    L = cs.lib()
    E = cs.ERR_CODE
    assert L.cs_status_error(0) == cs.OK
    assert L.cs_status_error(cs.STATUS_TIMEOUT) == E["TIMEOUT"]
    assert L.cs_status_error(cs.STATUS_TIMEOUT | 0x80000000) == E["TIMEOUT"]
    for word in (2, 4, 0x100, 0x80000000, 0xFFFFFFFE):
        assert L.cs_status_error(word) == E["STATUS"], hex(word)
        assert b"reserved bits" in L.cs_last_error_detail()
    assert L.cs_strerror(E["STATUS"]).decode() == "device status word holds reserved bits"
    # No header bit besides the timeout: the library defines no other status.
    text = open(cs.HEADER_PATHS[0]).read()
    assert re.findall(r"#define (CS_STATUS_\w+)", text) == ["CS_STATUS_TIMEOUT"]


def test_supports_and_auto_dispatch():
    L = cs.lib()
    # host/src/lib.rs:43-45, 461-470
    assert L.cs_kernel_supports(cs.WARP, 32) == 1
    assert L.cs_kernel_supports(cs.WARP, 33) == 0
    for k in (cs.BASELINE, cs.TMA, cs.PIPELINE, cs.ONLINE):
        assert L.cs_kernel_supports(k, 1 << 20) == 1
    # host/src/lib.rs:169-177 (warp for cols <= 32), then this library's choice.
    assert cs.resolve_kernel("auto", 4096, 31) == "warp"
    assert cs.resolve_kernel("auto", 4096, 32) == "warp"
    assert cs.resolve_kernel("auto", 4096, 4096) == "pipeline"
    assert cs.resolve_kernel("auto", 32768, 32768) == "pipeline"
    assert cs.resolve_kernel("auto", 8, 1 << 20) == "pipeline"  # only 8 causal columns per row
    assert cs.resolve_kernel("auto", 70000, 70000) == "online"
    assert cs.resolve_kernel("baseline", 4, 4) == "baseline"


def test_byte_models():
    L = cs.lib()
    # host/src/lib.rs:472-487: causal counts (4,4)->10, (2,4)->3, (4,2)->7.
    for rows, cols, eligible in [(4, 4, 10.0), (2, 4, 3.0), (4, 2, 7.0)]:
        full = float(rows * cols)
        assert L.cs_roofline_bytes(rows, cols, 0) == 2 * eligible + 2 * full
        assert L.cs_logical_bytes(cs.BASELINE, rows, cols) == 6 * eligible + 2 * full
        for k in (cs.WARP, cs.TMA, cs.PIPELINE, cs.ONLINE):
            assert L.cs_logical_bytes(k, rows, cols) == 2 * eligible + 2 * full
    assert L.cs_logical_bytes(cs.AUTO, 4, 4) < 0
    # Benchmark shapes (triangle read + full write).
    assert L.cs_roofline_bytes(4096, 4096, 0) == 50_335_744
    assert L.cs_roofline_bytes(8192, 8192, 0) == 201_334_784
    assert L.cs_roofline_bytes(32768, 32768, 0) == 3_221_258_240
    assert L.cs_roofline_bytes(1000, 1037, 0) == 3_075_000 - 2 * 0  # 500500*2 + 2074000
    # Row-block shards add up to the whole matrix.
    total = sum(L.cs_roofline_bytes(b - a, 4096, a) for a, b in [(0, 1000), (1000, 3000), (3000, 4096)])
    assert total == L.cs_roofline_bytes(4096, 4096, 0)
    # Long rows beyond half the online ring are read twice.
    assert L.cs_logical_bytes(cs.ONLINE, 1 << 16, 1 << 16) > L.cs_roofline_bytes(1 << 16, 1 << 16, 0)


def test_validate_mirrors_reference_errors():
    L = cs.lib()
    E = cs.ERR_CODE
    assert L.cs_validate(1, 0, 4, 4, 8, 0, 0.125) == 0
    assert L.cs_validate(1, 0, 0, 4, 8, 0, 0.125) == E["EMPTY"]
    assert L.cs_validate(0, 0, 4, 4, 8, 0, 0.125) == E["EMPTY"]
    assert L.cs_validate(1, 0, 4, 4, 8, 0, -0.1) == E["BAD_SCALE"]
    assert L.cs_validate(1, 0, 4, 4, 8, 0, 1e31) == E["BAD_SCALE"]
    assert L.cs_validate(1, 0, 4, 4, 8, 0, float("nan")) == E["BAD_SCALE"]
    assert L.cs_validate(1, 0, 4, 4, 8, 0, 1e30) == 0
    assert L.cs_validate(1, 0, 4, 4, 8, 0, 0.0) == 0
    assert L.cs_validate(1, 0, 4, 9, 12, 0, 1.0) == E["PITCH"]  # not a multiple of 8
    assert L.cs_validate(1, 0, 4, 9, 8, 0, 1.0) == E["PITCH"]   # pitch < cols
    assert L.cs_validate(2, 31, 4, 8, 8, 0, 1.0) == E["WRONG_LENGTH"]  # stride < rows*pitch
    assert L.cs_validate(1, 0, 2**31, 8, 8, 0, 1.0) == E["WRONG_LENGTH"]
    assert L.cs_validate(1, 0, 8, 8, 8, 2**31 - 4, 1.0) == E["WRONG_LENGTH"]
    bad = np.array([0x3C00, 0x7E00], np.uint16)
    good = np.array([0x3C00, 0x0001], np.uint16)
    u16 = ctypes.POINTER(ctypes.c_uint16)
    assert L.cs_check_finite_host(bad.ctypes.data_as(u16), 2) == E["NON_FINITE"]
    assert L.cs_check_finite_host(good.ctypes.data_as(u16), 2) == 0
    assert L.cs_padded_pitch(1037) == 1040 and L.cs_padded_pitch(8) == 8


def test_half_conversions_match_oracle():
    L = cs.lib()
    for bits in range(0, 0x10000, 3):
        if bits & 0x7C00 == 0x7C00 and bits & 0x3FF:
            continue
        f = L.cs_half_to_f32(bits)
        assert L.cs_f32_to_half(f) == bits
    rng = np.random.default_rng(3)
    for x in np.concatenate([rng.normal(0, 1e4, 2000), rng.normal(0, 1e-5, 2000)]).astype(np.float32):
        assert L.cs_f32_to_half(float(x)) == O.h(float(x))


@pytest.mark.parametrize("pattern", patterns_ref.PATTERNS)
def test_make_input_matches_reference_generator(pattern):
    # host/src/lib.rs:218-256, restated independently in tests/patterns_ref.py
    for rows, cols, seed in [(9, 37, 17), (3, 9, 2), (5, 33, 0x13579BDF)]:
        got = cs.make_input(rows, cols, pattern, seed)
        assert np.array_equal(got, patterns_ref.make_input(rows, cols, pattern, seed)), (rows, cols)


def test_patterns_finite_and_seeded():
    # host/src/lib.rs:488-501
    for p in cs.PATTERNS:
        v = cs.make_input(9, 37, p, 17)
        assert v.size == 333
        assert all(math.isfinite(O.f(b)) for b in v)
    a = cs.make_input(3, 9, "random", 2)
    assert np.array_equal(a, cs.make_input(3, 9, "random", 2))
    assert not np.array_equal(a, cs.make_input(3, 9, "random", 3))


def test_verify_mirrors_reference():
    # host/src/lib.rs:502-529, 555-558, against the product verifier
    L = cs.lib()
    u16 = ctypes.POINTER(ctypes.c_uint16)

    def verify(got, exp, rows, cols, lens=None):
        acc = cs.Accuracy()
        g = np.ascontiguousarray(got, np.uint16)
        e = np.ascontiguousarray(exp, np.uint16)
        lg, le = (g.size, e.size) if lens is None else lens
        rc = L.cs_verify(g.ctypes.data_as(u16), lg, e.ctypes.data_as(u16), le, rows, cols,
                         ctypes.byref(acc))
        return rc, acc

    zeros = np.array([O.h(0.0)] * 16, np.uint16)
    y = O.causal_softmax(zeros, 4, 4, 1.0)[1]
    assert verify(y, y, 4, 4)[0] == 0
    ones = np.array([O.h(1.0)] * 9, np.uint16)
    assert verify(ones, ones, 3, 3)[0] == 4  # Mask
    rc, acc = verify([0x7C00], [0x7C00], 1, 1)
    assert rc == 2 and acc.index == 0  # NonFinite(0)
    rc, acc = verify([O.h(-0.0005)], [O.h(0.0)], 1, 1)
    assert rc == 3 and acc.index == 0  # Negative(0)
    assert verify([], [], 2**64 - 1, 2)[0] == 1  # Length
    # Same decisions as the oracle's restatement on random perturbations.
    rng = np.random.default_rng(1)
    x = np.array([O.h(v) for v in rng.normal(0, 3, 40 * 40)], np.uint16)
    ref = O.causal_softmax(x, 40, 40, 0.5)[1]
    for _ in range(20):
        got = ref.copy()
        i = int(rng.integers(0, got.size))
        got[i] = O.h(O.f(got[i]) + float(rng.choice([1e-4, 5e-3, 0.05])))
        rc, acc = verify(got, ref, 40, 40)
        name, oacc = O.verify(got, ref, 40, 40)
        assert O.VERIFY_NAMES[rc] == name
        assert acc.max_abs == pytest.approx(oacc.max_abs)


def test_bench_stats_mirror_reference():
    # host/src/lib.rs:530-576
    s = cs.bench_stats([5.0, 2.0, 9.0])
    assert (s["min_ms"], s["median_ms"], s["p95_ms"]) == (2.0, 5.0, 9.0)
    assert cs.bench_stats([2.0, 8.0])["median_ms"] == 5.0
    b = cs.bench_stats([1.0, 3.0, 5.0, 7.0, 9.0])
    assert (b["samples"], b["median_ms"], b["p95_ms"], b["p99_ms"]) == (5, 5.0, 9.0, 9.0)
    assert b["mean_ms"] == 5.0
    assert abs(b["stddev_ms"] - math.sqrt(8.0)) < 1e-12
    assert b["cv_pct"] > 0
    for bad in ([], [float("nan")], [-1.0]):
        with pytest.raises(cs.CausalSoftmaxError):
            cs.bench_stats(bad)
    assert cs.bench_stats([0.0])["cv_pct"] == 0.0
    line = cs.bench_report([1.0, 2.0, 3.0], "tma", 4096, 4096, 50335744.0)
    assert line.startswith("kernel=tma rows=4096 cols=4096 n=3 min_ms=1.00000 median_ms=2.00000")
    assert "approx_logical_GBps=25.17" in line and "Melem_per_s=8388.61" in line


def test_config_parse_mirrors_reference():
    # host/src/lib.rs:412-470, 552-554, 577-583
    c = cs.parse_config([])
    assert (c["rows"], c["cols"], c["scale"], c["iterations"], c["warmup"], c["verify"]) == \
        (4096, 4096, 0.125, 20, 5, 1)
    assert cs.resolve_kernel(c["kernel"], c["rows"], c["cols"]) == "pipeline"
    c = cs.parse_config(["--bench", "--rows", "12", "--cols", "17", "--scale", "0.5",
                         "--iterations", "7"])
    assert (c["action"], c["rows"], c["cols"], c["iterations"], c["scale"]) == (4, 12, 17, 7, 0.5)
    for bad in (["--rows", "0"], ["--scale", "NaN"], ["--scale", "-0.5"], ["--scale", "1e31"],
                ["--cols"], ["--x"], ["--kernel", "wrong"], ["--cols", "33", "--kernel", "warp"],
                ["--cols", "2147483647"], ["--bench-suite", "--iterations", "0"],
                ["--rows", "-3"], ["--gpus", "3"], ["--pitch", "12", "--cols", "9"]):
        with pytest.raises(ValueError):
            cs.parse_config(bad)
    assert cs.parse_config(["--scale", "0"])["scale"] == 0.0
    assert cs.parse_config(["--cols", "31"])["cols"] == 31
    c = cs.parse_config(["--bench-suite", "--iterations", "8", "--warmup", "2"])
    assert (c["action"], c["iterations"]) == (5, 8)
    c = cs.parse_config(["--stress", "--config", "3", "--batch", "2", "--seed", "2", "--gpus", "8"])
    assert (c["rows"], c["cols"], c["config"], c["batch"], c["seed"], c["gpus"]) == (8192, 8192, 3, 2, 2, 8)
    with pytest.raises(ValueError, match="--probe"):
        cs.parse_config(["--help"])


def test_generator_is_counter_based_and_shardable():
    full = cs.generate(3, 2, batch=1, rows=64, cols=80, threads=3)
    part = cs.generate(3, 2, batch=1, rows=24, cols=80, first_row=20, threads=1)
    assert np.array_equal(full[0, 20:44], part[0])
    again = cs.generate(3, 2, batch=1, rows=64, cols=80, threads=1)
    assert np.array_equal(full, again)
    heads = cs.generate(4, 3, batch=4, rows=8, cols=16)
    assert np.array_equal(cs.generate(4, 3, batch=2, rows=8, cols=16, first_batch=2), heads[2:])
    assert not np.array_equal(heads[0], heads[1])
    # Padding columns are zero, values are finite halves.
    odd = cs.generate(2, 1, batch=2, rows=10, cols=13)
    assert odd.shape == (2, 10, 16) and np.all(odd[:, :, 13:] == 0)
    vals = np.array([O.f(b) for b in odd[:, :, :13].ravel()])
    assert np.all(np.isfinite(vals)) and vals.min() >= -8 and vals.max() <= 8


def test_generator_distributions():
    x = cs.generate(1, 0, batch=1, rows=256, cols=256)[0].ravel()
    v = np.array([O.f(b) for b in x[:20000]])
    assert abs(v.mean()) < 0.15 and abs(v.std() - 4.0) < 0.15
    s = cs.generate(3, 2, batch=1, rows=200, cols=200)[0]
    vals = np.vectorize(O.f)(s)
    big = np.abs(vals) == 60000.0
    assert 0.005 < big.mean() < 0.02
    for r in range(1, 200):
        row = vals[r, : r + 1]
        assert np.count_nonzero(row == row.max()) >= 2, r  # planted ties
    ramp = cs.generate(5, 4, batch=1, rows=4, cols=4096)[0]
    rv = np.vectorize(O.f)(ramp[0])
    assert rv[3000:].mean() - rv[:1000].mean() == pytest.approx(3.0, abs=0.3)


def test_oracle_free_self_check():
    rows, cols = 20, 27
    pitch = cs.padded_pitch(cols)
    x = cs.generate(2, 1, batch=1, rows=rows, cols=cols)
    y = O.softmax_strided(x.ravel(), 1, 0, rows, cols, pitch, 0, 1.0)
    rep = cs.check_output(y, batch=1, rows=rows, cols=cols, pitch=pitch)
    assert rep["mask_violations"] == 0 and rep["rowsum_violations"] == 0
    y2 = y.copy()
    y2[3 * pitch + 10] = O.h(0.25)
    rep = cs.check_output(y2, batch=1, rows=rows, cols=cols, pitch=pitch)
    assert rep["mask_violations"] == 1


def test_host_copy_bytes_cover_the_causal_prefixes():
    # cs_session_softmax_host moves rows in blocks of 256, each as wide as its
    # widest row; full-width rows in one block. Model it and check coverage.
    # A matrix larger than the chunk target (1/8 of the job, 8..256 MB of
    # device buffer) travels in row chunks, each blocked from its own offset.
    def blocks(rows, cols, off):
        tri = min(max(cols - 1 - off, 0), rows)
        per = 0
        for r0 in range(0, tri, 256):
            r1 = min(r0 + 256, tri)
            per += (r1 - r0) * min(off + r1, cols) * 2
        return per + (rows - tri) * cols * 2

    def model(batch, rows, cols, off):
        pitch = (cols + 7) // 8 * 8
        mat = rows * pitch * 2
        target = min(256 << 20, max(8 << 20, batch * mat // 8))
        rc = rows if mat <= target else max(1, min(rows, target // (pitch * 2)))
        return batch * sum(blocks(min(rc, rows - r0), cols, off + r0) for r0 in range(0, rows, rc))

    for batch, rows, cols, off in [(256, 4096, 4096, 0), (7, 300, 301, 0), (1, 100, 50, 2000),
                                   (3, 1000, 1037, 0), (1, 4096, 32, 0), (2, 513, 4096, 3000),
                                   (1, 1, 1, 0), (1, 8192, 8192, 0), (1, 32768, 32768, 0),
                                   (1, 20000, 20001, 5), (1, 4096, 4096, 0)]:
        got = cs.host_copy_bytes(batch, rows, cols, off)
        assert got == model(batch, rows, cols, off), (batch, rows, cols, off)
        causal = (sum(min(off + r + 1, cols) for r in range(rows)) * 2 * batch if rows < 5000
                  else 0)
        assert causal <= got <= batch * rows * cols * 2
    assert cs.host_copy_bytes(256, 4096, 4096) < 0.54 * 256 * 4096 * 4096 * 2
    assert cs.host_copy_bytes(0, 4, 4) == cs.ERR_CODE["EMPTY"]
