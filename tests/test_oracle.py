"""Pins the CPU oracle to the reference's own known-answer tests.

Each test restates one test of reference/src/lib.rs:154-362,
reference/src/online.rs:63-123 or host/src/lib.rs:409-584 (cited per test),
run against the C restatement in oracle/oracle.c. Literal values come from
tests/golden/reference_known_answers.json.
"""
import json
import math
import os

import numpy as np
import pytest

import oracle_ctypes as O

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden",
                                     "reference_known_answers.json")))
ERR = {"Empty": O.EMPTY, "WrongLength": O.WRONG_LENGTH, "BadScale": O.BAD_SCALE,
       "NonFinite": O.NON_FINITE}
USIZE_MAX = 2**64 - 1


def hx(s: str) -> int:
    return int(s, 16)


def hv(values) -> np.ndarray:
    return np.array([O.h(v) for v in values], dtype=np.uint16)


def fv(bits) -> np.ndarray:
    return np.array([O.f(b) for b in bits], dtype=np.float64)


# reference/src/lib.rs:165-183
def test_half_specials_and_ties():
    for case in GOLDEN["f32_to_half"]["cases"]:
        x = float.fromhex(case["x"]) if case["x"].startswith(("0x", "-0x")) else float(case["x"])
        assert O.h(x) == hx(case["bits"]), case
    for case in GOLDEN["half_to_f32"]["cases"]:
        got = O.f(hx(case["bits"]))
        if case["x"] == "nan":
            assert math.isnan(got)
        else:
            assert got == float.fromhex(case["x"]), case


# reference/src/lib.rs:268-276
def test_every_finite_half_roundtrips():
    for bits in range(0x10000):
        if bits & 0x7C00 == 0x7C00 and bits & 0x03FF:
            continue
        assert O.lib().or_f32_to_half(O.lib().or_half_to_f32(bits)) == bits, hex(bits)


def test_f64_to_half_agrees_with_f32_path_on_exact_values():
    # Every finite half is exactly representable in f64 and f32: both roundings agree.
    for bits in range(0, 0x7C00, 7):
        x = O.f(bits)
        assert O.h64(x) == bits
        assert O.h64(-x) == (bits | 0x8000)
    assert O.h64(65519.99) == 0x7BFF and O.h64(65520.0) == 0x7C00
    assert O.h64(2.0**-25) == 0 and O.h64(3 * 2.0**-25) == 2


# reference/src/lib.rs:185-187, 315-320
def test_exact_outputs():
    for case in GOLDEN["softmax_exact"]["cases"]:
        rc, y = O.causal_softmax(hv(case["input_f32"]), case["rows"], case["cols"], case["scale"])
        assert rc == O.OK
        assert [int(v) for v in y] == [hx(b) for b in case["output_bits"]]


# reference/src/lib.rs:189-203
def test_all_zero_triangular():
    rc, y = O.causal_softmax(hv([0.0] * 16), 4, 4, 1.0)
    assert rc == O.OK
    for r in range(4):
        for c in range(4):
            want = O.f(O.h(1.0 / (r + 1))) if c <= r else 0.0
            assert O.f(y[r * 4 + c]) == want


# reference/src/lib.rs:205-211
def test_large_logits_stable():
    g = GOLDEN["large_logits_stable"]
    rc, y = O.causal_softmax(hv(g["input_f32"]), g["rows"], g["cols"], g["scale"])
    assert rc == O.OK
    assert O.f(y[0]) == 1.0 and O.f(y[1]) == 0.0
    assert abs(O.f(y[2]) + O.f(y[3]) - 1.0) < g["row1_sum_tol"]


# reference/src/lib.rs:213-223
def test_rectangular_and_mask():
    scores = hv([(i % 7) - 2.0 for i in range(35)])
    rc, y = O.causal_softmax(scores, 5, 7, 0.25)
    assert rc == O.OK
    for r in range(5):
        s = np.float32(0)
        for c in range(7):
            s = np.float32(s + np.float32(O.f(y[r * 7 + c])))
        assert abs(float(s) - 1.0) < 0.002
        for c in range(r + 1, 7):
            assert y[r * 7 + c] == 0


# reference/src/lib.rs:225-233
def test_skinny_and_wide():
    for r, c in [(1, 17), (7, 1), (3, 257), (5, 15), (9, 256)]:
        rc, y = O.causal_softmax(hv([0.125] * (r * c)), r, c, 0.2)
        assert rc == O.OK
        for row in range(r):
            assert fv(y[row * c:(row + 1) * c]).sum() > 0.99


# reference/src/lib.rs:235-241
def test_padding_roundtrip():
    for r, c in [(1, 1), (5, 17), (4, 256), (3, 257)]:
        x = np.arange(r * c, dtype=np.uint16)
        padded = O.pad(x, r, c)
        assert np.array_equal(O.unpad(padded, r, c), x)
        assert padded.size % 8 == 0


# reference/src/lib.rs:243-258, 344-360
def test_errors():
    for case in GOLDEN["errors"]["cases"]:
        rows = USIZE_MAX if case["rows"] == "usize::MAX" else case["rows"]
        bits = np.array([hx(b) for b in case["input_bits"]], dtype=np.uint16)
        rc, _ = O.causal_softmax(bits, rows, case["cols"], case["scale"], length=case["len"])
        assert rc == ERR[case["error"]], case


# reference/src/lib.rs:260-265
def test_monotonic():
    g = GOLDEN["monotonic"]
    rc, y = O.causal_softmax(hv(g["input_f32"]), g["rows"], g["cols"], g["scale"])
    assert rc == O.OK
    a, b = g["greater"]
    assert O.f(y[a]) > O.f(y[b])
    assert y[g["zero_index"]] == 0


# reference/src/lib.rs:279-300
def test_independent_f64_oracle():
    for rows, cols in [(1, 1), (2, 9), (7, 3), (16, 17), (33, 257)]:
        x = hv([((i * 37 % 101) - 50.0) / 9.0 for i in range(rows * cols)])
        rc, result = O.causal_softmax(x, rows, cols, 0.25)
        assert rc == O.OK
        for row in range(rows):
            n = min(row + 1, cols)
            scores = [O.f(x[row * cols + c]) * 0.25 for c in range(n)]
            m = max(scores)
            denom = sum(math.exp(s - m) for s in scores)
            for col in range(cols):
                want = float(np.float32(math.exp(scores[col] - m) / denom)) if col < n else 0.0
                assert abs(O.f(result[row * cols + col]) - want) < 0.001


# reference/src/lib.rs:303-312
def test_subnormal_inputs_remain_finite():
    g = GOLDEN["subnormal_inputs"]
    x = np.array([hx(b) for b in g["input_bits"]], dtype=np.uint16)
    rc, p = O.causal_softmax(x, g["rows"], g["cols"], g["scale"])
    assert rc == O.OK
    assert all(math.isfinite(O.f(v)) for v in p)
    for r in range(3):
        assert fv(p[r * 3:(r + 1) * 3]).sum() > g["min_row_sum"]


# reference/src/lib.rs:323-332
def test_all_rows_normalize_under_varied_scales():
    x = hv([((i % 13) - 6.0) * 0.75 for i in range(35)])
    for scale in [0.001, 0.125, 1.0, 10.0]:
        rc, y = O.causal_softmax(x, 7, 5, scale)
        assert rc == O.OK
        for row in range(7):
            assert abs(fv(y[row * 5:(row + 1) * 5]).sum() - 1.0) < 0.002


# reference/src/lib.rs:335-341
def test_reference_deterministic():
    x = hv([(i % 17) / 8.0 for i in range(1024)])
    a = O.causal_softmax(x, 32, 32, 0.3)[1]
    b = O.causal_softmax(x, 32, 32, 0.3)[1]
    assert np.array_equal(a, b)


# reference/src/online.rs:69-76
def test_complete_butterfly_reaches_every_lane():
    g = GOLDEN["butterfly"]
    x = [float(i + 1) for i in range(32)]
    assert O.butterfly(x, False) == [g["sum_of_1_to_32"]] * 32
    assert O.butterfly(x, True) == [g["max_of_1_to_32"]] * 32
    sparse = [-math.inf] * 32
    sparse[31] = -7.0
    assert O.butterfly(sparse, True) == [g["sparse_lane31"]] * 32


# reference/src/online.rs:79-100
def test_ragged_tiles_match_independent_reference():
    for rows, cols in [(1, 1), (7, 17), (9, 129), (65, 257), (137, 259), (257, 513)]:
        scores = hv([((i * 7919 % 251) - 125.0) * 0.125 for i in range(rows * cols)])
        for scale in [0.0, 0.001, 0.125, 1.0, 10.0]:
            rc1, actual = O.tiled_online_softmax(scores, rows, cols, scale)
            rc2, expected = O.causal_softmax(scores, rows, cols, scale)
            assert rc1 == rc2 == O.OK
            g, w = fv(actual), fv(expected)
            assert np.all(np.abs(g - w) <= 0.003 + 0.003 * w)
            idx = np.arange(rows * cols)
            masked = (idx % cols) > (idx // cols)
            assert np.all(actual[masked] == 0)


# reference/src/online.rs:103-122
def test_extremes_are_finite_and_zero_scale_is_uniform():
    rows, cols = 139, 257
    scores = hv([65504.0 if i % 3 == 0 else -65504.0 for i in range(rows * cols)])
    for scale in [0.0, 1.0, 1.0e30]:
        rc, result = O.tiled_online_softmax(scores, rows, cols, scale)
        assert rc == O.OK
        vals = fv(result).reshape(rows, cols)
        assert np.all(np.isfinite(vals))
        for r in range(rows):
            s = np.float32(0)
            for c in range(cols):
                s = np.float32(s + np.float32(vals[r, c]))
            assert abs(float(s) - 1.0) < 0.003
            if scale == 0.0:
                assert np.all(result.reshape(rows, cols)[r, : r + 1] == O.h(1.0 / (r + 1)))


# host/src/lib.rs:502-529, 555-558
def test_verifier_known_answers():
    zeros = hv([0.0] * 16)
    y = O.causal_softmax(zeros, 4, 4, 1.0)[1]
    assert O.verify(y, y, 4, 4)[0] == "ok"
    ones = hv([1.0] * 9)
    assert O.verify(ones, ones, 3, 3)[0] == "mask"
    name, acc = O.verify(np.array([0x7C00], np.uint16), np.array([0x7C00], np.uint16), 1, 1)
    assert name == "non_finite" and acc.index == 0
    name, acc = O.verify(hv([-0.0005]), hv([0.0]), 1, 1)
    assert name == "negative" and acc.index == 0
    empty = np.zeros(0, np.uint16)
    assert O.verify(empty, empty, USIZE_MAX, 2)[0] == "length"


def test_strided_matches_dense_reference():
    # The batched/pitched/row-offset driver is the same per-row arithmetic.
    rng = np.random.default_rng(5)
    rows, cols = 37, 45
    x = hv(rng.uniform(-8, 8, rows * cols))
    _, dense = O.causal_softmax(x, rows, cols, 0.7)
    pitch = O.padded_pitch(cols)
    padded = O.pad(x, rows, cols)
    batch = np.concatenate([padded, padded])
    out = O.softmax_strided(batch, 2, rows * pitch, rows, cols, pitch, 0, 0.7, threads=3)
    for b in range(2):
        mat = out[b * rows * pitch:(b + 1) * rows * pitch]
        assert np.array_equal(O.unpad(mat, rows, cols), dense)
        assert np.all(mat.reshape(rows, pitch)[:, cols:] == 0)
    # Row-block shards with an absolute row offset reproduce the full matrix.
    top = O.softmax_strided(padded[: 20 * pitch], 1, 0, 20, cols, pitch, 0, 0.7)
    bottom = O.softmax_strided(padded[20 * pitch:], 1, 0, rows - 20, cols, pitch, 20, 0.7)
    assert np.array_equal(np.concatenate([top, bottom]), out[: rows * pitch])


def test_f64_oracle_acceptance_of_f32_spec():
    # The f32 specification itself passes the FP64 acceptance check.
    rng = np.random.default_rng(9)
    for rows, cols, scale in [(64, 64, 0.125), (50, 123, 1.0), (200, 37, 0.0), (9, 300, 10.0)]:
        x = hv(rng.normal(0, 4, rows * cols))
        _, spec = O.causal_softmax(x, rows, cols, scale)
        ref = O.softmax_strided(x, 1, 0, rows, cols, cols, 0, scale, f64=True)
        rep = O.accept(spec, ref, 1, 0, rows, cols, cols, 0)
        assert rep["ok"], rep
        assert rep["max_ulp"] <= 1


def test_acceptance_detects_planted_mistakes():
    # A mistake planted in the oracle's own output (on the CPU) is caught.
    rows, cols = 16, 24
    x = hv(np.linspace(-3, 3, rows * cols))
    ref = O.softmax_strided(x, 1, 0, rows, cols, cols, 0, 1.0, f64=True)
    bad = ref.copy()
    bad[0 * cols + 5] = O.h(1e-3)  # masked position
    assert O.accept(bad, ref, 1, 0, rows, cols, cols, 0)["mask_violations"] == 1
    bad = ref.copy()
    bad[10 * cols + 3] = O.h(O.f(bad[10 * cols + 3]) + 0.01)
    rep = O.accept(bad, ref, 1, 0, rows, cols, cols, 0)
    assert rep["elem_violations"] == 1 and rep["rowsum_violations"] == 1


def test_row_sum_floor_is_per_row_and_bounded():
    # A uniform row of n columns: every probability is 1/n rounded to FP16.
    # For n near 2^24 / (k + 1/2) the rounding error of each element is close
    # to half an ulp in the same direction, so the exactly rounded FP64 result
    # itself misses the 2e-3 row-sum bound. Such a row is accepted at its own
    # error plus the margin, and only there; a row whose oracle meets the
    # bound gets no allowance. Mistakes are planted in the oracle output.
    best = None
    for n in range(70000, 140000, 7):
        h = O.h64(1.0 / n)
        err = abs(n * O.f(h) - 1.0)
        if best is None or err > best[1]:
            best = (n, err)
    n, err = best
    assert err > 2.5e-3, best
    zeros = np.zeros(n, np.uint16)
    ref = O.softmax_strided(zeros, 1, 0, 1, n, n, n - 1, 0.0, f64=True)
    assert np.all(ref == O.h64(1.0 / n))
    # The oracle's own output: fails without an allowance, passes with one.
    assert not O.accept(ref, ref, 1, 0, 1, n, n, n - 1)["ok"]
    rep = O.accept(ref, ref, 1, 0, 1, n, n, n - 1, floor_margin=0.0)
    assert rep["ok"] and rep["floor_rows"] == 1 and rep["max_floor_excess"] == 0.0
    # One more ulp on 20 elements, away from 1: excess of 20 ulp.
    worse = ref.copy()
    step = 1 if n * O.f(ref[0]) > 1.0 else -1
    worse[:20] = (worse[:20].astype(np.int32) + step).astype(np.uint16)
    excess = 20 * abs(O.f(worse[0]) - O.f(ref[0]))
    assert O.accept(worse, ref, 1, 0, 1, n, n, n - 1, floor_margin=2 * excess)["ok"]
    rep = O.accept(worse, ref, 1, 0, 1, n, n, n - 1, floor_margin=excess / 2)
    assert not rep["ok"] and rep["rowsum_violations"] == 1
    # A row whose oracle meets the bound: no allowance at all.
    m = 4096
    x = hv(np.linspace(-2, 2, m))
    r2 = O.softmax_strided(x, 1, 0, 1, m, m, m - 1, 1.0, f64=True)
    bad = r2.copy()
    bad[-1] = O.h(O.f(bad[-1]) + 0.004)  # row sum off by ~4e-3, element beyond tolerance too
    rep = O.accept(bad, r2, 1, 0, 1, m, m, m - 1, floor_margin=1.0)
    assert not rep["ok"] and rep["floor_rows"] == 0 and rep["rowsum_violations"] == 1
