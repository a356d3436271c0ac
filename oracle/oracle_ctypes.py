"""ctypes binding of the CPU oracle (oracle/oracle.c) — TEST INFRASTRUCTURE ONLY.

Only the test suite, the smoke check and the CPU-baseline leg of bench.py load
this module; the product library never does. Every function here wraps a C
restatement of the reference CPU path (see oracle/oracle.h for the
reference/src/lib.rs and reference/src/online.rs line citations).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lock = threading.Lock()
_lib = None

OK, EMPTY, WRONG_LENGTH, BAD_SCALE, NON_FINITE = 0, 1, 2, 3, 4
VERIFY_NAMES = ["ok", "length", "non_finite", "negative", "mask", "element", "row_sum"]


def build() -> str:
    """Compile oracle/oracle.c with oracle/Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class Accuracy(ctypes.Structure):
    _fields_ = [
        ("max_abs", ctypes.c_float),
        ("max_relative", ctypes.c_float),
        ("max_row_sum_error", ctypes.c_float),
        ("index", ctypes.c_int64),
        ("got", ctypes.c_float),
        ("want", ctypes.c_float),
    ]


class AcceptReport(ctypes.Structure):
    _fields_ = [
        ("checked_rows", ctypes.c_int64),
        ("mask_violations", ctypes.c_int64),
        ("elem_violations", ctypes.c_int64),
        ("rowsum_violations", ctypes.c_int64),
        ("first_bad_index", ctypes.c_int64),
        ("max_abs", ctypes.c_double),
        ("max_ulp", ctypes.c_int64),
        ("max_rowsum_err", ctypes.c_double),
        ("oracle_max_rowsum_err", ctypes.c_double),
        ("floor_rows", ctypes.c_int64),
        ("max_floor_excess", ctypes.c_double),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(
                os.path.getmtime(os.path.join(_HERE, f)) for f in ("oracle.c", "oracle.h")
            ):
                build()
            L = ctypes.CDLL(_LIB_PATH)
            u16p = ctypes.POINTER(ctypes.c_uint16)
            sz, i64, f32 = ctypes.c_size_t, ctypes.c_int64, ctypes.c_float
            L.or_half_to_f32.argtypes = [ctypes.c_uint16]
            L.or_half_to_f32.restype = ctypes.c_float
            L.or_f32_to_half.argtypes = [ctypes.c_float]
            L.or_f32_to_half.restype = ctypes.c_uint16
            L.or_f64_to_half.argtypes = [ctypes.c_double]
            L.or_f64_to_half.restype = ctypes.c_uint16
            L.or_validate.argtypes = [u16p, sz, sz, sz, f32]
            L.or_causal_softmax.argtypes = [u16p, sz, sz, sz, f32, u16p]
            L.or_tiled_online_softmax.argtypes = [u16p, sz, sz, sz, f32, u16p]
            L.or_butterfly.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int,
                                       ctypes.POINTER(ctypes.c_float)]
            L.or_butterfly.restype = None
            L.or_padded_pitch.argtypes = [sz]
            L.or_padded_pitch.restype = sz
            L.or_pad.argtypes = [u16p, sz, sz, u16p]
            L.or_pad.restype = None
            L.or_unpad.argtypes = [u16p, sz, sz, u16p]
            L.or_unpad.restype = None
            strided = [u16p, u16p, i64, i64, i64, i64, i64, i64, f32, ctypes.c_int]
            L.or_causal_softmax_strided.argtypes = strided
            L.or_causal_softmax_f64_strided.argtypes = strided
            L.or_verify.argtypes = [u16p, u16p, sz, sz, sz, sz, ctypes.POINTER(Accuracy)]
            L.or_accept_strided.argtypes = [u16p, u16p, i64, i64, i64, i64, i64, i64,
                                            ctypes.c_double, i64, ctypes.c_double, ctypes.c_double,
                                            ctypes.POINTER(AcceptReport)]
            L.or_generate.argtypes = [u16p, ctypes.c_int, ctypes.c_uint64, i64, i64, i64, i64, i64,
                                      i64, i64, ctypes.c_int]
            _lib = L
    return _lib


def _u16(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint16)


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))


def h(x: float) -> int:
    """reference/src/lib.rs:48-83 f32_to_half (x is first rounded to f32)."""
    return int(lib().or_f32_to_half(float(np.float32(x))))


def f(bits: int) -> float:
    """reference/src/lib.rs:30-45 half_to_f32."""
    return float(lib().or_half_to_f32(int(bits) & 0xFFFF))


def h64(x: float) -> int:
    return int(lib().or_f64_to_half(float(x)))


def validate(scores, rows: int, cols: int, scale: float, length: int | None = None) -> int:
    s = _u16(scores)
    n = s.size if length is None else length
    ptr = _p(s) if s.size else ctypes.POINTER(ctypes.c_uint16)()
    return lib().or_validate(ptr, n, rows, cols, scale)


def causal_softmax(scores, rows: int, cols: int, scale: float, length: int | None = None):
    """reference/src/lib.rs:85-108. Returns (error_code, output array or None)."""
    s = _u16(scores)
    n = s.size if length is None else length
    out = np.zeros(max(s.size, 1), dtype=np.uint16)
    ptr = _p(s) if s.size else ctypes.POINTER(ctypes.c_uint16)()
    rc = lib().or_causal_softmax(ptr, n, rows, cols, scale, _p(out))
    return rc, (out[: s.size] if rc == OK else None)


def tiled_online_softmax(scores, rows: int, cols: int, scale: float):
    s = _u16(scores)
    out = np.zeros(max(s.size, 1), dtype=np.uint16)
    rc = lib().or_tiled_online_softmax(_p(s), s.size, rows, cols, scale, _p(out))
    return rc, (out[: s.size] if rc == OK else None)


def butterfly(values, maximum: bool) -> list[float]:
    a = (ctypes.c_float * 32)(*[float(v) for v in values])
    o = (ctypes.c_float * 32)()
    lib().or_butterfly(a, 1 if maximum else 0, o)
    return list(o)


def padded_pitch(cols: int) -> int:
    return int(lib().or_padded_pitch(cols))


def pad(scores, rows: int, cols: int) -> np.ndarray:
    s = _u16(scores)
    out = np.zeros(rows * padded_pitch(cols), dtype=np.uint16)
    lib().or_pad(_p(s), rows, cols, _p(out))
    return out


def unpad(padded, rows: int, cols: int) -> np.ndarray:
    s = _u16(padded)
    out = np.zeros(rows * cols, dtype=np.uint16)
    lib().or_unpad(_p(s), rows, cols, _p(out))
    return out


def softmax_strided(inp: np.ndarray, batch: int, batch_stride: int, rows: int, cols: int,
                    pitch: int, row_offset: int, scale: float, threads: int = 0,
                    f64: bool = False) -> np.ndarray:
    """Batched/pitched/row-offset form of reference/src/lib.rs:85-108 (f32) or of the
    FP64 restatement; the output has the input's strided layout."""
    x = _u16(inp)
    out = np.zeros_like(x)
    if threads <= 0:
        threads = os.cpu_count() or 1
    fn = lib().or_causal_softmax_f64_strided if f64 else lib().or_causal_softmax_strided
    rc = fn(_p(x), _p(out), batch, batch_stride, rows, cols, pitch, row_offset,
            float(scale), threads)
    if rc != OK:
        raise ValueError(f"oracle rejected the shape (code {rc})")
    return out


def generate(config: int, seed: int, batch: int, rows: int, cols: int, pitch: int | None = None,
             first_batch: int = 0, first_row: int = 0, threads: int = 0,
             out: np.ndarray | None = None) -> np.ndarray:
    """Seeded workload matrices (oracle.h or_generate): uint16 half bits of shape
    (batch, rows, pitch), written into `out` when given."""
    pitch = padded_pitch(cols) if pitch is None else pitch
    if out is None:
        out = np.empty((batch, rows, pitch), dtype=np.uint16)
    if out.dtype != np.uint16 or out.size != batch * rows * pitch:
        raise ValueError("out must be uint16 of batch*rows*pitch elements")
    if not out.flags.c_contiguous:
        raise ValueError("out must be contiguous")
    if threads <= 0:
        threads = os.cpu_count() or 1
    rc = lib().or_generate(_p(out), config, seed, batch, rows * pitch, rows, cols, pitch,
                           first_batch, first_row, threads)
    if rc != OK:
        raise ValueError(f"oracle generator rejected the shape (code {rc})")
    return out


def roofline_bytes(rows: int, cols: int, row_offset: int = 0) -> float:
    """Algorithmic bytes of one matrix: 2*T (causal prefix read) + 2*rows*cols
    (full write), T = causal elements of rows [row_offset, row_offset+rows)
    (host/src/lib.rs:52-56 for row_offset 0)."""
    tri = max(0, min(rows, cols - 1 - row_offset))
    t = tri * (row_offset + 1) + tri * (tri - 1) // 2 + (rows - tri) * cols
    return 2.0 * t + 2.0 * rows * cols


def verify(got, expected, rows: int, cols: int, len_override: tuple | None = None):
    """host/src/lib.rs:280-328. Returns (name, Accuracy)."""
    g, e = _u16(got), _u16(expected)
    acc = Accuracy()
    lg, le = (g.size, e.size) if len_override is None else len_override
    gp = _p(g) if g.size else ctypes.POINTER(ctypes.c_uint16)()
    ep = _p(e) if e.size else ctypes.POINTER(ctypes.c_uint16)()
    rc = lib().or_verify(gp, ep, lg, le, rows, cols, ctypes.byref(acc))
    return VERIFY_NAMES[rc], acc


def accept(got: np.ndarray, f64_ref: np.ndarray, batch: int, batch_stride: int, rows: int,
           cols: int, pitch: int, row_offset: int, abs_tol: float = 2e-3, ulp_tol: int = 2,
           rowsum_tol: float = 2e-3, floor_margin: float = -1.0) -> dict:
    """North-star acceptance: masked == 0x0000, unmasked within ulp_tol FP16 ulp or
    abs_tol absolute of the FP64 oracle, |row sum - 1| <= rowsum_tol (or, with
    floor_margin >= 0, within the FP64 oracle's own FP16 row-sum error plus
    floor_margin on rows where that error already exceeds rowsum_tol)."""
    g, r = _u16(got), _u16(f64_ref)
    rep = AcceptReport()
    rc = lib().or_accept_strided(_p(g), _p(r), batch, batch_stride, rows, cols, pitch,
                                 row_offset, abs_tol, ulp_tol, rowsum_tol, floor_margin,
                                 ctypes.byref(rep))
    d = rep.as_dict()
    d["ok"] = rc == 0
    return d
