"""Python binding of the B200 fused causal softmax C ABI (include/causal_softmax.h).

This module is plumbing: it loads lib/libcausal_softmax.so with ctypes and
passes raw device pointers (from torch tensors) and CUDA stream handles to the
C entry points. There is no fallback: if the CUDA library is missing or the
device is not sm_100, every call raises.

Kernel names follow the reference host surface (host/src/lib.rs:5-42):
auto, baseline, warp, tma, pipeline, online.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.dirname(_HERE)
LIB_PATH = os.path.join(PKG_DIR, "lib", "libcausal_softmax.so")
HEADER_PATHS = [os.path.join(os.path.dirname(PKG_DIR), "include", n)
                for n in ("causal_softmax.h", "causal_softmax_host.h")]

AUTO, BASELINE, WARP, TMA, PIPELINE, ONLINE = range(6)
KERNELS = {"auto": AUTO, "baseline": BASELINE, "warp": WARP, "tma": TMA,
           "pipeline": PIPELINE, "online": ONLINE}
KERNEL_NAMES = {v: k for k, v in KERNELS.items()}

OK = 0
ERR = {
    -1: "EMPTY", -2: "WRONG_LENGTH", -3: "BAD_SCALE", -4: "NON_FINITE", -5: "WARP_COLS",
    -6: "ALIGNMENT", -7: "PITCH", -8: "BAD_KERNEL", -9: "DEVICE", -10: "CUDA", -11: "TIMEOUT",
    -12: "NULL", -13: "PADDING", -14: "UNSUPPORTED", -15: "PROBE", -16: "ARG", -17: "STATUS",
}
ERR_CODE = {v: k for k, v in ERR.items()}
STATUS_TIMEOUT = 1
DEBUG_SKIP_LOADS = 1

PATTERNS = ["zeros", "ramp", "alternating", "spikes", "extreme", "tiny", "random"]


class CausalSoftmaxError(RuntimeError):
    def __init__(self, code: int, where: str = ""):
        self.code = code
        self.name = ERR.get(code, str(code))
        L = lib()
        msg = L.cs_strerror(code).decode()
        detail = L.cs_last_error_detail().decode()
        super().__init__(f"{where}: {self.name} ({msg}){' — ' + detail if detail else ''}")


class LaunchInfo(ctypes.Structure):
    _fields_ = [
        ("kernel", ctypes.c_int32), ("grid", ctypes.c_int32), ("block", ctypes.c_int32),
        ("smem_bytes", ctypes.c_int32), ("stages", ctypes.c_int32),
        ("vec_per_thread", ctypes.c_int32), ("ctas_per_sm", ctypes.c_int32),
        ("launches", ctypes.c_int32), ("units", ctypes.c_int64),
        ("algorithmic_bytes", ctypes.c_double), ("modelled_bytes", ctypes.c_double),
    ]

    def as_dict(self) -> dict:
        d = {n: getattr(self, n) for n, _ in self._fields_}
        d["kernel_name"] = KERNEL_NAMES.get(self.kernel, str(self.kernel))
        return d


class Accuracy(ctypes.Structure):
    _fields_ = [("max_abs", ctypes.c_float), ("max_relative", ctypes.c_float),
                ("max_row_sum_error", ctypes.c_float), ("index", ctypes.c_int64),
                ("got", ctypes.c_float), ("want", ctypes.c_float)]


class SelfCheck(ctypes.Structure):
    _fields_ = [("rows_checked", ctypes.c_int64), ("mask_violations", ctypes.c_int64),
                ("nonfinite_or_negative", ctypes.c_int64), ("rowsum_violations", ctypes.c_int64),
                ("max_rowsum_err", ctypes.c_double)]


class BenchStats(ctypes.Structure):
    _fields_ = [("samples", ctypes.c_int64)] + [
        (n, ctypes.c_double) for n in ("min_ms", "median_ms", "p95_ms", "p99_ms", "max_ms",
                                       "mean_ms", "stddev_ms", "cv_pct")]


class Config(ctypes.Structure):
    _fields_ = [("action", ctypes.c_int32), ("kernel", ctypes.c_int32),
                ("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("pitch", ctypes.c_int64),
                ("batch", ctypes.c_int64), ("scale", ctypes.c_float),
                ("iterations", ctypes.c_int32), ("warmup", ctypes.c_int32),
                ("verify", ctypes.c_int32), ("config", ctypes.c_int32),
                ("seed", ctypes.c_uint64), ("gpus", ctypes.c_int32)]


_lock = threading.Lock()
_lib = None


def lib():
    """Load the CUDA library (built in-tree by build.py); raises if it is missing."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with build.py (nvcc, sm_100a); "
                    "there is no CPU fallback")
            L = ctypes.CDLL(LIB_PATH)
            _declare(L)
            _lib = L
    return _lib


def _declare(L) -> None:
    c_int, c_i32, c_i64, c_f32, c_f64 = (ctypes.c_int, ctypes.c_int32, ctypes.c_int64,
                                         ctypes.c_float, ctypes.c_double)
    vp, u16p, sz = ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint16), ctypes.c_size_t
    sig = {
        "cs_abi_version": (c_int, []),
        "cs_strerror": (ctypes.c_char_p, [c_int]),
        "cs_last_error_detail": (ctypes.c_char_p, []),
        "cs_kernel_name": (ctypes.c_char_p, [c_int]),
        "cs_kernel_parse": (c_int, [ctypes.c_char_p]),
        "cs_kernel_supports": (c_int, [c_int, c_i64]),
        "cs_resolve_kernel": (c_int, [c_int, c_i64, c_i64]),
        "cs_logical_bytes": (c_f64, [c_int, c_i64, c_i64]),
        "cs_roofline_bytes": (c_f64, [c_i64, c_i64, c_i64]),
        "cs_padded_pitch": (c_i64, [c_i64]),
        "cs_validate": (c_int, [c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_f32]),
        "cs_check_finite_host": (c_int, [u16p, c_i64]),
        "cs_status_error": (c_int, [ctypes.c_uint32]),
        "cs_plan_create": (c_int, [ctypes.POINTER(vp), c_int, vp, vp, c_i64, c_i64, c_i32, c_i32,
                                   c_i32, c_i32]),
        "cs_plan_launch": (c_int, [vp, c_int, c_f32, vp]),
        "cs_plan_status": (c_int, [vp, ctypes.POINTER(ctypes.c_uint32)]),
        "cs_plan_set_timeout": (c_int, [vp, ctypes.c_uint64]),
        "cs_plan_set_row_split": (c_int, [vp, c_i32, c_i32]),
        "cs_plan_set_tuning": (c_int, [vp, c_int, c_int, c_int, c_int]),
        "cs_plan_set_prefetch": (c_int, [vp, c_int]),
        "cs_plan_describe": (c_int, [vp, c_int, ctypes.POINTER(LaunchInfo)]),
        "cs_plan_launch_debug": (c_int, [vp, c_int, c_f32, vp, ctypes.c_uint32, ctypes.c_uint64]),
        "cs_plan_destroy": (None, [vp]),
        "cs_softmax": (c_int, [c_int, vp, vp, c_i32, c_i32, c_i32, c_f32, vp]),
        "cs_softmax_batched": (c_int, [c_int, vp, vp, c_i64, c_i64, c_i32, c_i32, c_i32, c_i32,
                                       c_f32, vp]),
        "cs_softmax_noalloc": (c_int, [c_int, vp, vp, c_i64, c_i64, c_i32, c_i32, c_i32, c_i32,
                                       c_f32, c_i32, ctypes.POINTER(ctypes.c_uint32), vp]),
        "cs_noalloc_status": (c_int, [c_i32, ctypes.POINTER(ctypes.c_uint32), vp]),
        "cs_session_create": (c_int, [ctypes.POINTER(vp), c_int]),
        "cs_session_probe": (c_int, [vp]),
        "cs_session_softmax_host": (c_int, [vp, c_int, u16p, u16p, c_i64, c_i32, c_i32, c_i32,
                                            c_f32]),
        "cs_session_prepare": (c_int, [vp, u16p, c_i32, c_i32]),
        "cs_session_launch": (c_int, [vp, c_int, c_f32]),
        "cs_session_result": (c_int, [vp, u16p]),
        "cs_session_stream": (vp, [vp]),
        "cs_host_copy_bytes": (c_i64, [c_i64, c_i32, c_i32, c_i32]),
        "cs_session_destroy": (None, [vp]),
        "cs_host_register": (c_int, [vp, sz]),
        "cs_host_unregister": (c_int, [vp]),
        "cs_device_sm_count": (c_int, [c_int]),
        # host surface (causal_softmax_host.h)
        "cs_pattern_name": (ctypes.c_char_p, [c_int]),
        "cs_f32_to_half": (ctypes.c_uint16, [c_f32]),
        "cs_half_to_f32": (c_f32, [ctypes.c_uint16]),
        "cs_make_input": (c_int, [u16p, c_i64, c_i64, c_int, ctypes.c_uint32]),
        "cs_generate": (c_int, [vp, c_int, ctypes.c_uint64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                c_i64, c_i64, c_int]),
        "cs_verify": (c_int, [u16p, sz, u16p, sz, sz, sz, ctypes.POINTER(Accuracy)]),
        "cs_check_output": (c_int, [vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_f64,
                                    ctypes.POINTER(SelfCheck)]),
        "cs_bench_stats_from_ms": (c_int, [ctypes.POINTER(c_f64), c_i64,
                                           ctypes.POINTER(BenchStats)]),
        "cs_bench_report": (c_int, [ctypes.POINTER(BenchStats), ctypes.c_char_p, c_i64, c_i64,
                                    c_f64, ctypes.c_char_p, sz]),
        "cs_config_parse": (c_int, [c_int, ctypes.POINTER(ctypes.c_char_p),
                                    ctypes.POINTER(Config), ctypes.c_char_p, sz]),
        "cs_config_validate": (c_int, [ctypes.POINTER(Config), ctypes.c_char_p, sz]),
        "cs_config_help": (ctypes.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def check(rc: int, where: str) -> None:
    if rc != OK:
        raise CausalSoftmaxError(rc, where)


def kernel_id(kernel) -> int:
    if isinstance(kernel, str):
        k = KERNELS.get(kernel)  # the canonical names, without a call into the library
        if k is not None:
            return k
        k = lib().cs_kernel_parse(kernel.encode())
        if k < 0:
            raise CausalSoftmaxError(k, f"kernel {kernel!r}")
        return k
    return int(kernel)


def host_copy_bytes(batch: int, rows: int, cols: int, row_offset: int = 0) -> int:
    """Bytes Session.softmax_host moves in each direction (causal row blocks)."""
    return int(lib().cs_host_copy_bytes(batch, rows, cols, row_offset))


def padded_pitch(cols: int) -> int:
    return int(lib().cs_padded_pitch(cols))


def roofline_bytes(rows: int, cols: int, row_offset: int = 0) -> float:
    return float(lib().cs_roofline_bytes(rows, cols, row_offset))


def resolve_kernel(kernel, rows: int, cols: int) -> str:
    k = lib().cs_resolve_kernel(kernel_id(kernel), rows, cols)
    check(k if k < 0 else OK, "resolve_kernel")
    return KERNEL_NAMES[k]


def _stream_handle(stream) -> int:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class Plan:
    """cs_plan: a launch target (device buffers + geometry) reused across launches."""

    def __init__(self, d_in: int, d_out: int, *, rows: int, cols: int, pitch: int | None = None,
                 batch: int = 1, batch_stride: int | None = None, row_offset: int = 0,
                 device: int = 0):
        pitch = padded_pitch(cols) if pitch is None else pitch
        if batch_stride is None:
            batch_stride = rows * pitch
        self.rows, self.cols, self.pitch, self.batch = rows, cols, pitch, batch
        self.batch_stride, self.row_offset, self.device = batch_stride, row_offset, device
        h = ctypes.c_void_p()
        check(lib().cs_plan_create(ctypes.byref(h), device, d_in, d_out, batch, batch_stride,
                                   rows, cols, pitch, row_offset), "cs_plan_create")
        self._h = h

    @classmethod
    def for_tensors(cls, x, y, *, cols: int, row_offset: int = 0):
        """x, y: torch tensors [batch, rows, pitch] or [rows, pitch] of float16 on one device."""
        if x.shape != y.shape or x.dim() not in (2, 3):
            raise ValueError("input/output must have equal [batch,] rows, pitch shapes")
        if not (x.is_contiguous() and y.is_contiguous()):
            raise ValueError("tensors must be contiguous")
        batch = x.shape[0] if x.dim() == 3 else 1
        rows, pitch = x.shape[-2], x.shape[-1]
        return cls(x.data_ptr(), y.data_ptr(), rows=rows, cols=cols, pitch=pitch, batch=batch,
                   batch_stride=rows * pitch, row_offset=row_offset, device=x.device.index or 0)

    def launch(self, kernel="auto", scale: float = 0.125, stream=None) -> None:
        check(lib().cs_plan_launch(self._h, kernel_id(kernel), scale, _stream_handle(stream)),
              "cs_plan_launch")

    def launch_debug(self, kernel, scale: float, flags: int, timeout_ns: int, stream=None) -> None:
        check(lib().cs_plan_launch_debug(self._h, kernel_id(kernel), scale, _stream_handle(stream),
                                         flags, timeout_ns), "cs_plan_launch_debug")

    def status(self) -> tuple[int, int]:
        st = ctypes.c_uint32()
        rc = lib().cs_plan_status(self._h, ctypes.byref(st))
        return rc, st.value

    def set_timeout(self, ns: int) -> None:
        check(lib().cs_plan_set_timeout(self._h, ns), "cs_plan_set_timeout")

    def set_row_split(self, split_row: int, split_offset: int) -> None:
        """Local rows split_row.. are absolute rows split_offset.. (a folded
        shard: a row block and its mirror); split_row 0 undoes it."""
        check(lib().cs_plan_set_row_split(self._h, split_row, split_offset),
              "cs_plan_set_row_split")

    def set_tuning(self, vec: int = 0, stages: int = 0, l2_hint: int = -1,
                   zero_fill_tma: int = -1) -> None:
        check(lib().cs_plan_set_tuning(self._h, vec, stages, l2_hint, zero_fill_tma),
              "cs_plan_set_tuning")

    def set_prefetch(self, prefetch_units: int = -1) -> None:
        check(lib().cs_plan_set_prefetch(self._h, prefetch_units), "cs_plan_set_prefetch")

    def describe(self, kernel="auto") -> dict:
        info = LaunchInfo()
        check(lib().cs_plan_describe(self._h, kernel_id(kernel), ctypes.byref(info)),
              "cs_plan_describe")
        return info.as_dict()

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cs_plan_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """cs_session: host-buffer path (the reference Session / prepare / launch / result)."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().cs_session_create(ctypes.byref(h), device), "cs_session_create")
        self._h = h

    def probe(self) -> None:
        check(lib().cs_session_probe(self._h), "cs_session_probe")

    def softmax_host(self, h_in, h_out, *, batch: int, rows: int, cols: int, scale: float,
                     kernel="auto", row_offset: int = 0) -> None:
        """h_in/h_out: numpy uint16 arrays of batch*rows*cols dense halves (pinned for speed)."""
        check(lib().cs_session_softmax_host(self._h, kernel_id(kernel), _u16p(h_in), _u16p(h_out),
                                            batch, rows, cols, row_offset, scale),
              "cs_session_softmax_host")

    def prepare(self, h_in, rows: int, cols: int) -> None:
        check(lib().cs_session_prepare(self._h, _u16p(h_in), rows, cols), "cs_session_prepare")

    def launch(self, kernel="auto", scale: float = 0.125) -> None:
        check(lib().cs_session_launch(self._h, kernel_id(kernel), scale), "cs_session_launch")

    def result(self, h_out) -> None:
        check(lib().cs_session_result(self._h, _u16p(h_out)), "cs_session_result")

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().cs_session_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def _u16p(a):
    import numpy as np

    if not (isinstance(a, np.ndarray) and a.dtype == np.uint16 and a.flags.c_contiguous):
        raise TypeError("expected a C-contiguous numpy uint16 array")
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))


def softmax(x, *, cols: int, scale: float, kernel="auto", row_offset: int = 0, out=None,
            stream=None):
    """Causal softmax of torch float16 tensor(s) [batch,] rows, pitch (pitch % 8 == 0).

    Returns the output tensor (same shape; columns >= the causal width and the
    padding are exactly +0.0)."""
    import torch

    if x.dtype != torch.float16 or not x.is_cuda:
        raise TypeError("x must be a CUDA float16 tensor")
    y = torch.empty_like(x) if out is None else out
    batch = x.shape[0] if x.dim() == 3 else 1
    rows, pitch = x.shape[-2], x.shape[-1]
    with torch.cuda.device(x.device):
        check(lib().cs_softmax_batched(kernel_id(kernel), x.data_ptr(), y.data_ptr(), batch,
                                       rows * pitch, rows, cols, pitch, row_offset, scale,
                                       _stream_handle(stream)), "cs_softmax_batched")
    return y


# ---------------------------------------------------------------- host surface

def make_input(rows: int, cols: int, pattern, seed: int):
    """host/src/lib.rs:218-256 through the C++ host library."""
    import numpy as np

    p = PATTERNS.index(pattern) if isinstance(pattern, str) else int(pattern)
    out = np.zeros(rows * cols, dtype=np.uint16)
    check(lib().cs_make_input(_u16p(out), rows, cols, p, seed & 0xFFFFFFFF), "cs_make_input")
    return out


def generate(config: int, seed: int, *, batch: int, rows: int, cols: int, pitch: int | None = None,
             first_batch: int = 0, first_row: int = 0, threads: int = 0, out=None):
    """Seeded benchmark workload (see causal_softmax_host.h) as uint16 [batch, rows, pitch]."""
    import numpy as np

    pitch = padded_pitch(cols) if pitch is None else pitch
    if out is None:
        out = np.empty((batch, rows, pitch), dtype=np.uint16)
    ptr = out.ctypes.data if hasattr(out, "ctypes") else int(out.data_ptr())
    check(lib().cs_generate(ptr, config, seed, batch, rows * pitch, rows, cols, pitch, first_batch,
                            first_row, threads), "cs_generate")
    return out


def bench_stats(ms) -> dict:
    arr = (ctypes.c_double * len(ms))(*ms)
    s = BenchStats()
    check(lib().cs_bench_stats_from_ms(arr, len(ms), ctypes.byref(s)), "cs_bench_stats_from_ms")
    return {n: getattr(s, n) for n, _ in BenchStats._fields_}


def bench_report(ms, name: str, rows: int, cols: int, logical_bytes: float) -> str:
    arr = (ctypes.c_double * len(ms))(*ms)
    s = BenchStats()
    check(lib().cs_bench_stats_from_ms(arr, len(ms), ctypes.byref(s)), "cs_bench_stats_from_ms")
    buf = ctypes.create_string_buffer(512)
    lib().cs_bench_report(ctypes.byref(s), name.encode(), rows, cols, logical_bytes, buf, 512)
    return buf.value.decode()


def check_output(out, *, batch: int, rows: int, cols: int, pitch: int, row_offset: int = 0,
                 rowsum_tol: float = 2e-3) -> dict:
    """Oracle-free structural check of a uint16 output array (host memory)."""
    import numpy as np

    a = np.ascontiguousarray(out, dtype=np.uint16)
    rep = SelfCheck()
    lib().cs_check_output(a.ctypes.data, batch, rows * pitch, rows, cols, pitch, row_offset,
                          rowsum_tol, ctypes.byref(rep))
    return {n: getattr(rep, n) for n, _ in SelfCheck._fields_}


def parse_config(args: list[str]) -> dict:
    arr = (ctypes.c_char_p * max(1, len(args)))(*[a.encode() for a in args])
    cfg = Config()
    err = ctypes.create_string_buffer(1024)
    rc = lib().cs_config_parse(len(args), arr, ctypes.byref(cfg), err, 1024)
    if rc != 0:
        raise ValueError(err.value.decode())
    return {n: getattr(cfg, n) for n, _ in Config._fields_}
