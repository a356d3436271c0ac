"""Helpers for the GPU parity tests: move uint16 half bits to/from the device
with torch (plumbing only), launch through the C ABI, and compare against the
CPU oracle. Test infrastructure.

Tolerances (the acceptance bar of this library, checked against the FP64
oracle rounded to half): masked entries bit-exact 0x0000; unmasked within
ULP_TOL FP16 ulp or ABS_TOL absolute; |row sum - 1| <= ROWSUM_TOL. A row
whose exactly rounded FP64 result already misses ROWSUM_TOL (FP16 rounding
of many small probabilities, e.g. uniform rows of ~70000+ columns) may miss
it by that much (ROWSUM_FLOOR_MARGIN = 0: no worse than exact rounding);
every such row is recorded in FLOOR_LOG and counted at the end of the test
session. No case of the suite has needed it on a B200. The f32
specification (reference/src/lib.rs:85-108) is held to the same element
bound, and the reference's own verifier (host/src/lib.rs:280-328: 0.003 +
0.003*w per element, 0.02 per row sum, non-negative, finite, masked == 0)
must accept the output.
"""
from __future__ import annotations

import numpy as np
import torch

import causal_softmax as cs
import oracle_ctypes as O

ABS_TOL = 2e-3
ULP_TOL = 2
ROWSUM_TOL = 2e-3
ROWSUM_FLOOR_MARGIN = 0.0
FLOOR_LOG: list[dict] = []
SENTINEL = 0xFB00  # gpu/src/driver.rs:78-79

KERNELS = ["baseline", "warp", "tma", "pipeline", "online"]


def supported(kernel: str, cols: int) -> bool:
    return kernel != "warp" or cols <= 32


def to_dev(x: np.ndarray) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(x).view(np.int16))
    return t.cuda().view(torch.float16)


def from_dev(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def sentinel_like(t: torch.Tensor) -> torch.Tensor:
    s = np.int16(np.uint16(SENTINEL).view(np.int16))
    return torch.full(t.shape, int(s), dtype=torch.int16, device=t.device).view(torch.float16)


def run(kernel: str, x: np.ndarray, *, cols: int, scale: float, row_offset: int = 0,
        tuning: tuple | None = None) -> np.ndarray:
    """Run one plan launch on x ([batch,] rows, pitch uint16) into a sentinel-filled output."""
    d_in = to_dev(x)
    d_out = sentinel_like(d_in)
    with cs.Plan.for_tensors(d_in, d_out, cols=cols, row_offset=row_offset) as plan:
        if tuning:
            plan.set_tuning(*tuning)
        plan.launch(kernel, scale)
        rc, status = plan.status()
        assert rc == 0 and status == 0, (rc, status)
    torch.cuda.synchronize()
    return from_dev(d_out)


def layout(x: np.ndarray):
    batch = x.shape[0] if x.ndim == 3 else 1
    rows, pitch = x.shape[-2], x.shape[-1]
    return batch, rows, pitch


def check(got: np.ndarray, x: np.ndarray, *, cols: int, scale: float, row_offset: int = 0,
          what: str = "") -> dict:
    """Assert the acceptance bar against the FP64 oracle and the element
    bound against the f32 specification; returns the acceptance report."""
    batch, rows, pitch = layout(x)
    flat_x, flat_g = x.reshape(-1), got.reshape(-1)
    ref64 = O.softmax_strided(flat_x, batch, rows * pitch, rows, cols, pitch, row_offset, scale,
                              f64=True)
    rep = O.accept(flat_g, ref64, batch, rows * pitch, rows, cols, pitch, row_offset,
                   ABS_TOL, ULP_TOL, ROWSUM_TOL, ROWSUM_FLOOR_MARGIN)
    if rep["floor_rows"]:
        FLOOR_LOG.append({"what": what, "rows": rep["floor_rows"], "checked": rep["checked_rows"],
                          "max_excess": rep["max_floor_excess"],
                          "oracle_max_rowsum_err": rep["oracle_max_rowsum_err"]})
    assert rep["ok"], f"{what}: FP64 acceptance failed {rep}"
    spec = O.softmax_strided(flat_x, batch, rows * pitch, rows, cols, pitch, row_offset, scale)
    rep32 = O.accept(flat_g, spec, batch, rows * pitch, rows, cols, pitch, row_offset,
                     ABS_TOL, ULP_TOL, 1.0)
    assert rep32["elem_violations"] == 0 and rep32["mask_violations"] == 0, \
        f"{what}: f32-spec comparison failed {rep32}"
    rep["max_ulp_vs_f32_spec"] = rep32["max_ulp"]
    rep["bitwise_equal_f32_spec"] = float(np.mean(flat_g == spec))
    if row_offset == 0:
        for b in range(batch):
            g = O.unpad(got.reshape(batch, rows, pitch)[b].ravel(), rows, cols)
            w = O.unpad(spec.reshape(batch, rows, pitch)[b].ravel(), rows, cols)
            name, acc = O.verify(g, w, rows, cols)
            assert name == "ok", f"{what}: reference verifier says {name} at {acc.index}"
    return rep


def pattern_input(rows: int, cols: int, pattern: str, seed: int = 0x13579BDF) -> np.ndarray:
    """host/src/lib.rs:218-256 input, padded to the 16-byte pitch (reference/src/lib.rs:136-143)."""
    dense = cs.make_input(rows, cols, pattern, seed)
    return O.pad(dense, rows, cols).reshape(rows, cs.padded_pitch(cols))
