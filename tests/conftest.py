"""Shared pytest setup: the `gpu` marker and import paths.

CPU tests (`-m "not gpu"`) cover the oracle against the reference's known
answers, the host-side logic and the C-ABI library's exports. GPU tests
(`-m gpu`) run the CUDA kernels through the C ABI and compare with the oracle.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "gb200-sm100a-tma-fused-causal-attention-softmax_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")
for p in (PKG_DIR, ORACLE_DIR, os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Rows whose row sum was accepted through the FP64 oracle's own FP16
    rounding error (gpu_helpers.FLOOR_LOG), per checked case."""
    mod = sys.modules.get("gpu_helpers")
    if mod is None or not hasattr(mod, "FLOOR_LOG"):
        return
    log = mod.FLOOR_LOG
    tr = terminalreporter
    tr.write_sep("-", f"row sums accepted through the oracle's own error: {len(log)} case(s)")
    if not log:
        return
    worst = max(e["max_excess"] for e in log)
    tr.write_line(f"largest excess over the exactly rounded result: {worst:.3g} "
                  f"(allowed {mod.ROWSUM_FLOOR_MARGIN:g})")
    for e in log:
        tr.write_line(f"  {e['what']}: {e['rows']} of {e['checked']} rows, excess <= "
                      f"{e['max_excess']:.3g}, oracle's own error up to {e['oracle_max_rowsum_err']:.3g}")
