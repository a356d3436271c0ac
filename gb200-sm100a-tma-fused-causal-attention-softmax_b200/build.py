"""Build recipe for the CUDA library (and CLI) of the B200 fused causal softmax.

    python build.py            # build lib/libcausal_softmax.so and bin/csm if stale
    python build.py --force    # rebuild

nvcc cross-compiles for sm_100a only (-gencode arch=compute_100a,code=sm_100a);
no GPU is needed to build. The ptxas resource report (registers, spills,
shared memory per kernel) is written to lib/ptxas.txt.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
INCLUDE = os.path.join(ROOT, "include")
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
BIN_DIR = os.path.join(HERE, "bin")
LIB_PATH = os.path.join(LIB_DIR, "libcausal_softmax.so")
CLI_PATH = os.path.join(BIN_DIR, "csm")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --fmad=false: no multiply-add contraction in device code. The kernels rely
# on x*scale being rounded exactly once (so the row maximum's exponent is
# exactly 0 after subtracting the rounded maximum), as the f32 specification
# rounds it; a contracted x*scale - max would leave the product's rounding
# residual, which at scale 1e30 is large enough to overflow exp.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler",
              "-fPIC,-ffp-contract=off", "--expt-relaxed-constexpr"]

LIB_SOURCES = [os.path.join(CSRC, "api.cu"), os.path.join(CSRC, "host", "host.cpp")]
CLI_SOURCES = [os.path.join(CSRC, "host", "cli.cpp")]


def _nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build the library")
    return path


def _inputs() -> list[str]:
    files = []
    for d in (CSRC, INCLUDE):
        for base, _, names in os.walk(d):
            files += [os.path.join(base, n) for n in names
                      if n.endswith((".cu", ".cuh", ".cpp", ".hpp", ".h"))]
    files.append(os.path.abspath(__file__))
    return files


def _stale(target: str) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(f) > t for f in _inputs())


class _BuildLock:
    """Inter-process lock so concurrent ranks or test workers build once."""

    def __enter__(self):
        import fcntl

        os.makedirs(LIB_DIR, exist_ok=True)
        self.fh = open(os.path.join(LIB_DIR, ".build.lock"), "w")
        fcntl.flock(self.fh, fcntl.LOCK_EX)
        return self

    def __exit__(self, *exc):
        import fcntl

        fcntl.flock(self.fh, fcntl.LOCK_UN)
        self.fh.close()


def build_library(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale(LIB_PATH):
        return LIB_PATH
    with _BuildLock():
        if not force and not _stale(LIB_PATH):
            return LIB_PATH
        return _build_library(verbose)


def _build_library(verbose: bool) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-Xptxas", "-v", "-shared", "-I", INCLUDE, "-I", CSRC,
           "-o", tmp, *LIB_SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libcausal_softmax.so")
    with open(os.path.join(LIB_DIR, "ptxas.txt"), "w") as fh:
        fh.write(" ".join(cmd) + "\n" + res.stderr)
    os.replace(tmp, LIB_PATH)
    if verbose:
        print(f"built {LIB_PATH}")
    return LIB_PATH


def build_cli(force: bool = False, verbose: bool = False) -> str | None:
    if not all(os.path.exists(s) for s in CLI_SOURCES):
        return None
    lib = build_library(force=force, verbose=verbose)
    if not force and os.path.exists(CLI_PATH) and os.path.getmtime(CLI_PATH) >= os.path.getmtime(lib) \
            and not _stale(CLI_PATH):
        return CLI_PATH
    os.makedirs(BIN_DIR, exist_ok=True)
    cmd = [_nvcc(), *ARCH, "-O2", "-std=c++17", "-I", INCLUDE, "-o", CLI_PATH, *CLI_SOURCES,
           "-L", LIB_DIR, "-lcausal_softmax", "-Xlinker", "-rpath,$ORIGIN/../lib", "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building the csm CLI")
    if verbose:
        print(f"built {CLI_PATH}")
    return CLI_PATH


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_cli(force=force, verbose=verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    build_all(force=args.force, verbose=True)
