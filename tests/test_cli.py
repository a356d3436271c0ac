"""The csm CLI (mirror of gpu/src/driver.rs:386-428 over the C ABI).

CPU: flag parsing and validation messages (host/src/lib.rs:103-182).
GPU: --probe, the --gpu-tests self-check matrix, and a --bench line.
"""
import os
import subprocess

import pytest

import build

CSM = build.CLI_PATH


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build_cli()
    assert os.path.exists(CSM)


def run(*args):
    return subprocess.run([CSM, *args], capture_output=True, text=True, timeout=600)


def test_help_and_errors():
    r = run("--help")
    assert r.returncode == 0 and "--probe" in r.stdout
    for args, msg in [(["--rows", "0"], "rows and cols must be positive"),
                      (["--scale", "NaN"], "scale must be finite"),
                      (["--cols", "33", "--kernel", "warp"], "warp specialization requires cols <= 32"),
                      (["--kernel", "wrong"], "unknown kernel"),
                      (["--x"], "unknown flag: --x"),
                      (["--cols"], "missing value for --cols"),
                      (["--cols", "2147483647"], "padded pitch exceeds device i32 indexing")]:
        r = run(*args)
        assert r.returncode == 2 and msg in r.stderr, (args, r.stderr)


@pytest.mark.gpu
def test_cli_on_gpu():
    r = run("--probe")
    assert r.returncode == 0 and "PASS probe" in r.stdout, r.stderr
    r = run("--gpu-tests")
    assert r.returncode == 0 and "PASS GPU self-checks" in r.stdout, r.stdout + r.stderr
    r = run("--rows", "1000", "--cols", "1037", "--scale", "0.0883883")
    assert r.returncode == 0 and r.stdout.startswith("PASS"), r.stdout + r.stderr
    r = run("--bench", "--rows", "2048", "--cols", "2048", "--iterations", "5", "--warmup", "2")
    assert r.returncode == 0 and r.stdout.count("BENCH kernel=") == 4, r.stdout + r.stderr
