"""CPU tests of bench.py's two arms.

The reference arm (--impl reference) times the oracle's restatement of the
reference CPU path and must load nothing of this package: no Python module of
it and not its CUDA library. Both arms print the same `config` object, so the
driver compares like with like; the oracle's copy of the seeded workload
generator gives the same bits as the library's.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_PROBE = r"""
import json, runpy, sys
sys.argv = ["bench.py"] + sys.argv[1:]
try:
    runpy.run_path("bench.py", run_name="__main__")
except SystemExit as e:
    assert not e.code, e.code
maps = open("/proc/self/maps").read()
print("PROBE " + json.dumps({
    "product_so": "libcausal_softmax" in maps,
    "oracle_so": "liboracle" in maps,
    "product_module": "causal_softmax" in sys.modules,
    "torch": "torch" in sys.modules,
}))
"""


def _run_reference(gpus, *args):
    # As torchrun starts rank 0 of `gpus` ranks (the other ranks exit at once).
    env = dict(os.environ, WORLD_SIZE=str(gpus), RANK="0")
    p = subprocess.run([sys.executable, "-c", _PROBE, "--impl", "reference", *args], cwd=ROOT,
                       env=env, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr
    lines = p.stdout.strip().splitlines()
    probe = json.loads(next(l for l in lines if l.startswith("PROBE "))[6:])
    line = json.loads(next(l for l in lines if l.startswith("{")))
    return line, probe


@pytest.mark.parametrize("workload,gpus", [("c2b", 1), ("c2a", 1), ("c4", 8)])
def test_reference_arm_loads_only_the_oracle(workload, gpus):
    line, probe = _run_reference(gpus, "--workload", workload, "--steps", "2", "--warmup", "3",
                                 "--gpus", str(gpus))
    assert probe == {"product_so": False, "oracle_so": True, "product_module": False,
                     "torch": False}, probe
    assert line["impl"] == "reference"
    assert line["value"] > 0 and line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert "whole" in line["cpu_baseline"]["sample"]

    sys.path.insert(0, ROOT)
    import bench

    args = bench.argparse.Namespace(workload=workload, weak=False, contiguous_rows=False,
                                    kernel="auto")
    cfg, scaling = bench.job_config(args, dict(bench.WORKLOADS[workload]), gpus)
    assert line["config"] == json.loads(json.dumps(cfg))  # identical to the GPU arm's config
    assert line["scaling"] == scaling == "strong"
    if workload == "c4":
        assert line["config"]["matrices"] == 256 and line["config"]["matrices_per_rank"] == 32


def test_oracle_generator_matches_library_generator():
    import causal_softmax as cs
    import oracle_ctypes as O

    for cfg, seed, (b, r, c, p, fb, fr) in [(1, 0, (1, 70, 4096, 4096, 0, 0)),
                                            (2, 1, (2, 50, 1037, 1040, 0, 5)),
                                            (3, 2, (1, 40, 8192, 8192, 0, 3000)),
                                            (4, 3, (3, 16, 4096, 4096, 7, 11)),
                                            (5, 4, (1, 8, 32768, 32768, 0, 20000)),
                                            (2, 1, (1, 4096, 32, 32, 0, 0))]:
        a = O.generate(cfg, seed, b, r, c, p, fb, fr)
        want = cs.generate(cfg, seed, batch=b, rows=r, cols=c, pitch=p, first_batch=fb, first_row=fr)
        assert np.array_equal(a, want), cfg
    for rows, cols, off in [(4096, 4096, 0), (100, 4096, 4000), (50, 4096, 5000), (1000, 1037, 0),
                            (4096, 32, 0), (1, 1, 0)]:
        assert O.roofline_bytes(rows, cols, off) == cs.roofline_bytes(rows, cols, off)
