"""Static resource gate over the library's ptxas report (no GPU needed).

Plays the part of the reference's scripts/check_resources.py:15-59 (registers,
spills and occupancy per kernel entry), but reads the `-Xptxas -v` report
that every build writes to lib/ptxas.txt instead of compiled code. Rules:

* every kernel entry is reported once, compiled for sm_100a, with no ptxas
  error;
* a row-resident variant rowres_kernel<V, MAXT, MINB, store> keeps the
  residency its launch bounds promise: MINB CTAs of MAXT threads fit one SM,
  counting registers per SM sub-partition (16384 each; a CTA's warps are
  spread over the four, allocation in units of 256 registers per warp);
* spills are zero, except where BUDGETS grants a byte allowance with its
  reason; registers stay under the BUDGETS cap where one is set.

    python -m causal_softmax.resources [path/to/ptxas.txt]
"""
from __future__ import annotations

import math
import os
import re
import sys

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPORT = os.path.join(PKG_DIR, "lib", "ptxas.txt")

REGS_PER_SMSP = 16384
SMSP_PER_SM = 4

# (pattern on the readable name, max registers or None, spill store + load
# bytes allowed, reason)
BUDGETS = [
    (r"rowres_kernel<4, 224, 4, [01]>", 72, 128,
     "auto's choice for ~3000-5000-column rows: four CTAs per SM cap it at 72 registers; "
     "its few spilled bytes cost ~1% of the instructions (ncu), the occupancy is worth more"),
    (r"rowres_kernel<8, 448, 1, [01]>", 128, 0,
     "V = 8 at up to 14 warps; only a tuning request selects it since the shared-memory "
     "variant (V = 0) serves long rows"),
    (r"online_kernel<[12]>", 64, 0, "launch bounds of 1024 threads (the long-row shape)"),
    (r"cluster_kernel", 64, 0, "shared-memory passes with 17 warps per CTA; nothing to keep in registers"),
    (r"rowres_kernel<8, 256, 1, [01]>", 168, 0, "V = 8 at up to 8 warps; tuning request only"),
    (r"rowres_kernel<0, 1024, 1, [01]>", 64, 0, "shared-memory passes, 32 warps in one CTA"),
]

_ENTRY = re.compile(r"Compiling entry function '([^']+)' for '([^']+)'")
_PROPS = re.compile(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads")
_REGS = re.compile(r"Used (\d+) registers")
_ROWRES = re.compile(r"rowres_kernelILi(\d+)ELi(\d+)ELi(\d+)ELb([01])E")


def readable(mangled: str) -> str:
    m = _ROWRES.search(mangled)
    if m:
        return "rowres_kernel<%s, %s, %s, %s>" % m.groups()
    m = re.search(r"narrow_kernelILi(\d+)E", mangled)
    if m:
        return f"narrow_kernel<{m.group(1)}>"
    m = re.search(r"online_kernelILi(\d+)E", mangled)
    if m:
        return f"online_kernel<{m.group(1)}>"
    m = re.search(r"_ZN2cs\d+(\w+?)E", mangled)
    return m.group(1) if m else mangled


def parse_report(text: str) -> tuple[dict, list[str]]:
    """Per-kernel resources {mangled: {...}} and the problems found while reading."""
    problems = []
    if re.search(r"ptxas\s+(fatal|error)", text, re.I):
        problems.append("ptxas reported an error")
    starts = list(_ENTRY.finditer(text))
    if not starts:
        return {}, problems + ["no per-kernel reports"]
    kernels = {}
    for i, m in enumerate(starts):
        name, arch = m.groups()
        body = text[m.end():starts[i + 1].start() if i + 1 < len(starts) else len(text)]
        props, regs = _PROPS.search(body), _REGS.search(body)
        if name in kernels:
            problems.append(f"duplicate report for {readable(name)}")
            continue
        if arch != "sm_100a" or props is None or regs is None:
            problems.append(f"incomplete or wrong-target report for {readable(name)} ({arch})")
            continue
        stack, st, ld = map(int, props.groups())
        kernels[name] = {"name": readable(name), "arch": arch, "registers": int(regs.group(1)),
                         "stack_bytes": stack, "spill_store_bytes": st, "spill_load_bytes": ld}
    return kernels, problems


def resident_ctas(registers: int, threads: int) -> int:
    """CTAs of `threads` threads one SM holds by registers alone."""
    per_warp = math.ceil(registers * 32 / 256) * 256
    warps = math.ceil(threads / 32)
    n = 0
    while True:
        # A CTA's warps spread round-robin over the sub-partitions.
        per_smsp = math.ceil((n + 1) * warps / SMSP_PER_SM)
        if per_smsp * per_warp > REGS_PER_SMSP:
            return n
        n += 1


def check(text: str) -> tuple[list[str], dict]:
    kernels, problems = parse_report(text)
    for k in kernels.values():
        name, regs = k["name"], k["registers"]
        spill = k["spill_store_bytes"] + k["spill_load_bytes"]
        budget = next((b for b in BUDGETS if re.fullmatch(b[0], name)), None)
        max_regs, max_spill = (budget[1], budget[2]) if budget else (None, 0)
        if spill > max_spill:
            problems.append(f"{name}: {spill} spill bytes (allowed {max_spill})")
        if max_regs is not None and regs > max_regs:
            problems.append(f"{name}: {regs} registers (cap {max_regs})")
        m = re.fullmatch(r"rowres_kernel<(\d+), (\d+), (\d+), [01]>", name)
        if m:
            maxt, minb = int(m.group(2)), int(m.group(3))
            got = resident_ctas(regs, maxt)
            if got < minb:
                problems.append(f"{name}: {regs} registers hold {got} CTAs of {maxt} threads, "
                                f"launch bounds promise {minb}")
    return problems, kernels


def main(argv=None) -> int:
    path = (argv or sys.argv[1:] or [REPORT])[0]
    with open(path, encoding="utf-8") as fh:
        problems, kernels = check(fh.read())
    for k in sorted(kernels.values(), key=lambda k: k["name"]):
        print(f"{k['name']:<36} regs {k['registers']:>3}  stack {k['stack_bytes']:>4}  "
              f"spill st/ld {k['spill_store_bytes']}/{k['spill_load_bytes']}")
    for p in problems:
        print("FAIL", p)
    print("PASS" if not problems else f"{len(problems)} problem(s)")
    return 1 if problems else 0


if __name__ == "__main__":
    sys.exit(main())
