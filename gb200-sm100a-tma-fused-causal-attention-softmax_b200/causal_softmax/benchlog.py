"""BENCH lines (csm --bench / --bench-suite) to typed JSON records.

Plays the part of the reference's scripts/summarize_bench.py:11-61 for this
library's report format (host/src/lib.rs:383-406, which cs_bench_report
mirrors): every `BENCH key=value ...` line with a timing becomes one record;
integer fields are typed as integers, timings and rates as floats; a line
whose numbers are negative or not finite, or that lacks its category, kernel
or a positive shape, is an error with its line number.

    python -m causal_softmax.benchlog suite.txt [--output suite.json]
"""
from __future__ import annotations

import argparse
import json
import math
import sys

INT_KEYS = {"rows", "cols", "n", "streams", "queued", "calls_per_stream", "batch", "sms",
            "warmup", "repetitions", "verify"}
FLOAT_SUFFIXES = ("_ms", "_GBps", "_per_s", "_pct", "_speedup", "_bytes")


def parse_line(line: str) -> dict | None:
    """One record, or None for lines without a timing (headers, other output)."""
    line = line.strip()
    if not line.startswith("BENCH "):
        return None
    rec: dict = {}
    for tok in line.split()[1:]:
        key, sep, val = tok.partition("=")
        if not sep or not key or not val:
            continue
        if key in INT_KEYS:
            rec[key] = int(val)
        elif key.endswith(FLOAT_SUFFIXES) or key == "scale" or key.startswith("speedup_"):
            x = float(val)
            if not math.isfinite(x) or x < 0:
                raise ValueError(f"invalid number {key}={val}")
            rec[key] = x
        else:
            rec[key] = val
    if "median_ms" not in rec and "batch_p50_ms" not in rec:
        return None
    if "category" not in rec:
        raise ValueError("timing without a category")
    if "kernel" not in rec:
        raise ValueError("timing without a kernel")
    if rec.get("rows", 0) <= 0 or rec.get("cols", 0) <= 0:
        raise ValueError("timing without a positive shape")
    return rec


def parse_log(text: str) -> list[dict]:
    out = []
    for i, line in enumerate(text.splitlines(), 1):
        try:
            rec = parse_line(line)
        except (ValueError, OverflowError) as e:
            raise ValueError(f"line {i}: {e}") from e
        if rec is not None:
            out.append(rec)
    if not out:
        raise ValueError("no timing records")
    return out


def summarize(text: str, source: str = "") -> dict:
    recs = parse_log(text)
    cats: dict[str, int] = {}
    for r in recs:
        cats[r["category"]] = cats.get(r["category"], 0) + 1
    return {"source_file": source, "record_count": len(recs), "categories": cats, "records": recs}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("log")
    ap.add_argument("--output")
    a = ap.parse_args(argv)
    with open(a.log, encoding="utf-8") as fh:
        doc = summarize(fh.read(), a.log)
    text = json.dumps(doc, indent=2, sort_keys=True) + "\n"
    if a.output:
        with open(a.output, "w", encoding="utf-8") as fh:
            fh.write(text)
    else:
        sys.stdout.write(text)
    return 0


if __name__ == "__main__":
    sys.exit(main())
