#!/usr/bin/env python3
"""Run the reference suite's own Triton kernels, unmodified, on a B200.

The reference suite (huangyiqun/triton_chip_benchmarks) is plain Python +
Triton, driven through FlagGems.  This script runs its ``bench_suite.py`` as
is, with ``baseline/flag_gems`` (a FlagGems stand-in over torch.cuda) on the
import path, so its 17-row table can be set beside this repository's on the
same GPU.

    python baseline/triton_suite.py --install /path/to/reference   # once, here
    python baseline/triton_suite.py --output out/triton_suite.json [suite flags]
    python baseline/triton_suite.py --child bench_vector --output out/v.json --dtype bf16 ...

``--install`` copies the reference's top-level Python modules into
``baseline/_ref`` (git-ignored; it travels with the working tree to the GPU
box).  Every other flag goes to the reference's ``bench_suite.py`` unchanged
(``--device``, ``--timing``, ``--quick``, ``--metrics``, ``--timeout`` ...).
With ``--compare OURS.json`` the two tables are printed side by side.
``--summary IN OUT`` writes a compact copy of a suite JSON (rows without
command lines or file paths) for the repository's results.
``--child NAME`` runs one of the reference's per-metric scripts (``NAME.py``:
bench_bandwidth, bench_tensor, bench_vector) the same way, for a single row
(the reference's suite runner has no metric filter).
"""

from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
import shutil
import subprocess
import sys

HERE = Path(__file__).resolve().parent
REF = HERE / "_ref"


def install(source: Path) -> None:
    modules = sorted(source.glob("*.py"))
    if not any(m.name == "bench_suite.py" for m in modules):
        raise SystemExit(f"{source} does not hold the reference suite (no bench_suite.py)")
    REF.mkdir(exist_ok=True)
    for module in modules:
        shutil.copy2(module, REF / module.name)
    print(f"copied {len(modules)} modules into {REF}")


def run(suite_args: list[str], output: Path, script: str = "bench_suite") -> int:
    if not (REF / f"{script}.py").exists():
        raise SystemExit(f"{REF / (script + '.py')} is missing; run with --install <reference "
                         "checkout> first")
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join(
        [str(HERE), str(REF)] + ([env["PYTHONPATH"]] if env.get("PYTHONPATH") else []))
    output.parent.mkdir(parents=True, exist_ok=True)
    command = [sys.executable, "-u", str(REF / f"{script}.py"), "--output", str(output),
               *suite_args]
    print("running:", " ".join(command), flush=True)
    return subprocess.run(command, env=env, check=False).returncode


ROW_KEYS = ("metric", "group", "precision", "unit", "status", "value", "median_value",
            "timing_method", "configuration", "reason", "successful_configurations")


def summary(source: Path, out: Path) -> None:
    doc = json.loads(source.read_text())
    rows = []
    for row in doc["results"]:
        kept = {k: row[k] for k in ROW_KEYS if k in row}
        if "patterns" in row:
            kept["patterns"] = {name: {k: v for k, v in pattern.items()
                                       if k in ("value", "median_value", "configuration")}
                                for name, pattern in row["patterns"].items()}
        rows.append(kept)
    device = {k: v for k, v in doc.get("device", {}).items()
              if k in ("device_name", "architecture", "sm_count", "memory_capacity_gib")}
    out.write_text(json.dumps({"benchmark": doc.get("benchmark"), "status": doc.get("status"),
                               "timestamp_utc": doc.get("timestamp_utc"), "device": device,
                               "measurement_policy": doc.get("measurement_policy"),
                               "results": rows}, indent=1) + "\n")


def compare(reference: Path, ours: Path) -> None:
    theirs = {r["metric"]: r for r in json.loads(reference.read_text())["results"]}
    mine = {r["metric"]: r for r in json.loads(ours.read_text())["results"]}
    print(f"\n{'metric':<20} {'Triton (reference)':>22} {'libtcb':>22} {'ratio':>8}")
    for key, row in mine.items():
        other = theirs.get(key, {})

        def cell(r):
            v = r.get("value")
            return f"{v:.2f} {r.get('status', '')}" if v is not None else r.get("status", "-")

        ratio = (f"{row['value'] / other['value']:.2f}" if row.get("value") and other.get("value")
                 else "-")
        print(f"{key:<20} {cell(other):>22} {cell(row):>22} {ratio:>8}")


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--install", type=Path, metavar="REFERENCE",
                        help="copy the reference suite's modules into baseline/_ref and exit")
    parser.add_argument("--output", type=Path, default=Path("triton_suite.json"))
    parser.add_argument("--compare", type=Path, metavar="OURS",
                        help="print this repository's table JSON beside the reference's")
    parser.add_argument("--summary", type=Path, nargs=2, metavar=("SUITE_JSON", "OUT"),
                        help="write a compact copy of a suite JSON and exit")
    parser.add_argument("--child", choices=("bench_bandwidth", "bench_tensor", "bench_vector"),
                        help="run one per-metric script of the reference instead of its suite")
    args, suite_args = parser.parse_known_args()
    if args.install is not None:
        install(args.install)
        return 0
    if args.summary is not None:
        summary(*args.summary)
        return 0
    rc = run(suite_args, args.output, args.child or "bench_suite")
    if args.child is None and args.compare is not None and args.output.exists():
        compare(args.output, args.compare)
    return rc


if __name__ == "__main__":
    raise SystemExit(main())
