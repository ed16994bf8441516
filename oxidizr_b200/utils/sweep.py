"""Training-throughput sweep over (sequence length, batch size, gradient accumulation), the
framework's counterpart of the reference's ``run_benchmark.sh`` (run_benchmark.sh:46-183).

    python -m oxidizr_b200.utils.sweep [-f config.yaml] [--grid S,B,G ...] [--max-steps N] [-- train args]

Each grid point runs ``oxidizr train --headless --seq-len S --batch-size B --grad-accum G
--max-steps N`` (plus any arguments after ``--``, e.g. ``-d tokens.bin --target-device cpu``) in its
own process and records its last ``{"step": ...}`` line.  Output, as upstream:
``benchmark/<timestamp>/logs.txt`` (every run's full output) and ``results.csv`` with the columns
``seq_length,batch_size,gradient_accumulation,effective_batch,vram_usage_mb,samples_per_s,notes``;
``notes`` is empty on success, else ``OOM``, ``ERROR``, ``TIMEOUT``, ``UNKNOWN_ERROR`` or
``NO_OUTPUT``.  Unlike upstream's parser (which looks for ``{'step':`` and so records every run as
``NO_OUTPUT``) the trainer's JSON lines are read as JSON.  ``samples_per_s`` is the headless
``it/s`` field (samples per second since the start).  For device-timed tokens/s of the
benchmark configs use ``bench.py``.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
from typing import List, Optional, Sequence, Tuple

# the upstream grid: every sequence length with batch 1..5 and accumulation 1..2
DEFAULT_GRID: List[Tuple[int, int, int]] = [(s, b, g) for s in (128, 256, 384, 512, 1024)
                                            for b in range(1, 6) for g in (1, 2)]
HEADER = "seq_length,batch_size,gradient_accumulation,effective_batch,vram_usage_mb,samples_per_s,notes"


def parse_grid(items: Sequence[str]) -> List[Tuple[int, int, int]]:
    out = []
    for it in items:
        s, b, g = (int(x) for x in it.split(","))
        out.append((s, b, g))
    return out


def classify(rc: Optional[int], output: str) -> Tuple[str, Optional[dict]]:
    """(notes, last step record) of one run."""
    if rc is None:
        return "TIMEOUT", None
    if rc != 0:
        low = output.lower()
        if "out of memory" in low or "out_of_memory" in low:
            return "OOM", None
        if "error" in low or "failed" in low or "traceback" in low:
            return "ERROR", None
        return "UNKNOWN_ERROR", None
    last = None
    for line in output.splitlines():
        if line.startswith('{"step"'):
            try:
                last = json.loads(line)
            except json.JSONDecodeError:
                continue
    return ("", last) if last is not None else ("NO_OUTPUT", None)


def csv_row(seq: int, batch: int, grad: int, notes: str, rec: Optional[dict]) -> str:
    vram = rec.get("vram", "") if rec else ""
    its = rec.get("it/s", "") if rec else ""
    return f"{seq},{batch},{grad},{batch * grad},{vram},{its},{notes}"


def run(grid, config: Optional[str], max_steps: int, extra: Sequence[str], out_root: str, timeout: float,
        python: str = sys.executable) -> str:
    stamp = datetime.datetime.now().strftime("%Y%m%d_%H%M%S")
    bench_dir = os.path.join(out_root, stamp)
    os.makedirs(bench_dir, exist_ok=True)
    logs = os.path.join(bench_dir, "logs.txt")
    results = os.path.join(bench_dir, "results.csv")
    with open(results, "w") as fh:
        fh.write(HEADER + "\n")
    with open(logs, "w") as fh:
        fh.write(f"=== Oxidizr Benchmark Run ===\nTimestamp: {stamp}\n")
        if config:
            fh.write(f"Config: {config}\n")
        fh.write("=" * 38 + "\n\n")
    repo = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    env = dict(os.environ, PYTHONPATH=os.pathsep.join(p for p in (repo, os.environ.get("PYTHONPATH")) if p))
    for seq, batch, grad in grid:
        cmd = [python, "-m", "oxidizr_b200", "train", *(["-f", config] if config else []), "--headless",
               "--seq-len", str(seq), "--batch-size", str(batch), "--grad-accum", str(grad),
               "--max-steps", str(max_steps), *extra]
        print(f"Running: seq={seq}, batch={batch}, grad_accum={grad}", flush=True)
        # each point's run.json / steps.json go under the sweep's own directory,
        # never into the caller's working directory
        env["OXIDIZED_RUN_DIR"] = os.path.join(bench_dir, "runs", f"seq{seq}_b{batch}_g{grad}")
        try:
            r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)
            rc, output = r.returncode, r.stdout + r.stderr
        except subprocess.TimeoutExpired as e:
            rc = None
            output = (e.stdout or "") if isinstance(e.stdout, str) else ""
        notes, rec = classify(rc, output)
        with open(logs, "a") as fh:
            fh.write(f"Running: seq={seq}, batch={batch}, grad_accum={grad}\n--- Full Output ---\n{output}\n"
                     f"--- Exit Code: {rc} ---\n\n")
        with open(results, "a") as fh:
            fh.write(csv_row(seq, batch, grad, notes, rec) + "\n")
        print(f"  Result: {notes or 'SUCCESS'}" + (f" it/s={rec['it/s']} vram={rec['vram']}MB" if rec else ""),
              flush=True)
    print(f"Results: {results}")
    return results


def main(argv: Optional[Sequence[str]] = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    extra: List[str] = []
    if "--" in argv:
        i = argv.index("--")
        argv, extra = argv[:i], argv[i + 1:]
    ap = argparse.ArgumentParser(description="throughput sweep over (seq, batch, grad accumulation)")
    ap.add_argument("-f", "--config", default=None)
    ap.add_argument("--grid", nargs="*", default=None, help="S,B,G triples (default: the 50-point upstream grid)")
    ap.add_argument("--max-steps", type=int, default=1)
    ap.add_argument("--out", default="benchmark")
    ap.add_argument("--timeout", type=float, default=1800.0, help="seconds per grid point")
    a = ap.parse_args(argv)
    grid = parse_grid(a.grid) if a.grid else DEFAULT_GRID
    run(grid, a.config, a.max_steps, extra, a.out, a.timeout)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
