"""Kernel micro-benchmarks timed with CUDA events (warm-up, L2 flush between
iterations, synchronize on both sides), reported against the measured peaks in
``MEASURED_PEAKS.json`` when present.

Usage::

    python -m oxidizr_b200.utils.kbench gemm [--shapes M,N,K ...]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def measured_peaks() -> dict:
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


_FLUSH = {}


def flush_l2(device=None):
    """Write a buffer larger than the 126 MB L2."""
    dev = torch.device(device or "cuda")
    buf = _FLUSH.get(dev)
    if buf is None:
        buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
        _FLUSH[dev] = buf
    buf.zero_()


def time_fn(fn, iters: int = 20, warmup: int = 5, flush: bool = True) -> float:
    """Median milliseconds per call."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            flush_l2()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return statistics.median(times)


def bench_gemm(shapes, iters=20):
    from ..ops.gemm import mm
    peaks = measured_peaks()
    rows = []
    for (M, N, K, lay) in shapes:
        a_t, b_t = lay[0] == "t", lay[1] == "t"
        a = torch.randn((K, M) if a_t else (M, K), device="cuda").bfloat16()
        b = torch.randn((K, N) if b_t else (N, K), device="cuda").bfloat16()
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ms = time_fn(lambda: mm(a, b, a_t=a_t, b_t=b_t, out=out), iters)
        A = a.t() if a_t else a
        B = b.t() if b_t else b
        ms_ref = time_fn(lambda: torch.matmul(A, B.t()), iters)
        tf = 2.0 * M * N * K / ms / 1e9
        tf_ref = 2.0 * M * N * K / ms_ref / 1e9
        rows.append({"M": M, "N": N, "K": K, "layout": lay, "ms": round(ms, 4), "tflops": round(tf, 1),
                     "frac_of_peak": round(tf / peaks["bf16_tflops"], 3), "peak_source": peaks["source"],
                     "torch_ms": round(ms_ref, 4), "torch_tflops": round(tf_ref, 1)})
        print(json.dumps(rows[-1]), flush=True)
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm"])
    ap.add_argument("--shapes", nargs="*", default=None, help="M,N,K[,layout] with layout nn|nt|tt")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    if args.what == "gemm":
        if args.shapes:
            shapes = []
            for s in args.shapes:
                parts = s.split(",")
                shapes.append((int(parts[0]), int(parts[1]), int(parts[2]), parts[3] if len(parts) > 3 else "nn"))
        else:
            T = 16384
            shapes = [(8192, 8192, 8192, "nn"), (T, 4096, 2048, "nn"), (T, 2048, 2048, "nn"),
                      (T, 11264, 2048, "nn"), (T, 2048, 5632, "nn"), (T, 2048, 5632, "nt"),
                      (5632, 2048, T, "tt"), (2048, 2048, T, "tt")]
        bench_gemm(shapes, args.iters)


if __name__ == "__main__":
    main()
