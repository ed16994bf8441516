"""NVLink peer-access microbenchmark (one process, two GPUs).

    python -m oxidizr_b200.utils.p2pbench [--mb 1024]

GPU 0 reads from / writes to a buffer on GPU 1 (peer access through NVSwitch)
and, for comparison, its own memory, with: SM loads, SM stores (CTAs x
threads x 16-byte vectors in flight per thread), bulk copies through the TMA
engine (chunk bytes x stages in flight per CTA), and the copy engine
(cudaMemcpyPeerAsync via torch).  Prints one JSON line per configuration and
a summary of the best of each kind (GB/s, CUDA-event timed after warm-up).
The kernels are in the separate tools extension (csrc/tools/), not in the
training library.
"""
from __future__ import annotations

import argparse
import json

import torch


def _time(fn, iters=5):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--mb", type=int, default=1024)
    args = ap.parse_args(argv)
    from .. import _ext
    from ..ops._C import ext, status
    assert torch.cuda.device_count() >= 2, "needs two GPUs"
    ok = ext().enable_peer_access(0, 1)
    e = _ext.load_tools()
    nbytes = args.mb << 20
    torch.cuda.set_device(0)
    remote = torch.empty(nbytes, dtype=torch.uint8, device="cuda:1")
    local = torch.empty(nbytes, dtype=torch.uint8, device="cuda:0")
    sink = torch.zeros(4, dtype=torch.int32, device="cuda:0")
    st = status("cuda:0")
    best = {}
    rows = []

    def rec(kind, where, cfg, ms):
        gbs = nbytes / (ms * 1e-3) / 1e9
        rows.append({"kind": kind, "where": where, **cfg, "ms": round(ms, 3), "GBps": round(gbs, 1)})
        key = f"{kind}_{where}"
        if gbs > best.get(key, (0, None))[0]:
            best[key] = (round(gbs, 1), cfg)

    for where, buf in (("peer", remote), ("local", local)):
        ptr = buf.data_ptr()
        for ctas in (16, 32, 64, 148, 296):
            for threads in (256, 512):
                for unr in (4, 8, 16):
                    cfg = {"ctas": ctas, "threads": threads, "unroll": unr}
                    rec("sm_load", where, cfg, _time(lambda: e.p2p_read(ptr, nbytes, sink, ctas, threads, unr)))
                    rec("sm_store", where, cfg, _time(lambda: e.p2p_write(ptr, nbytes, sink, ctas, threads, unr)))
        for ctas in (16, 32, 64, 148):
            for chunk in (4096, 16384, 32768):
                for stages in (2, 4, 8):
                    if chunk * stages > 96 * 1024:
                        continue
                    cfg = {"ctas": ctas, "chunk": chunk, "stages": stages}
                    rec("bulk_load", where, cfg, _time(lambda: e.p2p_bulk(False, ptr, nbytes, ctas, chunk, stages, st)))
                    rec("bulk_store", where, cfg, _time(lambda: e.p2p_bulk(True, ptr, nbytes, ctas, chunk, stages, st)))
    rec("copy_engine", "peer", {}, _time(lambda: remote.copy_(local, non_blocking=True)))
    torch.cuda.synchronize()
    for r in rows:
        print(json.dumps(r))
    print(json.dumps({"peer_access": ok, "bytes": nbytes, "best": best}))


if __name__ == "__main__":
    main()
