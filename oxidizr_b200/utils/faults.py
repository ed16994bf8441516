"""Host-side fault injection and profiling hooks for the training loop.

``OXI_FAULT="rank:step:kind[,rank:step:kind...]"`` makes rank ``rank`` fail at
the start of optimizer step ``step`` (0-based global step) in one of these ways:

* ``raise`` -- raise ``InjectedFault`` (the process exits with an error);
* ``exit``  -- leave the process at once with exit code 17, no cleanup;
* ``hang``  -- stop joining the collectives (sleep), with no kernel in flight;
* ``nan``   -- make this step's loss NaN (exercises the non-finite check).

Every failure is made on the host between steps, never on the GPU: the other
ranks learn of it through the process group (an error or its timeout) and the
launcher's watchdog.  Upstream has no fault injection; its failure handling is
the NaN check of the loss (trainer.rs:153-214) and the run.json status
(commands/train.rs:721-726), which this framework keeps.

``OXI_NVTX=1`` wraps forward / backward / optimizer in NVTX ranges, and
``OXI_PROFILE_STEPS="a:b"`` calls cudaProfilerStart at step a and
cudaProfilerStop at step b, so a profiler started with capture disabled
records only that window.
"""
from __future__ import annotations

import contextlib
import os
import time
from typing import Dict, Optional, Tuple


class InjectedFault(RuntimeError):
    pass


def _parse(spec: str) -> Dict[Tuple[int, int], str]:
    out = {}
    for item in filter(None, (s.strip() for s in spec.split(","))):
        r, st, kind = item.split(":")
        if kind not in ("raise", "exit", "hang", "nan"):
            raise ValueError(f"OXI_FAULT: unknown kind {kind!r}")
        out[(int(r), int(st))] = kind
    return out


_plan: Optional[Dict[Tuple[int, int], str]] = None


def fault_for(rank: int, step: int) -> Optional[str]:
    """The fault kind planned for (rank, step), if any (``nan`` is returned, not applied)."""
    global _plan
    if _plan is None:
        _plan = _parse(os.environ.get("OXI_FAULT", ""))
    kind = _plan.get((rank, step))
    if kind == "raise":
        raise InjectedFault(f"injected fault on rank {rank} at step {step}")
    if kind == "exit":
        os._exit(17)
    if kind == "hang":
        time.sleep(float(os.environ.get("OXI_FAULT_HANG_S", "3600")))
    return kind


def nvtx_range(name: str):
    if os.environ.get("OXI_NVTX") != "1":
        return contextlib.nullcontext()
    import torch
    return torch.cuda.nvtx.range(name)


def profile_window(step: int) -> None:
    spec = os.environ.get("OXI_PROFILE_STEPS")
    if not spec:
        return
    a, b = (int(x) for x in spec.split(":"))
    import torch
    if step == a:
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
    elif step == b:
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
