"""Access to the compiled kernel library and its per-device status word.

Every kernel receives a pointer to a small int32 status buffer on its device.
Bounded waits and debug checks record an error code there instead of trapping;
``check_status`` reads it back (a host sync) and raises if it is non-zero.
"""
from __future__ import annotations

import os

import torch

from .. import _ext

_STATUS = {}

ERRORS = {
    1: "pipeline wait timed out",
    2: "cross-GPU wait timed out",
    3: "bounds check failed",
    4: "non-finite value",
}


def raw_ext():
    """The extension module; raises if it cannot be built/loaded."""
    return _ext.load(required=True)


def ext():
    """The extension module (behind the launch-counting proxy)."""
    return counted_ext()


def status(device) -> torch.Tensor:
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(16, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = t
    return t


def read_status(device, reset: bool = True) -> int:
    s = status(device)
    v = int(s[0].item())
    if reset and v:
        s.zero_()
    return v


def check_status(device) -> None:
    v = read_status(device)
    if v:
        raise RuntimeError(f"oxidizr kernel status {v}: {ERRORS.get(v, 'unknown error')}")


class _Counter:
    """Counts calls into the kernel library (each call launches one kernel,
    except a handful that launch two; see ``LAUNCHES_PER_CALL``)."""

    LAUNCHES_PER_CALL = {"gemm_ce": 1, "adamw": 1}

    def __init__(self):
        self.enabled = False
        self.count = 0

    def wrap(self, mod):
        counter = self

        class _Proxy:
            def __getattr__(self, name):
                fn = getattr(mod, name)
                if not callable(fn):
                    return fn

                def call(*a, **k):
                    if counter.enabled:
                        counter.count += counter.LAUNCHES_PER_CALL.get(name, 1)
                    if not _DEBUG_SYNC:
                        return fn(*a, **k)
                    # debugging aid: find the first launch that faults (OXI_DEBUG_SYNC=1)
                    import torch
                    torch.cuda.synchronize()
                    r = fn(*a, **k)
                    try:
                        torch.cuda.synchronize()
                    except RuntimeError as e:
                        raise RuntimeError(f"oxidizr kernel call {name!r} failed: {e}") from e
                    return r
                return call

            def __dir__(self):
                return dir(mod)

        return _Proxy()


_DEBUG_SYNC = os.environ.get("OXI_DEBUG_SYNC") == "1"
launch_counter = _Counter()
_PROXY = None


def counted_ext():
    """The extension behind a proxy that counts kernel launches while enabled."""
    global _PROXY
    if _PROXY is None:
        _PROXY = launch_counter.wrap(raw_ext())
    return _PROXY
