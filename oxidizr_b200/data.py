"""Token data pipeline: raw u32 token files, rank sharding, prefetch, H2D.

Upstream: ``src/data.rs`` (``LitDataLoader`` 45-243, ``PrefetchDataLoader``
344-523, ``create_dummy_data`` 256-262, ``write_tokens_to_file`` 274-291).
The heavy lifting (mmap, slicing, the prefetch thread) is the native
``oxidizr_b200_data`` module built from ``csrc_host/dataloader.cpp``.

``next_batch()`` returns ``(inputs, targets)`` as ``int64 [B, S]`` tensors on the
loader's device.  On CUDA the [B, S+1] block is copied from a pinned slot with
a non-blocking copy on the current stream.
"""
from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys
import threading
from typing import Optional, Tuple

import numpy as np
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_BUILD = os.path.join(REPO, "build", "oxidizr_b200_data")
_SRC = os.path.join(REPO, "csrc_host", "dataloader.cpp")
_lock = threading.Lock()
_mod = None


def _native():
    global _mod
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is not None:
            return _mod
        so = os.path.join(_BUILD, "oxidizr_b200_data.so")
        if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(_SRC):
            os.makedirs(_BUILD, exist_ok=True)
            from torch.utils.cpp_extension import load
            from ._ext import _clear_stale_lock
            _clear_stale_lock(_BUILD)
            _mod = load(name="oxidizr_b200_data", sources=[_SRC], extra_cflags=["-O3", "-std=c++17"],
                        build_directory=_BUILD, with_cuda=False, verbose=False)
        else:
            loader = importlib.machinery.ExtensionFileLoader("oxidizr_b200_data", so)
            spec = importlib.util.spec_from_file_location("oxidizr_b200_data", so, loader=loader)
            _mod = importlib.util.module_from_spec(spec)
            loader.exec_module(_mod)
            sys.modules["oxidizr_b200_data"] = _mod
        return _mod


def synthetic_tokens(vocab_size: int, total_tokens: int, seed: int = 0) -> np.ndarray:
    """Seeded uniform u32 tokens in [0, vocab) (replaces the unseeded
    ``create_dummy_data``)."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab_size, size=total_tokens, dtype=np.uint32)


def write_tokens(path: str, tokens) -> None:
    _native().write_tokens(path, np.ascontiguousarray(tokens, dtype=np.uint32))


def read_tokens(path: str) -> np.ndarray:
    return np.fromfile(path, dtype=np.uint32)


class TokenDataLoader:
    """Batches of ``(inputs, targets)`` with the upstream cursor semantics."""

    def __init__(self, source, batch_size: int, seq_len: int, device="cpu", rank: int = 0, world_size: int = 1,
                 prefetch: int = 0):
        nat = _native()
        self.batch_size, self.seq_len = int(batch_size), int(seq_len)
        self.device = torch.device(device)
        self.path = source if isinstance(source, str) else None
        if isinstance(source, str):
            self._ld = nat.TokenLoader(source, self.batch_size, self.seq_len, rank, world_size)
        else:
            self._ld = nat.TokenLoader(np.ascontiguousarray(source, dtype=np.uint32), self.batch_size,
                                       self.seq_len, rank, world_size)
        self.rank, self.world_size = rank, world_size
        self.prefetch = int(prefetch)
        pin = self.device.type == "cuda"
        nslots = max(self.prefetch, 1) + (1 if pin else 0)
        self._slots = [torch.empty(self.batch_size, self.seq_len + 1, dtype=torch.int32, pin_memory=pin)
                       for _ in range(nslots)]
        self._events = [None] * nslots
        self._held: Optional[int] = None
        self._consumed_cursor = self._ld.cursor()
        if self.prefetch > 0:
            self._ld.start_prefetch([s.data_ptr() for s in self._slots])
        self._slot_rr = 0

    # -- upstream trait surface
    def dataset_size(self) -> int:
        return int(self._ld.dataset_size())

    def shard_size(self) -> int:
        return int(self._ld.shard_end() - self._ld.shard_start())

    @property
    def cursor(self) -> int:
        """Cursor after the last batch handed out (used for resume)."""
        return int(self._consumed_cursor)

    def set_cursor(self, c: int) -> None:
        if self.prefetch > 0:
            self._ld.stop_prefetch()
            self._ld.set_cursor(int(c))
            self._ld.start_prefetch([s.data_ptr() for s in self._slots])
        else:
            self._ld.set_cursor(int(c))
        self._consumed_cursor = int(c)

    def _next_block(self) -> Tuple[torch.Tensor, int]:
        if self.prefetch > 0:
            if self._held is not None:
                ev = self._events[self._held]
                if ev is not None:
                    ev.synchronize()
                self._ld.release(self._held)
                self._held = None
            slot, off = self._ld.acquire()
            self._held = slot
        else:
            slot = self._slot_rr
            self._slot_rr = (self._slot_rr + 1) % len(self._slots)
            ev = self._events[slot]
            if ev is not None:
                ev.synchronize()
            off = self._ld.fill(self._slots[slot].data_ptr())
        self._consumed_cursor = off + self.batch_size * self.seq_len
        return self._slots[slot], slot

    def next_block(self) -> torch.Tensor:
        """The raw ``int32 [B, S+1]`` block on the loader's device."""
        host, slot = self._next_block()
        if self.device.type == "cuda":
            dev = host.to(self.device, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            self._events[slot] = ev
            return dev
        return host.clone()

    def next_batch(self) -> Tuple[torch.Tensor, torch.Tensor]:
        blk = self.next_block().long()
        return blk[:, :-1], blk[:, 1:]

    def close(self):
        if self.prefetch > 0:
            self._ld.stop_prefetch()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
