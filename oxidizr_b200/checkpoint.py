"""Checkpoint files in the upstream layout, plus an optimizer sidecar.

Files in ``checkpoint_dir`` (trainer.rs:465-551, config.rs:390-470, 646-686):

* ``{prefix}_step_{N}.safetensors``  weights, upstream tensor names, model dtype
* ``checkpoint_step_{N}.meta.json``   step/timestamp/config hash/data hash/file/dtype
* ``{prefix}_final.safetensors``     final weights, no meta
* ``config.json``                    inference config, written once
* ``{prefix}_step_{N}.optim.safetensors``  (new) f32 master weights, AdamW
  moments, step, data cursor; upstream ignores it, and a checkpoint without it
  resumes like upstream (fresh moments)

``prefix = {name}_{max_seq_len}_{params}_{dtype}`` (config.rs:126-134).
"""
from __future__ import annotations

import datetime
import json
import os
import threading
import re
from typing import Dict, Optional, Tuple

import torch
from safetensors.torch import load_file, save_file

from .config import ModelConfig, blazr_config_json, serde_json_dumps
from .utils.hashing import compute_file_hash, compute_model_config_hash

_STEP_RE = re.compile(r"_step_(\d+)\.safetensors$")


def _owns_storage(t: torch.Tensor) -> bool:
    """A contiguous host tensor that is the whole of its storage (shares memory with nothing)."""
    return (t.device.type == "cpu" and t.is_contiguous() and t.storage_offset() == 0
            and t.untyped_storage().nbytes() == t.numel() * t.element_size())


def _cpu_contig(sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Host tensors that safetensors accepts: views of a shared buffer (flat parameters) are
    copied out; tensors that already own their storage are passed through once (a second
    name for the same storage gets a copy)."""
    out, seen = {}, set()
    for k, v in sd.items():
        v = v.detach()
        if _owns_storage(v) and v.data_ptr() not in seen:
            seen.add(v.data_ptr())
            out[k] = v
        else:
            out[k] = v.to("cpu").contiguous().clone()
    return out


def host_snapshot(sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Host copies, each owning its storage, taken now (the originals keep changing)."""
    return {k: v.detach().to("cpu", copy=True).contiguous() for k, v in sd.items()}


class CheckpointMeta:
    FIELDS = ("step", "timestamp", "model_config_hash", "data_file_path", "data_file_hash", "checkpoint_file",
              "dtype")

    def __init__(self, step, timestamp, model_config_hash, data_file_path, data_file_hash, checkpoint_file,
                 dtype="f32"):
        self.step = int(step)
        self.timestamp = timestamp
        self.model_config_hash = model_config_hash
        self.data_file_path = data_file_path
        self.data_file_hash = data_file_hash
        self.checkpoint_file = checkpoint_file
        self.dtype = dtype

    @staticmethod
    def new(step: int, model_cfg: ModelConfig, data_file_path: str, checkpoint_file: str) -> "CheckpointMeta":
        ts = datetime.datetime.now().strftime("%Y-%m-%d %H:%M:%S")
        return CheckpointMeta(step, ts, compute_model_config_hash(model_cfg), data_file_path,
                              compute_file_hash(data_file_path), checkpoint_file, model_cfg.dtype)

    def to_json(self) -> str:
        return serde_json_dumps({k: getattr(self, k) for k in self.FIELDS}, pretty=True)

    def save(self, checkpoint_dir: str) -> str:
        path = os.path.join(checkpoint_dir, f"checkpoint_step_{self.step}.meta.json")
        with open(path, "w") as fh:
            fh.write(self.to_json())
        return path

    @staticmethod
    def load(path: str) -> "CheckpointMeta":
        with open(path) as fh:
            d = json.load(fh)
        missing = [k for k in CheckpointMeta.FIELDS[:-1] if k not in d]
        if missing:
            raise ValueError(f"meta file {path} missing fields {missing}")
        return CheckpointMeta(**{k: d.get(k, "f32") for k in CheckpointMeta.FIELDS})

    def validate(self, model_cfg: ModelConfig, data_file_path: str) -> dict:
        cur_m = compute_model_config_hash(model_cfg)
        cur_d = compute_file_hash(data_file_path)
        v = {
            "model_matches": self.model_config_hash == cur_m,
            "data_matches": self.data_file_hash == cur_d,
            "dtype_matches": self.dtype == model_cfg.dtype,
            "checkpoint_model_hash": self.model_config_hash, "current_model_hash": cur_m,
            "checkpoint_data_hash": self.data_file_hash, "current_data_hash": cur_d,
            "checkpoint_dtype": self.dtype, "current_dtype": model_cfg.dtype,
        }
        v["is_valid"] = v["model_matches"] and v["data_matches"]  # dtype may differ
        return v


def find_latest_checkpoint(checkpoint_dir: str) -> Optional[Tuple[str, str, int]]:
    """Highest ``*_step_N.safetensors`` that has a ``checkpoint_step_N.meta.json``."""
    if not os.path.isdir(checkpoint_dir):
        return None
    best = None
    for fn in os.listdir(checkpoint_dir):
        if "_step_" not in fn or not fn.endswith(".safetensors") or fn.endswith(".optim.safetensors"):
            continue
        m = _STEP_RE.search(fn)
        if not m:
            continue
        step = int(m.group(1))
        meta = os.path.join(checkpoint_dir, f"checkpoint_step_{step}.meta.json")
        if os.path.exists(meta) and (best is None or step > best[2]):
            best = (os.path.join(checkpoint_dir, fn), meta, step)
    return best


def step_from_filename(path: str) -> int:
    stem = os.path.basename(path)
    if stem.endswith(".safetensors"):
        stem = stem[: -len(".safetensors")]
    if "_step_" in stem:
        try:
            return int(stem.split("_step_")[-1])
        except ValueError:
            return 0
    return 0


def save_blazr_config_if_needed(checkpoint_dir: str, model_cfg: ModelConfig) -> bool:
    os.makedirs(checkpoint_dir, exist_ok=True)
    path = os.path.join(checkpoint_dir, "config.json")
    if os.path.exists(path):
        return False
    with open(path, "w") as fh:
        fh.write(blazr_config_json(model_cfg))
    return True


def _save_atomic(tensors: Dict[str, torch.Tensor], path: str, metadata: Optional[Dict[str, str]] = None) -> None:
    """safetensors file written under a temporary name and renamed into place: a crash mid-write
    (or a background write cut short) never leaves a truncated file under the real name."""
    tmp = f"{path}.tmp{os.getpid()}"
    try:
        save_file(tensors, tmp, metadata=metadata)
        os.replace(tmp, path)
    finally:
        if os.path.exists(tmp):
            os.remove(tmp)


def save_weights(model, path: str, state_dict: Optional[Dict[str, torch.Tensor]] = None) -> None:
    _save_atomic(_cpu_contig(state_dict if state_dict is not None else model.export_ref()), path)


def load_weights(model, path: str) -> None:
    sd = load_file(path)
    model.import_ref(sd)


def optim_sidecar_path(weights_path: str) -> str:
    assert weights_path.endswith(".safetensors")
    return weights_path[: -len(".safetensors")] + ".optim.safetensors"


def save_checkpoint(model, optimizer, step: int, model_cfg: ModelConfig, checkpoint_dir: str,
                    data_file_path: Optional[str], max_checkpoints: int, extra: Optional[dict] = None,
                    state_dict: Optional[Dict[str, torch.Tensor]] = None,
                    optim_state: Optional[Dict[str, torch.Tensor]] = None) -> str:
    """trainer.rs:465-493 (+ sidecar).  Returns the weights path.

    ``state_dict`` / ``optim_state``: already gathered tensors (data-parallel
    runs gather them collectively on every rank, then rank 0 writes)."""
    os.makedirs(checkpoint_dir, exist_ok=True)
    prefix = model_cfg.checkpoint_prefix()
    path = os.path.join(checkpoint_dir, f"{prefix}_step_{step}.safetensors")
    save_weights(model, path, state_dict)
    if optimizer is not None:
        st = dict(optim_state if optim_state is not None else optimizer.state_tensors())
        meta = {"step": str(optimizer.step_count), "format": "oxidizr_b200.flat_adamw.v1"}
        if extra:
            meta.update({k: str(v) for k, v in extra.items()})
        _save_atomic(_cpu_contig(st), optim_sidecar_path(path), metadata=meta)
    if data_file_path:
        try:
            CheckpointMeta.new(step, model_cfg, data_file_path, path).save(checkpoint_dir)
        except OSError as e:
            print(f"Warning: Failed to save checkpoint metadata: {e}")
    if max_checkpoints > 0:
        cleanup_old_checkpoints(checkpoint_dir, max_checkpoints)
    return path


class OptimizerSnapshot:
    """The parts of an optimizer that ``save_checkpoint`` reads, frozen at one step (host copies)."""

    def __init__(self, step_count: int, state: Dict[str, torch.Tensor]):
        self.step_count = step_count
        self._state = state

    def state_tensors(self) -> Dict[str, torch.Tensor]:
        return self._state


class AsyncCheckpointWriter:
    """Writes checkpoint files on a background thread, so a training step only waits for the
    device-to-host snapshot, not for serialisation and disk.  At most one write is in flight:
    ``submit`` first waits for the previous one.  The thread is not a daemon, so the process
    finishes a pending write before it exits; an error in a write is raised by the next
    ``submit`` or ``wait``."""

    def __init__(self):
        self._thread: Optional[threading.Thread] = None
        self._error: Optional[BaseException] = None

    def submit(self, fn, *args, **kwargs) -> None:
        self.wait()

        def run():
            try:
                fn(*args, **kwargs)
            except BaseException as e:  # noqa: BLE001 - handed to the training thread
                self._error = e

        self._thread = threading.Thread(target=run, name="oxidizr-checkpoint-writer", daemon=False)
        self._thread.start()

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if self._error is not None:
            err, self._error = self._error, None
            raise err

    @property
    def busy(self) -> bool:
        return self._thread is not None and self._thread.is_alive()


def cleanup_old_checkpoints(checkpoint_dir: str, max_checkpoints: int) -> None:
    """Keep the newest ``max_checkpoints`` step files (trainer.rs:496-541)."""
    found = []
    for fn in os.listdir(checkpoint_dir):
        if "_step_" in fn and fn.endswith(".safetensors") and not fn.endswith(".optim.safetensors"):
            m = _STEP_RE.search(fn)
            if m:
                found.append((int(m.group(1)), os.path.join(checkpoint_dir, fn)))
    found.sort()
    for step, path in found[: max(0, len(found) - max_checkpoints)]:
        stem = path[: -len(".safetensors")]
        locals_ = [os.path.join(checkpoint_dir, f) for f in os.listdir(checkpoint_dir)
                   if f.startswith(os.path.basename(stem) + ".optim.local")]
        for p in [path, optim_sidecar_path(path), os.path.join(checkpoint_dir, f"checkpoint_step_{step}.meta.json")] + \
                locals_:
            try:
                os.remove(p)
            except FileNotFoundError:
                pass


def save_final(model, model_cfg: ModelConfig, checkpoint_dir: str, name: str = "final",
               state_dict: Optional[Dict[str, torch.Tensor]] = None) -> str:
    os.makedirs(checkpoint_dir, exist_ok=True)
    path = os.path.join(checkpoint_dir, f"{model_cfg.checkpoint_prefix()}_{name}.safetensors")
    save_weights(model, path, state_dict)
    return path


def local_sidecar_path(weights_path: str, rank: int) -> str:
    """Per-rank optimizer state of parameters that rank holds alone (expert shards)."""
    assert weights_path.endswith(".safetensors")
    return weights_path[: -len(".safetensors")] + f".optim.local{rank}.safetensors"


def save_local_optimizer(local_opt, weights_path: str, rank: int, step: int) -> None:
    _save_atomic(_cpu_contig(local_opt.state_tensors()), local_sidecar_path(weights_path, rank),
                 metadata={"step": str(step), "format": "oxidizr_b200.flat_adamw.v1"})


def load_local_optimizer(local_opt, weights_path: str, rank: int) -> bool:
    sp = local_sidecar_path(weights_path, rank)
    if local_opt is None or not os.path.exists(sp):
        return False
    tens = load_file(sp)
    with torch.no_grad():
        local_opt.flat.master.copy_(tens["master"].to(local_opt.flat.master.device))
        if local_opt.flat.flat is not local_opt.flat.master:
            local_opt.flat.flat.copy_(local_opt.flat.master)
        local_opt.m.copy_(tens["exp_avg"].to(local_opt.m.device))
        local_opt.v.copy_(tens["exp_avg_sq"].to(local_opt.v.device))
    return True


def load_optimizer_sidecar(optimizer, weights_path: str) -> Optional[dict]:
    sp = optim_sidecar_path(weights_path)
    if optimizer is None or not os.path.exists(sp):
        return None
    from safetensors import safe_open
    with safe_open(sp, framework="pt") as fh:
        meta = dict(fh.metadata() or {})
        tens = {k: fh.get_tensor(k) for k in fh.keys()}
    optimizer.load_state_tensors(tens, int(meta.get("step", "0")))
    return meta


def clear_checkpoint_directory(checkpoint_dir: str) -> int:
    """commands/train.rs:90-136 (without the prompt)."""
    n = 0
    if not os.path.isdir(checkpoint_dir):
        return 0
    for fn in os.listdir(checkpoint_dir):
        if fn.endswith(".safetensors") or fn.endswith(".meta.json") or fn == "config.json":
            try:
                os.remove(os.path.join(checkpoint_dir, fn))
                n += 1
            except OSError as e:
                print(f"Warning: Failed to remove {fn}: {e}")
    return n
