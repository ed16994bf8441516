"""Training loop (trainer.rs): gradient accumulation, loss = CE + alpha * aux,
optimizer step, headless JSON / interactive logging, periodic and final
checkpoints.

Differences from upstream, by design (upstream behaviour in brackets):
* true gradient accumulation, one optimizer step per ``gradient_accumulation``
  micro-batches [upstream steps inside the accumulation loop, trainer.rs:237,245];
* true global-norm clipping at ``max_grad_norm`` (default 1.0) on the device
  [upstream pre-scales the next step's loss by the previous norm, trainer.rs:131-141];
* the MoE auxiliary loss is differentiable [detached, model.rs:589-590];
* no host synchronisation inside a step: the loss and grad norm are read only
  when a log line is printed.

Headless line (trainer.rs:336-337)::

  {"step": 1, "loss": 11.5161, "grad_norm": 0.2542, "learning_rate": 3.000000e-4, "epoch": 0.00, "it/s": 3.24, "vram": "0"}

Interactive mode appends ``{"epoch":..,"grad_norm":..,"learning_rate":..,"loss":..,"step":..}``
(alphabetical keys, serde_json's default map) to ``runs/<ts>/steps.json``.
"""
from __future__ import annotations

import math
import os
import sys
import time
from collections import deque
from typing import Callable, Optional

import torch

from .checkpoint import (AsyncCheckpointWriter, OptimizerSnapshot, host_snapshot, save_blazr_config_if_needed,
                         save_checkpoint, save_final)
from .config import LitConfig, serde_json_dumps


def rust_exp(x: float, prec: int = 6) -> str:
    """Rust ``{:.6e}``: mantissa with ``prec`` decimals, exponent without sign padding."""
    s = f"{x:.{prec}e}"
    mant, exp = s.split("e")
    return f"{mant}e{int(exp)}"


def format_duration(secs: float) -> str:
    t = int(round(secs))
    d, h, m, s = t // 86400, (t % 86400) // 3600, (t % 3600) // 60, t % 60
    if d:
        return f"{d}d{h:02d}h"
    if h:
        return f"{h}h{m:02d}m"
    if m:
        return f"{m}m{s:02d}s"
    return f"{s}s"


def vram_string(device) -> str:
    if torch.device(device).type != "cuda":
        return "0"
    try:
        return str(int(torch.cuda.memory_reserved(device) / (1024 * 1024)))
    except Exception:
        return "0"


class NonFiniteLoss(RuntimeError):
    pass


class Trainer:
    def __init__(self, cfg: LitConfig, model, optimizer, loader, *, device, headless: bool = True,
                 steps_json_path: Optional[str] = None, start_step: int = 0, data_file_path: Optional[str] = None,
                 rank: int = 0, world_size: int = 1, dataset_size: Optional[int] = None,
                 out: Callable[[str], None] = print, on_checkpoint: Optional[Callable] = None,
                 cuda_graph: bool = False):
        self.cfg = cfg
        self.tc = cfg.trainer
        self.model = model
        self.opt = optimizer
        self.loader = loader
        self.device = torch.device(device)
        self.headless = headless
        self.steps_json_path = steps_json_path
        self.global_step = start_step
        self.start_step = start_step
        self.data_file_path = data_file_path
        self.rank, self.world_size = rank, world_size
        self.out = out
        self.batch_size = loader.batch_size
        self.seq_len = loader.seq_len
        self.dataset_size = dataset_size if dataset_size is not None else loader.dataset_size()
        tps = self.batch_size * self.seq_len * self.tc.gradient_accumulation * world_size
        self.steps_per_epoch = max(1, (self.dataset_size + tps - 1) // tps)
        self.total_steps = self.steps_per_epoch * self.tc.num_epochs
        self.on_checkpoint = on_checkpoint
        self.last_loss = None
        self.last_grad_norm = None
        # whole-step CUDA graph (forward, backward, optimizer): one replay per step
        self.cuda_graph = bool(cuda_graph) and self._graph_eligible()
        self._graph = None
        self._graph_warm = 0
        self._graph_in = None
        self._graph_out = None
        self._graph_launches = 0
        # rank 0 writes periodic checkpoints on a background thread (OXI_SYNC_CHECKPOINT=1: inline)
        self._writer = None if os.environ.get("OXI_SYNC_CHECKPOINT", "0") == "1" else AsyncCheckpointWriter()

    def _graph_eligible(self) -> bool:
        """A captured step needs one process (the NVLink sync kernels take per-step
        epochs as launch arguments), a CUDA device and an optimizer whose bias
        correction lives on the device."""
        return (self.device.type == "cuda" and self.world_size == 1
                and hasattr(self.opt, "_step_state") and getattr(self.opt, "local", None) is None)

    @property
    def effective_steps(self) -> int:
        if self.tc.max_steps == 0:
            return self.total_steps
        return min(self.tc.max_steps, self.total_steps)

    # ------------------------------------------------------------ one step
    def training_step(self):
        """Returns (mean CE loss, grad norm) as device scalars."""
        from .utils.faults import fault_for, profile_window
        fault = fault_for(self.rank, self.global_step)
        profile_window(self.global_step)
        accum = self.tc.gradient_accumulation
        if self.cuda_graph:
            batches = [self.loader.next_batch() for _ in range(accum)]
            total_ce, gnorm = self._graph_step(batches)
        else:
            total_ce, gnorm = self._step_body(self.loader.next_batch for _ in range(accum))
        self.global_step += 1
        if fault == "nan":
            total_ce = total_ce * float("nan")
        return total_ce, gnorm

    def _step_body(self, batches):
        """Forward + backward over the micro-batches, then the optimizer; no host sync.
        ``batches`` yields (inputs, targets) pairs or callables returning them."""
        from .utils.faults import nvtx_range
        accum = self.tc.gradient_accumulation
        alpha = float(self.tc.load_balance_alpha)
        total_ce = torch.zeros((), dtype=torch.float32, device=self.device)
        for micro, b in enumerate(batches):
            if hasattr(self.opt, "accumulating"):
                self.opt.accumulating = micro < accum - 1
            x, y = b() if callable(b) else b
            with nvtx_range("forward"):
                ce, aux = self.model(x, y)
            loss = ce.float()
            if aux:
                loss = loss + alpha * torch.stack([a.float() for a in aux]).mean()
            with nvtx_range("backward"):
                (loss / accum).backward()
            total_ce = total_ce + ce.detach().float()
        with nvtx_range("optimizer"):
            gnorm = self.opt.step()
        return total_ce / accum, gnorm

    def _graph_step(self, batches):
        """Eager warm-up steps (kernel attributes, allocator), then capture the whole
        step into a CUDA graph over static input buffers and replay it every step."""
        from .ops._C import launch_counter
        if self._graph is None:
            self._graph_warm += 1
            if self._graph_warm <= 2:
                return self._step_body(batches)
            self._graph_in = [(x.clone(), y.clone()) for x, y in batches]
            torch.cuda.synchronize(self.device)
            torch.cuda.empty_cache()  # the graph gets its own pool; drop the eager steps' cache
            graph = torch.cuda.CUDAGraph()
            was, n0 = launch_counter.enabled, launch_counter.count
            launch_counter.enabled = True
            with torch.cuda.graph(graph):
                self._graph_out = self._step_body(self._graph_in)
            self._graph_launches = launch_counter.count - n0
            launch_counter.enabled, launch_counter.count = was, n0
            self._graph = graph
        for (xs, ys), (x, y) in zip(self._graph_in, batches):
            xs.copy_(x, non_blocking=True)
            ys.copy_(y, non_blocking=True)
        self._graph.replay()
        if launch_counter.enabled:
            launch_counter.count += self._graph_launches
        return self._graph_out

    def _check_finite(self, loss: float, grad_norm: float = 0.0):
        if not math.isfinite(loss):
            raise NonFiniteLoss("NaN loss detected")
        if not math.isfinite(grad_norm):
            # the optimizer already skipped that step on the device; stop as for a NaN loss
            raise NonFiniteLoss("non-finite gradient norm detected")

    # ------------------------------------------------------------ loops
    def fit(self):
        if self.rank == 0:
            save_blazr_config_if_needed(self.tc.checkpoint_dir, self.cfg.model)
        if self.headless:
            self._fit_headless()
        else:
            self._fit_normal()

    def _fit_headless(self):
        t0 = time.perf_counter()
        for step in range(self.start_step, self.effective_steps):
            loss_t, gn_t = self.training_step()
            if step % self.tc.log_interval == 0 or step == 0:
                loss, gn = float(loss_t), float(gn_t)
                self._check_finite(loss, gn)
                self.last_loss, self.last_grad_norm = loss, gn
                elapsed = time.perf_counter() - t0
                samples = (step + 1 - self.start_step) * self.batch_size * self.tc.gradient_accumulation
                its = samples / elapsed if elapsed > 0 else 0.0
                epoch = (step + 1) / self.steps_per_epoch
                if self.rank == 0:
                    self.out('{"step": %d, "loss": %.4f, "grad_norm": %.4f, "learning_rate": %s, "epoch": %.2f, '
                             '"it/s": %.2f, "vram": "%s"}' % (step + 1, loss, gn, rust_exp(self.tc.learning_rate),
                                                             epoch, its, vram_string(self.device)))
        self._final()

    def _fit_normal(self):
        window = deque(maxlen=5)
        t_last = time.perf_counter()
        total = self.effective_steps
        if self.start_step > 0 and self.rank == 0:
            self.out(f"Resuming from step {self.start_step}")
        for step in range(self.start_step, total):
            loss_t, gn_t = self.training_step()
            now = time.perf_counter()
            window.append(now - t_last)
            t_last = now
            avg = sum(window) / len(window)
            its = 1.0 / avg if avg > 0 else 0.0
            if step % self.tc.log_interval == 0 or step == 0:
                loss, gn = float(loss_t), float(gn_t)
                self._check_finite(loss, gn)
                self.last_loss, self.last_grad_norm = loss, gn
                epoch = (step + 1) / self.steps_per_epoch
                if self.rank == 0:
                    if self.steps_json_path:
                        line = serde_json_dumps({"epoch": epoch, "grad_norm": gn,
                                                 "learning_rate": float(self.tc.learning_rate), "loss": loss,
                                                 "step": step + 1})
                        with open(self.steps_json_path, "a") as fh:
                            fh.write(line + "\n")
                    eta = format_duration(avg * (total - step - 1))
                    self.out(f"[{step + 1:>7}/{total:<7}] {eta} loss: {loss:.4f} | grad: {gn:.4f} | {its:.2f} it/s")
            if step > 0 and step % self.tc.save_interval == 0:
                if self.rank == 0:
                    self.out(f"Checkpoint saved: step {step}")
                self.save(step)
        self._final()
        if self.rank == 0 and self.last_loss is not None:
            self.out(f"Training complete | final loss: {self.last_loss:.4f} | grad: {self.last_grad_norm:.4f}")

    # ------------------------------------------------------------ checkpoints
    def _gather_weights(self):
        """Weights in upstream names on rank 0 (collective when experts are sharded)."""
        sync = getattr(self.opt, "sync_params", None)
        if sync is not None:
            sync()  # a sharded optimizer's parameter all-gather may still be landing
        if hasattr(self.model, "export_ref_gathered"):
            return self.model.export_ref_gathered()
        return self.model.export_ref() if self.rank == 0 else None

    def save(self, step: int):
        """Every rank calls this: sharded optimizer state and expert shards are
        gathered collectively; rank 0 writes the files, each rank writes the
        state of the parameters it holds alone."""
        if self.on_checkpoint is not None:
            self.on_checkpoint(step)
            return
        sd = self._gather_weights()
        st = None
        if getattr(self.opt, "collective_state", False) or self.rank == 0:
            st = self.opt.state_tensors()
        from .checkpoint import save_local_optimizer
        prefix = self.cfg.model.checkpoint_prefix()
        path = os.path.join(self.tc.checkpoint_dir, f"{prefix}_step_{step}.safetensors")
        if self.rank == 0:
            extra = {"data_cursor": getattr(self.loader, "cursor", 0)}
            if self._writer is None:
                save_checkpoint(self.model, self.opt, step, self.cfg.model, self.tc.checkpoint_dir,
                                self.data_file_path, self.tc.max_checkpoints, extra=extra, state_dict=sd,
                                optim_state=st)
            else:
                # host copies now (training goes on updating the device tensors), files later
                sd_h, st_h = host_snapshot(sd), host_snapshot(st)
                self._writer.submit(save_checkpoint, None, OptimizerSnapshot(self.opt.step_count, st_h), step,
                                    self.cfg.model, self.tc.checkpoint_dir, self.data_file_path,
                                    self.tc.max_checkpoints, extra=extra, state_dict=sd_h, optim_state=st_h)
        local = getattr(self.opt, "local", None)
        if local is not None:
            os.makedirs(self.tc.checkpoint_dir, exist_ok=True)
            save_local_optimizer(local, path, self.rank, step)

    def flush_checkpoints(self) -> None:
        """Wait for a checkpoint write in flight (and raise its error, if it failed)."""
        if self._writer is not None:
            self._writer.wait()

    def _final(self):
        self.flush_checkpoints()
        sd = self._gather_weights()
        if self.rank == 0:
            prefix = self.cfg.model.checkpoint_prefix()
            self.out(f"Saving final checkpoint to {self.tc.checkpoint_dir}/{prefix}_final.safetensors")
            save_final(self.model, self.cfg.model, self.tc.checkpoint_dir, state_dict=sd)
