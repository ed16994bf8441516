"""Host-side stand-ins for a memory / race sanitizer.

The reference has no sanitizer or race detection at all; these checks are what this
framework runs instead of compute-sanitizer (not available on the target GPU pool):

* **Canary buffers.**  :class:`Guarded` places a tensor inside a larger allocation whose
  head and tail hold a fixed bit pattern.  :meth:`Guarded.check` reports how many guard
  elements on each side were overwritten, which catches a kernel writing past either end
  of an output it was given (``out=`` buffers, in-place ops).
* **Rerun comparison.**  :func:`rerun_check` runs the same deterministic work twice from
  the same state and reports the largest difference between the two results.  The CUDA
  reductions add f32 partials with atomics in a run-dependent order, so a few ulps of
  difference are expected on a GPU; a difference far above that (or any difference on a
  CPU) points at a race or at uninitialised memory being read.
* **Training-step rerun** (``python -m oxidizr_b200.utils.sanitize --model <m>``): builds a
  ``bench.py`` model twice from the same seed, runs the same steps on the same batch, and
  prints the largest loss and parameter differences; ``--canary`` also runs the GEMM with
  guarded output buffers over every operand layout.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from dataclasses import dataclass
from typing import Callable, Dict, Iterable, Optional, Sequence

import torch

# a bit pattern that no kernel result is likely to produce by chance: a quiet NaN payload
# for floating types (compared bitwise), 0x5A bytes for integer types
_CANARY_BITS = {2: 0x7FA5, 4: 0x7FC5A5A5, 8: 0x7FF8A5A5A5A5A5A5, 1: 0x5A}
_INT_VIEW = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}


def _as_bits(t: torch.Tensor) -> torch.Tensor:
    return t.view(_INT_VIEW[t.element_size()])


def _canary_value(esize: int) -> int:
    v = _CANARY_BITS[esize]
    bits = 8 * esize
    return v - (1 << bits) if v >= 1 << (bits - 1) else v  # as a signed integer of that width


@dataclass
class GuardReport:
    head_overwritten: int
    tail_overwritten: int

    @property
    def ok(self) -> bool:
        return self.head_overwritten == 0 and self.tail_overwritten == 0


class Guarded:
    """A contiguous tensor of ``shape`` with ``guard`` canary elements before and after it.

    ``tensor`` is the view to hand to a kernel; ``check()`` compares the guards bitwise.
    """

    def __init__(self, shape: Sequence[int], dtype: torch.dtype, device, guard: int = 4096,
                 fill: Optional[float] = None):
        n = 1
        for s in shape:
            n *= int(s)
        self.n, self.guard = n, int(guard)
        self.buf = torch.empty(n + 2 * self.guard, dtype=dtype, device=device)
        bits = _as_bits(self.buf)
        bits.fill_(_canary_value(self.buf.element_size()))
        self.tensor = self.buf[self.guard:self.guard + n].view(*shape)
        if fill is not None:
            self.tensor.fill_(fill)

    def check(self) -> GuardReport:
        bits = _as_bits(self.buf)
        c = _canary_value(self.buf.element_size())
        head = int((bits[:self.guard] != c).sum().item())
        tail = int((bits[self.guard + self.n:] != c).sum().item())
        return GuardReport(head, tail)


def max_abs_diff(a, b) -> float:
    """Largest |a - b| over (nested) tensors, f64; NaN where exactly one side is NaN."""
    if isinstance(a, torch.Tensor):
        x, y = a.detach().double().cpu(), b.detach().double().cpu()
        nan_mismatch = torch.isnan(x) ^ torch.isnan(y)
        if bool(nan_mismatch.any()):
            return float("nan")
        d = (x - y).abs()
        d = torch.where(torch.isnan(d), torch.zeros_like(d), d)  # NaN on both sides: equal
        return float(d.max().item()) if d.numel() else 0.0
    if isinstance(a, (list, tuple)):
        return max((max_abs_diff(p, q) for p, q in zip(a, b)), default=0.0)
    if isinstance(a, dict):
        return max((max_abs_diff(a[k], b[k]) for k in a), default=0.0)
    return abs(float(a) - float(b))


def rerun_check(fn: Callable[[], object], runs: int = 2) -> float:
    """Run ``fn`` (which must rebuild its own state: same seed, same inputs) ``runs`` times
    and return the largest difference of any result against the first run."""
    first = fn()
    worst = 0.0
    for _ in range(runs - 1):
        d = max_abs_diff(first, fn())
        if d != d:  # NaN
            return d
        worst = max(worst, d)
    return worst


# ------------------------------------------------------------------ training-step rerun
def bench_model_config(model_name: str, layers: Optional[int] = None):
    """``bench.py``'s config for ``model_name``, optionally cut to its first ``layers`` layers."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import bench

    cfg = bench.bench_config(model_name)
    if layers is not None:
        cfg.model.num_layers = layers
        if getattr(cfg.model, "mamba_layers", None):
            cfg.model.mamba_layers = [i for i in cfg.model.mamba_layers if i < layers]
    return cfg


def train_run(cfg, steps: int, device: torch.device) -> Dict[str, object]:
    """Build the model of ``cfg`` (seed 0) and run ``steps`` training steps on one fixed
    seeded batch; returns the per-step (loss, grad norm) and the final parameters."""
    from ..models import build_model
    from ..optim import AdamW, AdamWConfig, FlatParams
    from ..trainer import Trainer

    m, t = cfg.model, cfg.trainer
    model = build_model(m, device=device, seed=0)
    opt = AdamW(FlatParams(list(model.named_parameters()), device), AdamWConfig(lr=t.learning_rate))
    g = torch.Generator(device="cpu").manual_seed(1234)
    blk = torch.randint(0, m.vocab_size, (t.batch_size, m.max_seq_len + 1), generator=g).to(device)

    class Batches:
        batch_size, seq_len = t.batch_size, m.max_seq_len

        def dataset_size(self):
            return 10 ** 12

        def next_batch(self):
            return blk[:, :-1], blk[:, 1:]

    tr = Trainer(cfg, model, opt, Batches(), device=device, headless=True, out=lambda s: None)
    losses = []
    for _ in range(steps):
        ce, gnorm = tr.training_step()
        losses.append((float(ce), float(gnorm)))
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    params = {n: p.detach().clone() for n, p in model.named_parameters()}
    return {"losses": losses, "params": params}


def canary_gemm_sweep(device: torch.device) -> Dict[str, GuardReport]:
    """The tcgen05 GEMM into guarded outputs: every operand layout, bf16 and f32 (+= beta)
    outputs, ragged M / N / K."""
    from ..ops.gemm import mm
    out: Dict[str, GuardReport] = {}
    torch.manual_seed(0)
    for (M, N, K) in ((300, 520, 200), (1024, 768, 512), (77, 1000, 136)):
        for a_t in (False, True):
            for b_t in (False, True):
                a = torch.randn((K, M) if a_t else (M, K), device=device).bfloat16()
                b = torch.randn((K, N) if b_t else (N, K), device=device).bfloat16()
                # 16-byte aligned rows for the TMA descriptors (else mm takes its torch path)
                if a_t and M % 8:
                    a = torch.nn.functional.pad(a, (0, 8 - M % 8))[:, :M]
                if b_t and N % 8:
                    b = torch.nn.functional.pad(b, (0, 8 - N % 8))[:, :N]
                gb = Guarded((M, N), torch.bfloat16, device)
                mm(a, b, a_t=a_t, b_t=b_t, out=gb.tensor)
                gf = Guarded((M, N), torch.float32, device, fill=0.0)
                mm(a, b, a_t=a_t, b_t=b_t, out=gf.tensor, beta=1.0)
                key = f"{M}x{N}x{K} {'t' if a_t else 'n'}{'t' if b_t else 'n'}"
                out[key + " bf16"] = gb.check()
                out[key + " f32+="] = gf.check()
    return out


def main(argv: Optional[Iterable[str]] = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", default="llama")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--layers", type=int, default=2, help="layers of the bench model to build (small case)")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--canary", action="store_true", help="also run the guarded-output GEMM sweep (GPU)")
    args = ap.parse_args(list(argv) if argv is not None else None)
    dev = torch.device(args.device)
    res: Dict[str, object] = {"model": args.model, "steps": args.steps, "device": str(dev)}
    cfg = bench_model_config(args.model, args.layers)
    runs = [train_run(cfg, args.steps, dev) for _ in range(2)]
    res["max_loss_diff"] = max_abs_diff(runs[0]["losses"], runs[1]["losses"])
    res["max_param_diff"] = max_abs_diff(runs[0]["params"], runs[1]["params"])
    rc = 0
    if args.canary and dev.type == "cuda":
        rep = canary_gemm_sweep(dev)
        bad = {k: (r.head_overwritten, r.tail_overwritten) for k, r in rep.items() if not r.ok}
        res["canary_cases"] = len(rep)
        res["canary_overwritten"] = bad
        rc = 1 if bad else 0
    print(json.dumps(res))
    return rc


if __name__ == "__main__":
    raise SystemExit(main())
