"""Trainer callbacks: checkpointing, router-load monitor, profiler, environment meter.

A callback receives ``on_train_begin(trainer)``, ``on_step_end(trainer,
step, loss)`` and ``on_train_end(trainer)``.  ``CallbackList`` dispatches
to several.  Metrics are printed by rank 0 as one JSON line per log step
(``metrics_path`` also appends them to a file).

Reference parity: veomni/trainer/callbacks/checkpoint_callback.py:97-327
(checkpoint), trace_callback.py:49-326 (MoE router monitor), :353-377
(torch profiler), :379-486 (environment meter, hiermoe metrics flush).
"""

from __future__ import annotations

import json
import os
import time

import torch
import torch.distributed as dist

from ..utils.metrics import RouterLoadMonitor, environment_meter, placemoe_metrics


def _rank0() -> bool:
    return not dist.is_initialized() or dist.get_rank() == 0


class Callback:
    def on_train_begin(self, trainer) -> None:
        pass

    def on_step_end(self, trainer, step: int, loss: float) -> None:
        pass

    def on_train_end(self, trainer) -> None:
        pass


class CallbackList(Callback):
    def __init__(self, callbacks):
        self.callbacks = list(callbacks)

    def on_train_begin(self, trainer):
        for c in self.callbacks:
            c.on_train_begin(trainer)

    def on_step_end(self, trainer, step, loss):
        for c in self.callbacks:
            c.on_step_end(trainer, step, loss)

    def on_train_end(self, trainer):
        for c in self.callbacks:
            c.on_train_end(trainer)


class CheckpointCallback(Callback):
    """DCP checkpoint every ``save_steps`` steps under ``root/global_step_N`` (and at the end)."""

    def __init__(self, root: str, save_steps: int, save_at_end: bool = False):
        self.root, self.save_steps, self.save_at_end = root, save_steps, save_at_end

    def on_step_end(self, trainer, step, loss):
        if self.save_steps and (step + 1) % self.save_steps == 0:
            from ..checkpoint import save_checkpoint

            save_checkpoint(trainer, self.root)

    def on_train_end(self, trainer):
        if self.save_at_end:
            from ..checkpoint import save_checkpoint

            save_checkpoint(trainer, self.root)


class RouterMonitorCallback(Callback):
    """Expert-load statistics (logical and physical) from each step's routes."""

    def __init__(self, log_interval: int = 10):
        self.log_interval = max(1, log_interval)
        self.monitor = None
        self.last: dict = {}

    def on_train_begin(self, trainer):
        self.monitor = RouterLoadMonitor(trainer.model)

    def on_step_end(self, trainer, step, loss):
        self.monitor.observe()
        if (step + 1) % self.log_interval == 0:
            self.last = self.monitor.summary()
            trainer.metrics.update(self.last)
            self.monitor.reset()


class ProfilerCallback(Callback):
    """torch.profiler trace of steps [start, start + steps) written to ``out_dir`` (chrome trace)."""

    def __init__(self, out_dir: str, start: int = 2, steps: int = 2):
        self.out_dir, self.start, self.steps = out_dir, start, steps
        self.prof = None

    def on_step_end(self, trainer, step, loss):
        if step + 1 == self.start and self.prof is None:
            acts = [torch.profiler.ProfilerActivity.CPU]
            if torch.cuda.is_available():
                acts.append(torch.profiler.ProfilerActivity.CUDA)
            self.prof = torch.profiler.profile(activities=acts, record_shapes=False)
            self.prof.__enter__()
        elif self.prof is not None and step + 1 == self.start + self.steps:
            self.prof.__exit__(None, None, None)
            os.makedirs(self.out_dir, exist_ok=True)
            rank = dist.get_rank() if dist.is_initialized() else 0
            self.prof.export_chrome_trace(os.path.join(self.out_dir, f"trace_rank{rank}.json"))
            self.prof = None

    def on_train_end(self, trainer):
        if self.prof is not None:
            self.prof.__exit__(None, None, None)
            self.prof = None


class EnvironmentMeterCallback(Callback):
    """Tokens/s, TFLOP/s per GPU, MFU, memory and placement metrics every ``log_interval`` steps."""

    def __init__(self, tokens_per_step: int, flops_per_token: float, log_interval: int = 10,
                 metrics_path: str = ""):
        self.tokens_per_step, self.flops_per_token = tokens_per_step, flops_per_token
        self.log_interval = max(1, log_interval)
        self.metrics_path = metrics_path
        self._t = None
        self._steps = 0

    def on_train_begin(self, trainer):
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        self._t = time.perf_counter()

    def on_step_end(self, trainer, step, loss):
        self._steps += 1
        if (step + 1) % self.log_interval:
            return
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        now = time.perf_counter()
        step_ms = (now - self._t) * 1e3 / max(self._steps, 1)
        self._t, self._steps = now, 0
        m = environment_meter(self.tokens_per_step, step_ms, self.flops_per_token, trainer.world)
        m.update(placemoe_metrics(trainer.model))
        m.update({k: (float(v) if not isinstance(v, (int, float)) else v) for k, v in trainer.metrics.items()
                  if not hasattr(v, "shape") or getattr(v, "numel", lambda: 0)() == 1})
        m["step"], m["loss"] = step + 1, float(loss)
        if _rank0():
            line = json.dumps(m)
            print(line, flush=True)
            if self.metrics_path:
                os.makedirs(os.path.dirname(os.path.abspath(self.metrics_path)), exist_ok=True)
                with open(self.metrics_path, "a") as f:
                    f.write(line + "\n")
