"""Observability: MoE timing spans, step-phase timing, placement metrics, router load, MFU.

* ``TimingSpans`` records CUDA-event spans per (direction, component, section)
  and flushes them as per-step milliseconds; multi-GPU values are reduced as
  the max over ranks.  Enabled by ``PM_MOE_TIMING_DIR`` (JSON lines written
  there) or programmatically.
* ``StepPhases`` times named step phases (forward_backward, replica_sync,
  grad_clip, optimizer_step, hot_update, ...) with CUDA events and matching
  NVTX ranges for profilers.
* ``placemoe_metrics`` aggregates per-layer dispatch statistics (rows sent,
  dedup ratio, received assignments, capacity) under ``placemoe/`` names.
* ``RouterLoadMonitor`` accumulates per-layer expert load (logical) and
  physical slot load from the captured routes and the placement mapping.
* ``environment_meter`` gives tokens/s, model TFLOP/s, MFU against the
  measured peak and memory.

Reference parity: veomni/distributed/moe/timing.py:108-314 (MoE timing
spans, profile ranges), veomni/utils/full_timing_profiler.py:141-617 (step
phases), hiermoe/metrics.py:22-85, utils/moe_monitor.py:222-514 (router
load), utils/physical_moe_load.py:19-130, trainer/callbacks/trace_callback.py:379-486
(environment meter).
"""

from __future__ import annotations

import contextlib
import json
import os
import time
from collections import defaultdict

import torch
import torch.distributed as dist

TIMING_ENV = "PM_MOE_TIMING_DIR"


def _max_over_ranks(values: list[float]) -> list[float]:
    if not (dist.is_initialized() and dist.get_world_size() > 1) or not values:
        return values
    dev = torch.device("cuda") if torch.cuda.is_available() and dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


class TimingSpans:
    """CUDA-event spans keyed by (direction, component, section)."""

    def __init__(self, enabled: bool | None = None, out_dir: str | None = None):
        self.out_dir = out_dir if out_dir is not None else os.environ.get(TIMING_ENV, "")
        self.enabled = bool(self.out_dir) if enabled is None else enabled
        self._open: list[tuple[tuple[str, str, str], object, object]] = []

    @contextlib.contextmanager
    def span(self, direction: str, component: str, section: str = ""):
        if not self.enabled:
            yield
            return
        cuda = torch.cuda.is_available()
        key = (direction, component, section)
        if cuda:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push(f"{direction}/{component}/{section}")
            s.record()
        else:
            s = time.perf_counter()
        try:
            yield
        finally:
            if cuda:
                e.record()
                torch.cuda.nvtx.range_pop()
                self._open.append((key, s, e))
            else:
                self._open.append((key, s, time.perf_counter()))

    def flush(self, step: int) -> dict[str, float]:
        """Per-key total ms for the spans recorded since the last flush (max over ranks)."""
        if not self._open:
            return {}
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        acc: dict[str, float] = defaultdict(float)
        for key, s, e in self._open:
            ms = s.elapsed_time(e) if hasattr(s, "elapsed_time") else (e - s) * 1e3
            acc["/".join(k for k in key if k)] += ms
        self._open.clear()
        keys = sorted(acc)
        vals = _max_over_ranks([acc[k] for k in keys])
        out = dict(zip(keys, vals))
        rank0 = not dist.is_initialized() or dist.get_rank() == 0
        if self.out_dir and rank0:
            os.makedirs(self.out_dir, exist_ok=True)
            with open(os.path.join(self.out_dir, "moe_timing.jsonl"), "a") as f:
                f.write(json.dumps({"step": step, "ms": out}) + "\n")
        return out


class StepPhases:
    """Named step phases timed with CUDA events (plus NVTX ranges)."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self._events: list[tuple[str, object, object]] = []

    @contextlib.contextmanager
    def phase(self, name: str):
        if not self.enabled or not torch.cuda.is_available():
            t0 = time.perf_counter()
            yield
            if self.enabled:
                self._events.append((name, t0, time.perf_counter()))
            return
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(name)
        s.record()
        try:
            yield
        finally:
            e.record()
            torch.cuda.nvtx.range_pop()
            self._events.append((name, s, e))

    def collect(self) -> dict[str, float]:
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        out: dict[str, float] = defaultdict(float)
        for name, s, e in self._events:
            out[name] += s.elapsed_time(e) if hasattr(s, "elapsed_time") else (e - s) * 1e3
        self._events.clear()
        return dict(out)


def placemoe_metrics(model) -> dict[str, float]:
    """Aggregated dispatch statistics of the last step under placemoe/ names."""
    out: dict[str, float] = {}
    blocks = list(model.moe_blocks())
    ratios, sent, asg = [], 0.0, 0.0
    for blk in blocks:
        st = getattr(blk.ep, "stats", None) if blk.ep is not None else None
        if st:
            ratios.append(float(st.get("dedup_ratio", 1.0)))
            sent += float(st.get("sent_rows", 0))
            asg += float(st.get("sent_assignments", 0))
        pl = blk.placement
        if pl is not None:
            out[f"placemoe/placement_version/{blk.layer_idx}"] = float(pl.version)
    if ratios:
        out["placemoe/dedup_ratio"] = sum(ratios) / len(ratios)
        out["placemoe/sent_rows"] = sent
        out["placemoe/sent_assignments"] = asg
    ep = blocks[0].ep if blocks else None
    if ep is not None and hasattr(ep, "capacity_factor"):
        out["placemoe/ep_capacity_factor"] = float(ep.capacity_factor)
    return out


class RouterLoadMonitor:
    """Per-layer logical expert load and physical slot load, accumulated over steps."""

    def __init__(self, model):
        self.model = model
        self.logical: dict[int, torch.Tensor] = {}
        self.physical: dict[int, torch.Tensor] = {}
        self.steps = 0

    def observe(self) -> None:
        for blk in self.model.moe_blocks():
            route = blk.last_route
            if route is None:
                continue
            e = blk.cfg.num_experts
            cnt = torch.bincount(route.reshape(-1).long().cpu(), minlength=e).double()
            self.logical[blk.layer_idx] = self.logical.get(blk.layer_idx, torch.zeros(e, dtype=torch.float64)) + cnt
            pl = blk.placement
            if pl is not None and hasattr(pl, "lut_global"):
                lut = torch.as_tensor(pl.lut_global(), dtype=torch.long)  # logical -> physical slot (this rank's M)
                slots = lut[route.reshape(-1).long().cpu()]
                n = int(lut.max()) + 1 if lut.numel() else 0
                ph = torch.bincount(slots, minlength=max(n, 1)).double()
                prev = self.physical.get(blk.layer_idx)
                if prev is not None and prev.numel() < ph.numel():
                    prev = torch.nn.functional.pad(prev, (0, ph.numel() - prev.numel()))
                self.physical[blk.layer_idx] = ph if prev is None else prev[: ph.numel()] + ph
        self.steps += 1

    def summary(self) -> dict[str, float]:
        out = {}
        for layer, cnt in self.logical.items():
            mean = float(cnt.mean()) or 1.0
            out[f"router/max_over_mean/{layer}"] = float(cnt.max()) / mean
            out[f"router/cv/{layer}"] = float(cnt.std()) / mean
        for layer, cnt in self.physical.items():
            nz = cnt[cnt > 0]
            if nz.numel():
                out[f"router/physical_max_over_mean/{layer}"] = float(nz.max()) / float(nz.mean())
        return out

    def reset(self) -> None:
        self.logical.clear()
        self.physical.clear()
        self.steps = 0


def environment_meter(tokens: int, step_ms: float, flops_per_token: float, world: int,
                      peak_tflops: float | None = None) -> dict[str, float]:
    """Throughput, model TFLOP/s per GPU, MFU against the measured bf16 peak, memory."""
    if peak_tflops is None:
        peak_tflops = measured_bf16_tflops()
    tps = tokens / (step_ms / 1e3) if step_ms > 0 else 0.0
    tflops = flops_per_token * tps / max(world, 1) / 1e12
    out = {"env/tokens_per_s": tps, "env/model_tflops_per_gpu": tflops,
           "env/mfu": tflops / peak_tflops if peak_tflops else 0.0}
    if torch.cuda.is_available():
        out["env/max_mem_gb"] = torch.cuda.max_memory_allocated() / 2**30
    return out


def measured_bf16_tflops() -> float:
    """The measured bf16 GEMM peak of the machine (MEASURED_PEAKS.json at the repository root), else 1590."""
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    path = os.path.join(root, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0
