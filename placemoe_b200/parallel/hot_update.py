"""Asynchronous PlaceMoE hot updates at step boundaries.

Per training step (``on_step_end``):

1. the controller observes the step; if a planner job is running, rank 0
   polls it and broadcasts its status (running / done / failed);
2. a finished job's artifact is read on rank 0, broadcast, validated, checked
   for staleness (the placement versions it was planned from must still be
   current) and installed on every rank:
   * mapping-only: layout and owners must be unchanged; only M is swapped;
   * full: expert parameters AND AdamW moments of every changed slot are
     migrated (source copy chosen same-rank first, then the owner, then any
     copy), staged into fresh tensors and published only after every transfer
     of every rank succeeded; emptied slots are zeroed;
3. when an update is due and no job runs: routes of the last steps are
   captured into a bundle directory, the current layout is written (mapping
   mode) and rank 0 launches the planner subprocess (``taskset`` onto the
   planner CPUs when configured).

A failed planner keeps the current placement (``failure_policy: continue``)
or raises (``raise``).  Metrics of every event are kept in ``events``.

Reference parity: ExpertSwapManager hot-update orchestration
(veomni/distributed/moe/hiermoe/expert_swap.py:10568-11181), atomic migration
(:1358-1542), mapping-only install (:10920-10973).
"""

from __future__ import annotations

import json
import os
import subprocess
import time

import numpy as np
import torch
import torch.distributed as dist

from ..placemoe.artifacts import build_placemoe_artifact, validate_placemoe_artifact, write_artifact
from ..placemoe.runtime.config import PlaceMoERuntimeConfig
from ..placemoe.runtime.planner_process import (HotUpdateJob, PlannerCommandSpec, build_planner_command,
                                                default_planner_path, planner_environment, python_executable)
from ..placemoe.runtime.scheduler import HotUpdateController, UpdateKind
from ..placemoe.types import EMPTY_EXPERT, LayerPlan
from .migration import migrate_layer
from .route_capture import RouteRecorder

STATUS_IDLE, STATUS_RUNNING, STATUS_DONE, STATUS_FAILED = 0, 1, 2, 3


class HotUpdateManager:
    def __init__(self, trainer, config: PlaceMoERuntimeConfig, capture_steps: int = 2, group=None):
        self.trainer = trainer
        self.cfg = config
        self.group = group
        hu = config.hot_update
        self.controller = HotUpdateController(
            layout_interval_steps=hu.layout_interval_steps or 0,
            mapping_interval_steps=hu.mapping_interval_steps,
            last_update_step=hu.last_update_step,
            failure_policy=hu.failure_policy,
        )
        self.work_root = hu.work_root
        self.planner_path = hu.planner_path or default_planner_path()
        self.capture_steps = capture_steps
        self.recorder = RouteRecorder(trainer.model, os.path.join(self.work_root, "routes_live"), group)
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.events: list[dict] = []
        self._capture_left = 0
        self._pending_kind: UpdateKind | None = None
        self._job_seq = 0

    # --------------------------------------------------------------- helpers
    def _bcast_int(self, v: int) -> int:
        if self.world == 1:
            return v
        t = torch.tensor([v], dtype=torch.int64)
        if dist.get_backend(self.group) == "nccl":
            t = t.cuda()
        dist.broadcast(t, 0, group=self.group)
        return int(t.item())

    def _bcast_obj(self, obj):
        if self.world == 1:
            return obj
        box = [obj]
        dist.broadcast_object_list(box, 0, group=self.group)
        return box[0]

    def _versions(self) -> tuple[int, ...]:
        return tuple(blk.placement.version for blk in self.trainer.model.moe_blocks())

    def current_artifact(self) -> dict:
        plans = {blk.layer_key: blk.placement.plan for blk in self.trainer.model.moe_blocks()}
        return build_placemoe_artifact(plans, self.trainer.topology, source={"planner": "runtime-snapshot"})

    # ------------------------------------------------------------- step hook
    def on_step_end(self, trainer) -> None:
        step = trainer.global_step
        self.controller.observe_step(step)
        # 1) route capture for a pending launch
        if self._capture_left > 0:
            self.recorder.record_step(self.capture_steps - self._capture_left)
            self._capture_left -= 1
            if self._capture_left == 0:
                self._launch(self._pending_kind, step)
            else:
                self.recorder.enabled = True
            return
        # 2) active job
        if self.controller.active_job is not None:
            self._poll(step)
            return
        # 3) new update due
        kind = self.controller.next_update()
        if kind is not None:
            self._pending_kind = kind
            self._capture_left = self.capture_steps
            self.recorder.enabled = True
            self._job_seq += 1

    def _launch(self, kind: UpdateKind, step: int) -> None:
        self.recorder.enabled = False
        t0 = time.perf_counter()
        job_dir = os.path.join(self.work_root, f"job{self._job_seq:04d}_step{step:06d}")
        layout_path = os.path.join(job_dir, "layout.json")
        report_path = os.path.join(job_dir, "report.json")
        log_path = os.path.join(job_dir, "planner.log")
        proc = None
        if self.rank == 0:
            os.makedirs(job_dir, exist_ok=True)
            route_root = os.path.join(job_dir, "routes")
            if os.path.isdir(self.recorder.root):
                os.replace(self.recorder.root, route_root)
            input_layout = ""
            if kind is UpdateKind.MAPPING_ONLY:
                input_layout = os.path.join(job_dir, "current_layout.json")
                write_artifact(self.current_artifact(), input_layout)
            t = self.trainer.topology
            cfg = self.trainer.model_cfg
            spec = PlannerCommandSpec(
                python=python_executable(), planner_path=self.planner_path, route_root=route_root, kind=kind,
                layer_keys=[blk.layer_key for blk in self.trainer.model.moe_blocks()], ep_size=t.ep_size,
                ranks_per_node=t.ranks_per_node, num_experts=t.num_experts, slots_per_rank=t.slots_per_rank,
                primary_slots_per_rank=-(-t.num_experts // t.ep_size),
                redundant_slots_per_rank=t.slots_per_rank - (-(-t.num_experts // t.ep_size)),
                hidden_size=cfg.hidden_size, bytes_per_element=2, output_layout=layout_path,
                output_report=report_path, input_layout=input_layout)
            cmd = build_planner_command(spec, self.cfg.calibration, self.cfg.resources)
            cmd[cmd.index("--optimize-steps") + 1] = ",".join(str(i) for i in range(self.capture_steps))
            log = open(log_path, "w")
            proc = subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT,
                                    env=planner_environment(self.cfg.resources))
        job = HotUpdateJob(kind=kind, source_step=step, placement_versions=self._versions(),
                           submitted_at=time.time(), snapshot_ms=(time.perf_counter() - t0) * 1e3, job_dir=job_dir,
                           layout_path=layout_path, report_path=report_path, planner_log_path=log_path,
                           process=proc)
        self.controller.start(job)
        self.events.append({"event": "submitted", "kind": kind.value, "step": step,
                            "snapshot_ms": job.snapshot_ms})

    def _poll(self, step: int) -> None:
        job = self.controller.active_job
        status = STATUS_RUNNING
        if self.rank == 0:
            rc = job.process.poll() if job.process is not None else 1
            if rc is None:
                status = STATUS_RUNNING
            elif rc == 0 and os.path.exists(job.layout_path):
                status = STATUS_DONE
            else:
                status = STATUS_FAILED
        status = self._bcast_int(status)
        if status == STATUS_RUNNING:
            return
        self.controller.finish()
        planner_ms = (time.time() - job.submitted_at) * 1e3
        if status == STATUS_FAILED:
            self.events.append({"event": "failed", "kind": job.kind.value, "step": step, "planner_ms": planner_ms})
            if self.controller.failure_policy == "raise":
                raise RuntimeError(f"PlaceMoE planner failed; see {job.planner_log_path}")
            return
        payload = None
        if self.rank == 0:
            with open(job.layout_path) as f:
                payload = json.load(f)
        payload = self._bcast_obj(payload)
        self.apply_artifact(payload, job, step, planner_ms)

    # -------------------------------------------------------------- install
    def apply_artifact(self, payload: dict, job: HotUpdateJob | None, step: int, planner_ms: float = 0.0) -> bool:
        try:
            plans = validate_placemoe_artifact(payload)
        except ValueError as e:
            self.events.append({"event": "failed", "step": step, "reason": f"invalid artifact: {e}"})
            if self.controller.failure_policy == "raise":
                raise
            return False
        if job is not None and tuple(job.placement_versions) != self._versions():
            self.events.append({"event": "rejected_stale", "step": step})
            return False
        kind = job.kind if job is not None else UpdateKind.FULL
        t0 = time.perf_counter()
        moved = 0
        blocks = self.trainer.model.moe_blocks()
        if kind is UpdateKind.MAPPING_ONLY:
            for blk in blocks:
                if blk.layer_key in plans:
                    blk.placement.install_mapping(plans[blk.layer_key])
        else:
            for blk in blocks:
                plan = plans.get(blk.layer_key)
                if plan is None:
                    continue
                moved += migrate_layer(self.trainer, blk, plan, group=self.group)
            self.trainer._norm_table = None
        self.trainer.optimizer.reset_tables()
        if dist.is_initialized():
            dist.barrier(group=self.group)
        self.events.append({"event": "applied", "kind": kind.value, "step": step, "planner_ms": planner_ms,
                            "migration_ms": (time.perf_counter() - t0) * 1e3, "moved_slots": moved,
                            "staleness_steps": step - (job.source_step if job else step)})
        return True


def changed_slots(old: np.ndarray, new: np.ndarray) -> np.ndarray:
    return np.flatnonzero(old != new)


__all__ = ["HotUpdateManager", "changed_slots", "EMPTY_EXPERT", "LayerPlan"]
