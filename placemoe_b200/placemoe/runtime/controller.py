"""Single-job lifecycle of asynchronous planner runs.

At most one planner job is active; while it runs, due events stay pending in
the scheduler and are popped once the job finishes.  ``failure_policy`` is
``continue`` (keep the current placement) or ``raise``.

Reference parity: veomni/distributed/moe/hiermoe/placemoe/runtime/controller.py:12-50.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .planner_process import HotUpdateJob
from .scheduler import HotUpdateScheduler, UpdateKind


@dataclass
class HotUpdateController:
    layout_interval_steps: int
    mapping_interval_steps: int
    last_update_step: int
    failure_policy: str = "continue"
    active_job: HotUpdateJob | None = None
    scheduler: HotUpdateScheduler = field(init=False)

    def __post_init__(self):
        if self.failure_policy not in ("continue", "raise"):
            raise ValueError("failure_policy must be 'continue' or 'raise'.")
        self.scheduler = HotUpdateScheduler(self.layout_interval_steps, self.mapping_interval_steps,
                                            self.last_update_step)

    def observe_step(self, training_step: int) -> None:
        self.scheduler.observe_step(training_step)

    def next_update(self) -> UpdateKind | None:
        return None if self.active_job is not None else self.scheduler.pop_next()

    def start(self, job: HotUpdateJob) -> None:
        if self.active_job is not None:
            raise RuntimeError("a PlaceMoE planner job is already active.")
        self.active_job = job

    def finish(self) -> HotUpdateJob | None:
        job, self.active_job = self.active_job, None
        return job
