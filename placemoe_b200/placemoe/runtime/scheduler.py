"""When hot updates happen, and which one runs next.

Two periodic update kinds: a full update (new layout L and mapping M, with
expert-state migration) every ``layout_interval_steps`` and a mapping-only
update (new M on the current L) every ``mapping_interval_steps``, both only
for steps in ``(0, last_update_step]``.  Pending work is a single slot
holding the strongest kind seen since the last pop: a full update makes a
pending mapping-only one redundant (it recomputes M too), and repeated due
steps coalesce.

``HotUpdateController`` adds the one-job-at-a-time rule on top: while a
planner job is active nothing is popped, so events due meanwhile wait in the
pending slot and run when the job finishes.  Its ``failure_policy`` tells the
caller what a failed planner means: ``continue`` with the current placement or
``raise``.

The timeline (which steps are due, precedence of full over mapping-only,
the update window) is the reference's, so one YAML gives one update timeline:
veomni/distributed/moe/hiermoe/placemoe/runtime/scheduler.py:9-53 and
controller.py:12-50.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Any


class UpdateKind(str, Enum):
    FULL = "full"  # values are the planner's --update-mode names
    MAPPING_ONLY = "mapping"

    @property
    def strength(self) -> int:
        return 2 if self is UpdateKind.FULL else 1


def due_update(step: int, layout_every: int, mapping_every: int, last_step: int) -> UpdateKind | None:
    """The update that step ``step`` triggers on its own (None outside the window or between periods)."""
    if step <= 0 or step > last_step:
        return None
    for kind, every in ((UpdateKind.FULL, layout_every), (UpdateKind.MAPPING_ONLY, mapping_every)):
        if every > 0 and step % every == 0:
            return kind
    return None


@dataclass
class HotUpdateScheduler:
    layout_interval_steps: int
    mapping_interval_steps: int
    last_update_step: int
    pending: UpdateKind | None = None

    def observe_step(self, training_step: int) -> None:
        due = due_update(training_step, self.layout_interval_steps, self.mapping_interval_steps,
                         self.last_update_step)
        if due is not None and (self.pending is None or due.strength > self.pending.strength):
            self.pending = due

    def pop_next(self) -> UpdateKind | None:
        kind, self.pending = self.pending, None
        return kind


@dataclass
class HotUpdateController:
    layout_interval_steps: int
    mapping_interval_steps: int
    last_update_step: int
    failure_policy: str = "continue"
    active_job: Any = None
    scheduler: HotUpdateScheduler = field(init=False)

    def __post_init__(self) -> None:
        if self.failure_policy not in ("continue", "raise"):
            raise ValueError(f"failure_policy is 'continue' or 'raise', not {self.failure_policy!r}")
        self.scheduler = HotUpdateScheduler(self.layout_interval_steps, self.mapping_interval_steps,
                                            self.last_update_step)

    def observe_step(self, training_step: int) -> None:
        self.scheduler.observe_step(training_step)

    def next_update(self) -> UpdateKind | None:
        """The update to start now; None while a job runs (due events keep waiting)."""
        return self.scheduler.pop_next() if self.active_job is None else None

    def start(self, job) -> None:
        if self.active_job is not None:
            raise RuntimeError("one planner job at a time: a job is still active")
        self.active_job = job

    def finish(self):
        job = self.active_job
        self.active_job = None
        return job
