"""Hot-update scheduling: independent layout (full) and mapping-only intervals.

Events due at a step are coalesced; a full update subsumes a pending
mapping-only one; nothing is scheduled outside (0, last_update_step].

Reference parity: veomni/distributed/moe/hiermoe/placemoe/runtime/scheduler.py:9-53.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum


class UpdateKind(str, Enum):
    FULL = "full"
    MAPPING_ONLY = "mapping"


@dataclass
class HotUpdateScheduler:
    layout_interval_steps: int
    mapping_interval_steps: int
    last_update_step: int
    pending_full: bool = False
    pending_mapping: bool = False

    @staticmethod
    def _due(step: int, interval: int) -> bool:
        return interval > 0 and step % interval == 0

    def observe_step(self, training_step: int) -> None:
        if not 0 < training_step <= self.last_update_step:
            return
        if self._due(training_step, self.layout_interval_steps):
            self.pending_full, self.pending_mapping = True, False
        elif self._due(training_step, self.mapping_interval_steps):
            self.pending_mapping = True

    def pop_next(self) -> UpdateKind | None:
        if self.pending_full:
            self.pending_full = self.pending_mapping = False
            return UpdateKind.FULL
        if self.pending_mapping:
            self.pending_mapping = False
            return UpdateKind.MAPPING_ONLY
        return None
