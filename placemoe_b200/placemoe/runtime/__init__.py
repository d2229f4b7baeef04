"""PlaceMoE runtime control: strict config, hot-update scheduling, planner process, CPU affinity."""

from .config import (CONFIG_ENV, HotUpdateConfig, PlaceMoECalibration, PlaceMoEConfigurationError,
                     PlaceMoEPlannerResources, PlaceMoERuntimeConfig)
from .cpu_affinity import CpuAffinityPlan, discover_physical_cores, format_cpu_list, parse_cpu_list, resolve_cpu_affinity
from .planner_process import HotUpdateJob, PlannerCommandSpec, build_planner_command, planner_environment
from .scheduler import HotUpdateController, HotUpdateScheduler, UpdateKind, due_update

__all__ = [
    "CONFIG_ENV", "HotUpdateConfig", "PlaceMoECalibration", "PlaceMoEConfigurationError", "PlaceMoEPlannerResources",
    "PlaceMoERuntimeConfig", "HotUpdateController", "CpuAffinityPlan", "discover_physical_cores", "format_cpu_list",
    "parse_cpu_list", "resolve_cpu_affinity", "HotUpdateJob", "PlannerCommandSpec", "build_planner_command",
    "planner_environment", "HotUpdateScheduler", "UpdateKind", "due_update",
]
