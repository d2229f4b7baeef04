"""PlaceMoE: profile-guided expert placement (replica counts, layout L, mapping M)."""

from .allocation import (bounded_group_shortlist, candidate_allocations, greedy_allocation, grouped_allocations,
                         instances_from_allocation, top_demand_allocation)
from .artifacts import (PLACEMOE_ARTIFACT_SCHEMA_VERSION, build_placemoe_artifact, load_artifact,
                        validate_placemoe_artifact, write_artifact)
from .evaluator import PlanCost, RouteReplayEvaluator
from .mapping import initialize_mapping, mapping_rank_loads, optimize_mapping, validate_instance_mapping
from .materialize import layout_from_ranks, materialize_plan, select_owners
from .optimizer import (OptimizationResult, OptimizerCandidate, OptimizerConfig, optimize_fixed_layout_mapping,
                        optimize_replica_allocation)
from .partition import PartitionConfig, PartitionResult, partition_items, partition_objective, spectral_embedding
from .placement import PlacementConfig, PlacementResult, place_instances, rank_placement_is_unique
from .seeds import eplb_plan, fixed_ep_plan, mirrored_r2_plan
from .statistics import profile_route_statistics, project_statistics_to_copies, uniform_copy_statistics
from .types import EMPTY_EXPERT, LayerPlan, PlaceMoETopology, ProfileStatistics, identity_plan

__all__ = [n for n in dir() if not n.startswith("_")]
