"""Process-wide MoE-parallel state and its fail-fast validation.

``configure_hiermoe`` validates the combination of settings before any model
is built and records the resolved state (process group, EP size, the
dispatch mode actually used, the perf model) for the rest of the framework:

* placement (replica slots or an artifact) requires expert weights that are
  not additionally sharded over data parallelism (``ep_fsdp_size == 1``) and
  no optimizer/parameter CPU offload (migration moves device state);
* hierarchical (multi-stage) dedup is requested per node level; on one
  NVSwitch domain (EP size <= ranks per node) every mode resolves to direct
  rank-level dedup, and multi-node hierarchical modes need a fitted perf model;
* token dedup needs the dedup-capable transports (peer-memory or NCCL).

Reference parity: veomni/distributed/moe/hiermoe/state.py:55-255 (state,
configure_hiermoe and its checks at :152-171), :505-525 (metrics access).
"""

from __future__ import annotations

import dataclasses

_MODES = ("direct", "hierarchical", "two_stage", "three_stage")


class HierMoEConfigurationError(ValueError):
    pass


@dataclasses.dataclass
class HierMoEState:
    enabled: bool
    ep_size: int
    ranks_per_node: int
    requested_mode: str
    mode: str
    token_dedup: bool
    redundant_slots_per_rank: int
    transport: str
    activation_checkpointing: bool
    perf_model: object | None = None
    ep_group: object | None = None


_STATE: HierMoEState | None = None


def configure_hiermoe(config, *, ep_size: int, ranks_per_node: int | None = None, ep_group=None,
                      ep_fsdp_size: int = 1, activation_checkpointing_enabled: bool = False,
                      fsdp_offload_enabled: bool = False, perf_model=None, has_artifact: bool = False) -> HierMoEState:
    """Validate and record the MoE-parallel settings (``config`` is an arguments HierMoEConfig)."""
    global _STATE
    rpn = ranks_per_node or ep_size
    mode = getattr(config, "communication_mode", "direct")
    if mode not in _MODES:
        raise HierMoEConfigurationError(f"communication_mode must be one of {_MODES}, got {mode!r}")
    redundant = int(getattr(config, "redundant_slot_increment_per_device", 0))
    placement = redundant > 0 or has_artifact
    if placement and ep_fsdp_size != 1:
        raise HierMoEConfigurationError("expert placement needs ep_fsdp_size == 1 (expert slots are not sharded "
                                        "over data parallelism)")
    if placement and fsdp_offload_enabled:
        raise HierMoEConfigurationError("expert placement does not support CPU offload: migration moves device state")
    if redundant < 0:
        raise HierMoEConfigurationError("redundant_slot_increment_per_device must be >= 0")
    single_level = ep_size <= rpn
    if single_level:
        resolved = "direct"
    else:
        if mode != "direct" and perf_model is None:
            raise HierMoEConfigurationError(f"communication_mode {mode!r} across nodes needs a fitted perf model")
        resolved = perf_model.select_dimension() if (perf_model is not None and mode != "direct") else "direct"
    transport = getattr(config, "transport", "auto")
    if transport not in ("auto", "p2p", "nccl"):
        raise HierMoEConfigurationError(f"transport must be auto, p2p or nccl, got {transport!r}")
    _STATE = HierMoEState(enabled=bool(getattr(config, "enable", False)) or placement, ep_size=ep_size,
                          ranks_per_node=rpn, requested_mode=mode, mode=resolved,
                          token_dedup=bool(getattr(config, "token_dedup", True)),
                          redundant_slots_per_rank=redundant, transport=transport,
                          activation_checkpointing=activation_checkpointing_enabled, perf_model=perf_model,
                          ep_group=ep_group)
    return _STATE


def get_hiermoe_state() -> HierMoEState | None:
    return _STATE


def reset_hiermoe_state() -> None:
    global _STATE
    _STATE = None


def checkpoint_state(model) -> dict:
    """Placement state of every MoE layer (the extra_state payload that checkpoints carry)."""
    out = {"version": 3, "layers": {}}
    for blk in model.moe_blocks():
        pl = blk.placement
        if pl is None:
            continue
        out["layers"][blk.layer_key] = {
            "num_experts": int(blk.cfg.num_experts), "num_local_experts": int(pl.slots_per_rank),
            "slot_to_logical": [int(x) for x in pl.slot_to_logical],
            "owner_slots": [int(x) for x in pl.owner_slots],
            "source_logical_to_physical": [[int(x) for x in row] for row in pl.mapping],
            "placement_version": int(pl.version),
        }
    return out
