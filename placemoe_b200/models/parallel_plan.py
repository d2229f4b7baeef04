"""Declarative expert-parallel plan of the MoE decoders.

Expert tensors are split over the EP group along their first (expert) axis;
every other parameter is replicated on each GPU (dense weights stay resident,
their gradients are reduced in one flat bucket).  ``check_plan`` verifies a
built model against the plan: expert tensors hold exactly the topology's
slots per rank.

Reference parity: veomni/models/transformers/qwen3_moe/parallel_plan.py:6-16.
"""

from __future__ import annotations

import fnmatch

EP_PLAN = {
    "layers.*.mlp.gate_up_proj": "Shard(0)",
    "layers.*.mlp.down_proj": "Shard(0)",
}


def sharding_of(name: str) -> str:
    name = name[len("model."):] if name.startswith("model.") else name
    for pattern, spec in EP_PLAN.items():
        if fnmatch.fnmatch(name, pattern):
            return spec
    return "Replicate()"


def check_plan(model, slots_per_rank: int) -> list[str]:
    errors = []
    for name, p in model.named_parameters():
        if sharding_of(name) == "Shard(0)" and p.shape[0] != slots_per_rank:
            errors.append(f"{name}: {p.shape[0]} slots, plan expects {slots_per_rank}")
    return errors
