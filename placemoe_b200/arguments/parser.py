"""YAML + dotted CLI argument system.

    python tasks/train_text.py configs/olmoe.yaml --train.lr=1e-4 --model.preset=olmoe_1b_7b

The YAML has sections ``model``, ``data`` and ``train`` that map onto the
dataclasses below; ``--section.field=value`` overrides any field (values are
parsed as YAML scalars).  ``train.hiermoe`` carries the MoE placement knobs
used by the benchmark configurations.  ``save_args`` writes the resolved
arguments next to the checkpoints.

Reference parity: veomni/arguments/parser.py:161-229 and the dataclass tree
of veomni/arguments/arguments_types.py (ModelArguments, DataArguments,
TrainingArguments, HierMoEConfig :437-580).
"""

from __future__ import annotations

import dataclasses
import json
import os
import sys
from dataclasses import dataclass, field
from typing import Any

import yaml


@dataclass
class ModelArguments:
    preset: str = "olmoe_1b_7b"  # preset name (models/config.py) ...
    config_path: str = ""  # ... or a HuggingFace config.json / model directory
    weights_path: str = ""  # safetensors directory to load (optional)
    overrides: dict = field(default_factory=dict)  # field overrides of the model config


@dataclass
class DataArguments:
    train_path: str = "dummy"  # "dummy" = synthetic uniform token ids
    max_seq_len: int = 4096
    seed: int = 0


@dataclass
class HierMoEConfig:
    enable: bool = False
    token_dedup: bool = True
    communication_mode: str = "direct"  # one NVSwitch level: hierarchical modes resolve to direct
    redundant_slot_increment_per_device: int = 0
    capture_routes: bool = False
    route_capture_steps: int = 0  # capture the first N steps into route_root
    route_root: str = ""
    transport: str = "auto"  # "auto" (peer-memory kernels on CUDA), "nccl" (all-to-all baseline)


@dataclass
class TrainingArguments:
    output_dir: str = "output"
    global_batch_size: int = 8  # sequences per step over all ranks
    micro_batch_size: int = 2  # sequences per micro-batch per rank
    optimizer: str = "adamw"  # "adamw" | "muon"
    lr: float = 3e-4
    lr_warmup_ratio: float = 0.0
    lr_decay_style: str = "cosine"  # "constant" | "linear" | "cosine"
    lr_min_ratio: float = 0.1
    muon_lr: float = 0.02
    muon_momentum: float = 0.95
    weight_decay: float = 0.1
    max_grad_norm: float = 1.0
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    max_steps: int = 100
    seed: int = 0
    log_interval: int = 10
    save_steps: int = 0
    load_checkpoint_path: str = ""
    gradient_checkpointing: bool = False
    hiermoe: HierMoEConfig = field(default_factory=HierMoEConfig)


@dataclass
class Arguments:
    model: ModelArguments = field(default_factory=ModelArguments)
    data: DataArguments = field(default_factory=DataArguments)
    train: TrainingArguments = field(default_factory=TrainingArguments)


def _assign(obj, path: list[str], value: Any) -> None:
    head = path[0]
    if not hasattr(obj, head):
        raise ValueError(f"unknown argument {'.'.join(path)!r} on {type(obj).__name__}")
    if len(path) == 1:
        cur = getattr(obj, head)
        if dataclasses.is_dataclass(cur) and isinstance(value, dict):
            for k, v in value.items():
                _assign(cur, [k], v)
        elif isinstance(cur, tuple) and isinstance(value, list):
            setattr(obj, head, tuple(value))
        else:
            setattr(obj, head, value)
        return
    _assign(getattr(obj, head), path[1:], value)


def parse_args(argv: list[str] | None = None, cls=Arguments) -> Arguments:
    argv = list(sys.argv[1:] if argv is None else argv)
    args = cls()
    if argv and not argv[0].startswith("--"):
        with open(argv.pop(0)) as f:
            payload = yaml.safe_load(f) or {}
        for section, values in payload.items():
            _assign(args, [section], values)
    for item in argv:
        if not item.startswith("--") or "=" not in item:
            raise ValueError(f"expected --section.field=value, got {item!r}")
        key, raw = item[2:].split("=", 1)
        _assign(args, key.split("."), yaml.safe_load(raw))
    return args


def save_args(args: Arguments, output_dir: str) -> str:
    os.makedirs(output_dir, exist_ok=True)
    path = os.path.join(output_dir, "veomni_cli.yaml")
    with open(path, "w") as f:
        yaml.safe_dump(json.loads(json.dumps(dataclasses.asdict(args), default=list)), f)
    return path
