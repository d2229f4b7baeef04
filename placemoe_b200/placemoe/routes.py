"""Captured-route bundles (planner input).

On-disk format (an interchange format shared with the reference planner):
``<root>/step{S:04d}/layer{L:02d}_call{C}_all_ranks.pt`` holding
``{"format": "hiermoe-local-route-bundle-v1", "ep_size": N, "routes_by_rank": [LongTensor[T_r, k] x N], ...}``,
or per-rank files ``layer{L:02d}_call{C}_rank{R:02d}.pt`` holding ``{"routes", "ep_size"}``.
Routes are LOGICAL expert ids (the router's top-k before placement).

Reference parity: route capture at veomni/distributed/moe/hiermoe/expert_swap.py:10616-10682 and
the loader at scripts/profile/build_hiermoe_hierarchical_init_layout.py:195-251.
"""

from __future__ import annotations

import os
from pathlib import Path

import torch

ROUTE_BUNDLE_FORMAT = "hiermoe-local-route-bundle-v1"


def bundle_path(root, step: int, layer: int, call: int = 0) -> Path:
    return Path(root) / f"step{step:04d}" / f"layer{layer:02d}_call{call}_all_ranks.pt"


def write_route_bundle(root, step: int, layer: int, routes_by_rank, *, call: int = 0, extra: dict | None = None) -> Path:
    path = bundle_path(root, step, layer, call)
    path.parent.mkdir(parents=True, exist_ok=True)
    payload = {"format": ROUTE_BUNDLE_FORMAT, "ep_size": len(routes_by_rank), "step": step, "layer": layer,
               "routes_by_rank": [torch.as_tensor(r).detach().to("cpu", torch.long).contiguous() for r in routes_by_rank]}
    if extra:
        payload.update(extra)
    tmp = path.with_suffix(f".tmp{os.getpid()}")
    torch.save(payload, tmp)
    os.replace(tmp, path)
    return path


def load_routes(root, *, steps, layer: int, ep_size: int, call_indices=(0,)) -> list[list[torch.Tensor]]:
    samples = []
    root = Path(root)
    for step in steps:
        for call in call_indices:
            p = bundle_path(root, step, layer, call)
            if p.is_file():
                payload = torch.load(p, map_location="cpu", weights_only=False)
                rows = payload.get("routes_by_rank") if isinstance(payload, dict) else None
                if (not isinstance(payload, dict) or payload.get("format") != ROUTE_BUNDLE_FORMAT
                        or int(payload.get("ep_size", -1)) != ep_size or not isinstance(rows, (list, tuple))
                        or len(rows) != ep_size):
                    raise ValueError(f"Invalid bundled route capture: {p}.")
                out = []
                for r in rows:
                    if not torch.is_tensor(r) or r.ndim != 2:
                        raise ValueError(f"Invalid bundled route capture: {p}.")
                    out.append(r.to(torch.long).contiguous())
                samples.append(out)
                continue
            out = []
            for rank in range(ep_size):
                rp = root / f"step{step:04d}" / f"layer{layer:02d}_call{call}_rank{rank:02d}.pt"
                payload = torch.load(rp, map_location="cpu", weights_only=False)
                r = payload.get("routes") if isinstance(payload, dict) else None
                if not torch.is_tensor(r) or r.ndim != 2:
                    raise ValueError(f"Invalid route capture: {rp}.")
                if int(payload.get("ep_size", -1)) != ep_size:
                    raise ValueError(f"Route capture has a different EP size: {rp}.")
                out.append(r.to(torch.long).contiguous())
            samples.append(out)
    return samples


def available_steps(root) -> list[int]:
    root = Path(root)
    if not root.is_dir():
        return []
    return sorted(int(p.name[4:]) for p in root.iterdir() if p.is_dir() and p.name.startswith("step") and p.name[4:].isdigit())
