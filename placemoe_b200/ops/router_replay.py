"""Router replay: record each MoE layer's selected experts and substitute them later.

Modes: ``record`` keeps the top-k indices of every (layer, call) of a forward
pass; ``replay`` makes the router use recorded indices, with the routing
weights recomputed differentiably from the current logits at those experts
(so gradients still reach the router).  Used by RL-style training that must
score a batch with the routes that generated it.

Reference parity: veomni/utils/moe_router_replay.py:133-174 and its call
site in the patched Qwen3-MoE block (patched_modeling_qwen3_moe_gpu.py:346-378).
"""

from __future__ import annotations

import torch


class RouterReplay:
    def __init__(self):
        self.mode = "off"
        self._store: dict[tuple[int, int], torch.Tensor] = {}
        self._calls: dict[int, int] = {}

    def start_record(self) -> None:
        self.mode = "record"
        self._store.clear()
        self._calls.clear()

    def start_replay(self) -> None:
        self.mode = "replay"
        self._calls.clear()

    def stop(self) -> None:
        self.mode = "off"

    def _next_call(self, layer: int) -> int:
        c = self._calls.get(layer, 0)
        self._calls[layer] = c + 1
        return c

    def record(self, layer: int, idx: torch.Tensor) -> None:
        self._store[(layer, self._next_call(layer))] = idx.detach().clone()

    def fetch(self, layer: int) -> torch.Tensor:
        key = (layer, self._next_call(layer))
        if key not in self._store:
            raise KeyError(f"no recorded routes for layer {layer}, call {key[1]}")
        return self._store[key]

    def __len__(self) -> int:
        return len(self._store)


def replay_weights(logits: torch.Tensor, bias, idx: torch.Tensor, renorm: bool) -> torch.Tensor:
    """Routing weights of the given experts under the current logits (differentiable)."""
    z = logits.float() + (bias.float() if bias is not None else 0.0)
    p = torch.softmax(z, dim=-1)
    w = p.gather(1, idx.long())
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return w
