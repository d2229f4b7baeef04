"""Checkpoint / resume (torch.distributed.checkpoint) and HuggingFace export.

Directory layout: ``<root>/global_step_<N>/`` holding the DCP shards of the
model and optimizer state plus ``extra_state_rank<r>.json`` /
``extra_state.json`` (global step, RNG, learning-rate schedule position and the
``placemoe`` placement state: layout L, owners, mapping M and version of every
MoE layer).

Expert weights and their AdamW moments are stored per LOGICAL expert
(``model.layers.{i}.mlp.experts.{e}.gate_up_proj`` ...), written by the
rank holding the expert's owner copy.  Loading reads, for every local slot,
the logical expert it holds under the CURRENT placement, so a checkpoint
restores onto any layout, mapping or EP size; replicas are filled from the
same logical tensor and stay identical.  Dense parameters are replicated and
deduplicated by DCP.

``export_hf`` writes a HuggingFace-style safetensors directory with logical
experts (gathered from owner copies), split q/k/v projections and the
config.json of the model family.

Reference parity: veomni/checkpoint/dcp_checkpointer.py:53-615 and
checkpointer.py:30-93 (DCP + extra_state), veomni/utils/save_safetensor_utils.py
(HF export; the reference refuses non-identity placements, this exporter
gathers logical experts instead).
"""

from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp

from ..parallel.data_parallel import is_expert_param
from ..placemoe.types import LayerPlan

EXTRA_STATE = "extra_state.json"


def _world():
    return (dist.get_rank(), dist.get_world_size()) if dist.is_initialized() else (0, 1)


def _expert_key(layer_key: str, e: int, name: str) -> str:
    return f"{layer_key}.{e}.{name}"


def _owned_slots(blk):
    """(local slot, logical expert) pairs whose copy is the expert's owner."""
    pl = blk.placement
    out = []
    for j in range(pl.slots_per_rank):
        if not pl.is_redundant_local_slot(j):
            out.append((j, int(pl.local_logical[j])))
    return out


def _state_dicts(trainer, for_load: bool):
    """Model/optimizer state keyed by logical names; for loading, every local slot requests its expert."""
    from ..optim import state_tensors

    model, opt = trainer.model, trainer.optimizer
    ms, os_ = {}, {}
    for name, p in model.named_parameters():
        if is_expert_param(name):
            continue
        ms[name] = p.data
        for sk, t in state_tensors(opt, p):
            os_[f"{name}.{sk}"] = t
    for blk in model.moe_blocks():
        pl = blk.placement
        pairs = ([(j, int(pl.local_logical[j])) for j in range(pl.slots_per_rank) if pl.local_logical[j] >= 0]
                 if for_load else _owned_slots(blk))
        for pname in ("gate_up_proj", "down_proj"):
            p = getattr(blk, pname)
            sts = state_tensors(opt, p)
            for j, e in pairs:
                key = _expert_key(blk.layer_key, e, pname)
                if for_load and key in ms:  # second local copy of the same expert: filled after load
                    continue
                ms[key] = p.data[j]
                for sk, t in sts:
                    os_[f"{key}.{sk}"] = t[j]
    return ms, os_


def _placement_state(trainer) -> dict:
    out = {}
    for blk in trainer.model.moe_blocks():
        pl = blk.placement
        out[blk.layer_key] = {**pl.plan.to_runtime_payload(), "version": pl.version}
    return out


def _sync_params(trainer) -> None:
    """Sharded optimizers write their current masters into ``param.data`` (collective)."""
    sync = getattr(trainer.optimizer, "sync_params", None)
    if sync is not None:
        sync()


def _reload_params(trainer) -> None:
    """Optimizers that keep their own copies re-read loaded ``param.data`` / state."""
    reload = getattr(trainer.optimizer, "reload_from_params", None)
    if reload is not None:
        reload()


def save_checkpoint(trainer, root: str) -> str:
    rank, _ = _world()
    path = os.path.join(root, f"global_step_{trainer.global_step}")
    os.makedirs(path, exist_ok=True)
    _sync_params(trainer)
    # make sure optimizer state exists for every parameter (zeros before the first step)
    for p in trainer.model.parameters():
        trainer.optimizer._state(p)
    ms, os_ = _state_dicts(trainer, for_load=False)
    dcp.save({"model": ms, "optimizer": os_}, checkpoint_id=path)
    if rank == 0:
        extra = {
            "global_step": trainer.global_step,
            "optimizer_step": max((st.get("step", 0) for st in trainer.optimizer.state.values()), default=0),
            "torch_rng_state": torch.get_rng_state().tolist()[:16],
            "placemoe": _placement_state(trainer),
            "topology": {"ep_size": trainer.topology.ep_size, "ranks_per_node": trainer.topology.ranks_per_node,
                         "num_experts": trainer.topology.num_experts,
                         "slots_per_rank": trainer.topology.slots_per_rank},
        }
        with open(os.path.join(path, EXTRA_STATE), "w") as f:
            json.dump(extra, f)
    if dist.is_initialized():
        dist.barrier()
    return path


def placement_digest(trainer) -> int:
    """Cheap digest of the placement state (agreement check across ranks before a load)."""
    h = 0
    for key, row in _placement_state(trainer).items():
        for v in (row["slot_to_logical"] + sum(row["source_logical_to_physical"], []) + row["owner_slots"]):
            h = (h * 1000003 + int(v) + 7) % (1 << 61)
    return h


def load_checkpoint(trainer, path: str, *, restore_placement: bool = True) -> dict:
    """Restore model + optimizer (+ placement when the topology matches) from ``global_step_N``."""
    from ..optim import state_tensors

    if os.path.basename(os.path.normpath(path)).startswith("global_step_") is False:
        steps = sorted(int(d.split("_")[-1]) for d in os.listdir(path) if d.startswith("global_step_"))
        if not steps:
            raise FileNotFoundError(f"no global_step_* under {path}")
        path = os.path.join(path, f"global_step_{steps[-1]}")
    with open(os.path.join(path, EXTRA_STATE)) as f:
        extra = json.load(f)
    topo = extra.get("topology", {})
    same_topology = (topo.get("ep_size") == trainer.topology.ep_size
                     and topo.get("slots_per_rank") == trainer.topology.slots_per_rank)
    if restore_placement and same_topology:
        for blk in trainer.model.moe_blocks():
            row = extra["placemoe"].get(blk.layer_key)
            if row is None:
                continue
            plan = LayerPlan.from_runtime_payload(row)
            blk.placement.install_layout(plan)
            blk.placement.version = int(row.get("version", 0))
    # the preflight digest must agree on every rank before tensors are read
    if dist.is_initialized():
        d = torch.tensor([placement_digest(trainer) % (1 << 62)], dtype=torch.int64)
        lo, hi = d.clone(), d.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        if int(lo) != int(hi):
            raise RuntimeError("placement state differs across ranks; refusing to load")
    for p in trainer.model.parameters():
        trainer.optimizer._state(p)
    ms, os_ = _state_dicts(trainer, for_load=True)
    state = {"model": ms, "optimizer": os_}
    dcp.load(state, checkpoint_id=path)
    # fill second copies of experts held twice on one rank, and bump versions so bf16 copies refresh
    for blk in trainer.model.moe_blocks():
        pl = blk.placement
        first = {}
        for j in range(pl.slots_per_rank):
            e = int(pl.local_logical[j])
            if e < 0:
                continue
            if e in first:
                for pname in ("gate_up_proj", "down_proj"):
                    p = getattr(blk, pname)
                    p.data[j].copy_(p.data[first[e]])
                    for _, t in state_tensors(trainer.optimizer, p):
                        t[j].copy_(t[first[e]])
            else:
                first[e] = j
    with torch.no_grad():
        for p in trainer.model.parameters():
            p.add_(0)  # bump the version counter: compute copies are refreshed on next use
    step = int(extra.get("optimizer_step", 0))
    for st in trainer.optimizer.state.values():
        st["step"] = step
    trainer.global_step = int(extra["global_step"])
    trainer.optimizer.reset_tables()
    _reload_params(trainer)
    return extra


# ----------------------------------------------------------------------- HF export
def _hf_names(cfg, li: int):
    p = f"model.layers.{li}"
    return {
        "input_layernorm": f"{p}.input_layernorm.weight",
        "post_attention_layernorm": f"{p}.post_attention_layernorm.weight",
        "q": f"{p}.self_attn.q_proj.weight", "k": f"{p}.self_attn.k_proj.weight",
        "v": f"{p}.self_attn.v_proj.weight", "o": f"{p}.self_attn.o_proj.weight",
        "q_norm": f"{p}.self_attn.q_norm.weight", "k_norm": f"{p}.self_attn.k_norm.weight",
        "gate": f"{p}.mlp.gate.weight",
        "expert": f"{p}.mlp.experts.{{e}}.{{w}}.weight",
        "dense": f"{p}.mlp.{{w}}.weight",
    }


def export_hf(trainer, out_dir: str) -> str | None:
    """HuggingFace safetensors export with logical experts, or the dense MLP (rank 0 writes)."""
    from safetensors.torch import save_file

    rank, world = _world()
    _sync_params(trainer)
    model, cfg = trainer.model, trainer.model_cfg
    tensors: dict[str, torch.Tensor] = {}
    inter = cfg.moe_intermediate_size
    for li, layer in enumerate(model.layers):
        n = _hf_names(cfg, li)
        blk = layer.mlp
        owned = {}
        dense = cfg.is_dense
        if dense and rank == 0:
            gu = blk.w_gate_up.data[0].to("cpu", torch.bfloat16)
            tensors[n["dense"].format(w="gate_proj")] = gu[: cfg.intermediate_size].clone()
            tensors[n["dense"].format(w="up_proj")] = gu[cfg.intermediate_size:].clone()
            tensors[n["dense"].format(w="down_proj")] = blk.w_down.data[0].to("cpu", torch.bfloat16)
        for j, e in ([] if dense else _owned_slots(blk)):
            gu = blk.gate_up_proj.data[j].to("cpu", torch.bfloat16)
            owned[e] = (gu[:inter].clone(), gu[inter:].clone(), blk.down_proj.data[j].to("cpu", torch.bfloat16))
        if world > 1 and not dense:
            gathered = [None] * world
            dist.all_gather_object(gathered, owned)
            owned = {k: v for d in gathered for k, v in d.items()}
        if rank != 0:
            continue
        for e, (g, u, d) in owned.items():
            tensors[n["expert"].format(e=e, w="gate_proj")] = g
            tensors[n["expert"].format(e=e, w="up_proj")] = u
            tensors[n["expert"].format(e=e, w="down_proj")] = d
        at = layer.self_attn
        qkv = at.qkv_proj.data.to("cpu", torch.bfloat16)
        tensors[n["q"]] = qkv[: cfg.q_size].clone()
        tensors[n["k"]] = qkv[cfg.q_size: cfg.q_size + cfg.kv_size].clone()
        tensors[n["v"]] = qkv[cfg.q_size + cfg.kv_size:].clone()
        tensors[n["o"]] = at.o_proj.data.to("cpu", torch.bfloat16)
        if at.q_norm is not None:
            tensors[n["q_norm"]] = at.q_norm.data.to("cpu", torch.bfloat16)
            tensors[n["k_norm"]] = at.k_norm.data.to("cpu", torch.bfloat16)
        tensors[n["input_layernorm"]] = layer.input_layernorm.weight.data.to("cpu", torch.bfloat16)
        tensors[n["post_attention_layernorm"]] = layer.post_attention_layernorm.weight.data.to("cpu", torch.bfloat16)
        if not dense:
            tensors[n["gate"]] = blk.gate.data.to("cpu", torch.bfloat16)
    if rank != 0:
        return None
    tensors["model.embed_tokens.weight"] = model.embed_tokens.data.to("cpu", torch.bfloat16)
    tensors["model.norm.weight"] = model.norm.weight.data.to("cpu", torch.bfloat16)
    if model.lm_head is not None:
        tensors["lm_head.weight"] = model.lm_head.data.to("cpu", torch.bfloat16)
    os.makedirs(out_dir, exist_ok=True)
    save_file(tensors, os.path.join(out_dir, "model.safetensors"), metadata={"format": "pt"})
    arch = {"olmoe": "OlmoeForCausalLM", "qwen3": "Qwen3ForCausalLM", "llama": "LlamaForCausalLM"}
    hf_cfg = {
        "model_type": cfg.model_type, "architectures": [arch.get(cfg.model_type, "Qwen3MoeForCausalLM")],
        "vocab_size": cfg.vocab_size, "hidden_size": cfg.hidden_size, "num_hidden_layers": cfg.num_hidden_layers,
        "num_attention_heads": cfg.num_attention_heads, "num_key_value_heads": cfg.num_key_value_heads,
        "head_dim": cfg.head_dim, "moe_intermediate_size": cfg.moe_intermediate_size,
        "intermediate_size": cfg.intermediate_size if cfg.is_dense else cfg.moe_intermediate_size,
        "num_experts": cfg.num_experts,
        "num_experts_per_tok": cfg.num_experts_per_tok, "norm_topk_prob": cfg.norm_topk_prob,
        "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.rms_norm_eps,
        "router_aux_loss_coef": cfg.router_aux_loss_coef, "tie_word_embeddings": cfg.tie_word_embeddings,
        "torch_dtype": "bfloat16",
    }
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(hf_cfg, f, indent=2)
    return out_dir


def load_hf_weights(trainer, hf_dir: str) -> None:
    """Load a HuggingFace safetensors directory (logical experts) into the current placement."""
    from safetensors import safe_open

    model, cfg = trainer.model, trainer.model_cfg
    files = [os.path.join(hf_dir, f) for f in sorted(os.listdir(hf_dir)) if f.endswith(".safetensors")]
    handles = [safe_open(f, framework="pt") for f in files]

    def get(name):
        for h in handles:
            if name in h.keys():
                return h.get_tensor(name)
        raise KeyError(name)

    with torch.no_grad():
        model.embed_tokens.copy_(get("model.embed_tokens.weight"))
        model.norm.weight.copy_(get("model.norm.weight"))
        if model.lm_head is not None:
            model.lm_head.copy_(get("lm_head.weight"))
        for li, layer in enumerate(model.layers):
            n = _hf_names(cfg, li)
            at = layer.self_attn
            at.qkv_proj.copy_(torch.cat([get(n["q"]), get(n["k"]), get(n["v"])], 0))
            at.o_proj.copy_(get(n["o"]))
            if at.q_norm is not None:
                at.q_norm.copy_(get(n["q_norm"]))
                at.k_norm.copy_(get(n["k_norm"]))
            layer.input_layernorm.weight.copy_(get(n["input_layernorm"]))
            layer.post_attention_layernorm.weight.copy_(get(n["post_attention_layernorm"]))
            blk = layer.mlp
            if cfg.is_dense:
                blk.w_gate_up[0].copy_(torch.cat([get(n["dense"].format(w="gate_proj")),
                                                  get(n["dense"].format(w="up_proj"))], 0))
                blk.w_down[0].copy_(get(n["dense"].format(w="down_proj")))
                continue
            blk.gate.copy_(get(n["gate"]))
            for j, e in enumerate(blk.placement.local_logical.tolist()):
                if e < 0:
                    continue
                g = get(n["expert"].format(e=e, w="gate_proj"))
                u = get(n["expert"].format(e=e, w="up_proj"))
                blk.gate_up_proj[j].copy_(torch.cat([g, u], 0))
                blk.down_proj[j].copy_(get(n["expert"].format(e=e, w="down_proj")))
    _reload_params(trainer)


__all__ = ["save_checkpoint", "load_checkpoint", "export_hf", "load_hf_weights", "placement_digest"]
