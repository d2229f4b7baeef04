"""Qwen3-MoE / OLMoE-shaped decoder built from placemoe_b200 ops.

Layer:  h = x + o_proj(attn(qk_norm_rope(qkv_proj(rmsnorm(x)))))
        y = h + moe(rmsnorm(h))
        (each residual add runs inside the RMSNorm that follows it: ``forward_fused``)

* Attention projections are one fused QKV weight ``[(Hq + 2 Hkv) D, H]``.
* The MoE block keeps fp32 master expert weights for the physical slots this
  rank holds (``gate_up_proj [S, 2I, H]`` with gate rows first, then up rows,
  and ``down_proj [S, H, I]``) plus bf16 compute copies that the fused AdamW
  kernel refreshes (``bf16_shadow``).
* With expert parallelism the block routes through
  :mod:`placemoe_b200.parallel.ep`; without it through :func:`ops.moe.moe_block`.

CUDA tensors take the sm_100a kernels; CPU tensors take the PyTorch reference
paths (gloo tests, numerical oracle).

Reference parity: Qwen3MoeDecoderLayer / Qwen3MoeSparseMoeBlock / Qwen3MoeExperts
(veomni/models/transformers/qwen3_moe/generated/patched_modeling_qwen3_moe_gpu.py:257-378)
and the OLMoE modeling in veomni/models/transformers/olmoe.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import attention as attn_ops
from ..ops import loss as loss_ops
from ..ops import moe as moe_ops
from ..ops import mp as mp_ops
from ..ops import norm as norm_ops
from .config import MoEModelConfig, zipf_router_bias


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        return mp_ops.rmsnorm(x, self.weight, self.eps)

    def add_norm(self, x, res):
        """(x + res, norm(x + res)); (x, norm(x)) when ``res`` is None."""
        return mp_ops.add_rmsnorm(x, res, self.weight, self.eps)


class Attention(nn.Module):
    def __init__(self, cfg: MoEModelConfig):
        super().__init__()
        self.cfg = cfg
        h, d = cfg.hidden_size, cfg.head_dim
        self.hq, self.hkv, self.d = cfg.num_attention_heads, cfg.num_key_value_heads, d
        self.qkv_proj = nn.Parameter(torch.empty(cfg.q_size + 2 * cfg.kv_size, h))
        self.o_proj = nn.Parameter(torch.empty(h, cfg.q_size))
        if cfg.qk_norm == "per_head":
            self.q_norm = nn.Parameter(torch.ones(d))
            self.k_norm = nn.Parameter(torch.ones(d))
            self.q_group, self.k_group = d, d
        elif cfg.qk_norm == "full":
            self.q_norm = nn.Parameter(torch.ones(cfg.q_size))
            self.k_norm = nn.Parameter(torch.ones(cfg.kv_size))
            self.q_group, self.k_group = cfg.q_size, cfg.kv_size
        else:
            self.q_norm = self.k_norm = None
            self.q_group = self.k_group = 0
        self.register_buffer("inv_freq", norm_ops.rope_inv_freq(d, cfg.rope_theta), persistent=False)

    def forward(self, x, pos, seq_len, docs=None):
        # x: [T, H] (T = batch * seq_len, packed by sequence); docs: per-token document bounds.
        # With Ulysses sequence parallelism (self.sp) x holds this rank's chunk of seq_len tokens of
        # every sequence; q, k, v are re-split by heads around the attention over whole sequences.
        sp = getattr(self, "sp", None)
        full = seq_len * (sp.size if sp is not None else 1)
        qkv = mp_ops.linear(x, self.qkv_proj)
        q, k, v = norm_ops.qkv_norm_rope(qkv, self.q_norm, self.k_norm, pos, self.inv_freq, self.hq, self.hkv,
                                         self.d, self.q_group, self.k_group, self.cfg.rms_norm_eps,
                                         max_pos=full)
        if sp is None:
            o = attn_ops.causal_attention(q, k, v, seq_len, docs)  # [T, Hq, D]
            o = o.reshape(o.shape[0], -1)
        else:
            from ..parallel.ulysses import heads_to_seq, seq_to_heads

            b = x.shape[0] // seq_len
            q, k, v = (seq_to_heads(t, sp, b, seq_len) for t in (q, k, v))
            o = attn_ops.causal_attention(q, k, v, full, docs)  # [B*S, Hq/P, D]; docs of the whole rows
            o = heads_to_seq(o, sp, b, seq_len)
        return mp_ops.linear(o, self.o_proj)


class MoEBlock(nn.Module):
    """Router + experts for the physical slots held by this rank.

    ``placement`` (a :class:`placemoe_b200.parallel.placement.LayerPlacement`)
    maps logical experts to physical slots; ``ep`` (an
    :class:`placemoe_b200.parallel.ep.ExpertParallel`) performs the multi-rank
    dispatch/combine.  Without either, slots == logical experts on one device.
    """

    def __init__(self, cfg: MoEModelConfig, layer_idx: int, num_local_slots: int | None = None):
        super().__init__()
        self.cfg = cfg
        self.layer_idx = layer_idx
        h, i, e = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts
        s = e if num_local_slots is None else num_local_slots
        self.gate = nn.Parameter(torch.empty(e, h))
        self.gate_up_proj = nn.Parameter(torch.empty(s, 2 * i, h))
        self.down_proj = nn.Parameter(torch.empty(s, h, i))
        seed = layer_idx if cfg.router_bias_seed_per_layer else 0
        bias = zipf_router_bias(e, cfg.router_bias_zipf_s, cfg.router_bias_scale, seed)
        self.register_buffer("router_bias", torch.tensor(bias, dtype=torch.float32), persistent=False)
        self.placement = None  # set by the placement runtime
        self.ep = None  # set by parallelize
        self.layer_key = f"model.layers.{layer_idx}.mlp.experts"
        self.last_aux_loss = None
        self.last_route = None  # [T, k] logical routes of the last forward (route capture)
        self.route_sink = None  # RouteRecorder when routes are captured for the planner
        self.keep_expert_rows = True  # False: recompute dispatched rows in the backward (less memory)
        self.router_replay = None  # ops.router_replay.RouterReplay (record / replay selected experts)

    @property
    def num_local_slots(self) -> int:
        return self.gate_up_proj.shape[0]

    # ---------------------------------------------------------------- bf16 copies
    def compute_weights(self):
        """bf16 compute copies of the expert weights, refreshed when the masters change."""
        out = []
        for p in (self.gate_up_proj, self.down_proj):
            sh = getattr(p, "bf16_shadow", None)
            ver = p._version
            if sh is None or sh.shape != p.shape or sh.device != p.device:
                sh = p.detach().to(torch.bfloat16)
                p.bf16_shadow = sh
                p._shadow_version = ver
            elif getattr(p, "_shadow_version", None) != ver and not getattr(p, "_shadow_by_optimizer", False):
                sh.copy_(p.detach())
                p._shadow_version = ver
            out.append(sh)
        return out

    def forward(self, x):
        cfg = self.cfg
        t = x.shape[0]
        bias = self.router_bias if cfg.router_bias_zipf_s else None
        aux_coef = cfg.router_aux_loss_coef if self.training else 0.0
        if self.ep is not None:
            y, aux, route = self.ep.moe_forward(self, x, bias, aux_coef)
        elif x.is_cuda:
            w1, w2 = self.compute_weights()
            lut = self.placement.local_lut_device(x.device) if self.placement is not None else None
            y, aux, route = moe_ops.moe_block(x, self.gate, bias, w1, w2, self.gate_up_proj, self.down_proj,
                                              cfg.num_experts_per_tok, cfg.norm_topk_prob, self.num_local_slots,
                                              lut=lut, aux_coef=aux_coef, keep_rows=self.keep_expert_rows,
                                              replay=self.router_replay, layer=self.layer_idx)
        else:
            lut = self.placement.local_lut_cpu() if self.placement is not None else None
            y, aux, route = moe_ops.moe_block_reference(x, self.gate, bias, self.gate_up_proj, self.down_proj,
                                                        cfg.num_experts_per_tok, cfg.norm_topk_prob, aux_coef, lut,
                                                        return_route=True, replay=self.router_replay,
                                                        layer=self.layer_idx)
        self.last_aux_loss = aux
        self.last_route = route
        if self.route_sink is not None and route is not None:
            self.route_sink.collect(self, route)
        return y


class DenseMLP(nn.Module):
    """SwiGLU MLP of the dense families (Llama, Qwen3 dense): down(silu(gate x) * up x).

    The gate and up projections are one [1, 2I, H] tensor (gate rows first) and
    the down projection [1, H, I], so the CUDA path runs the fused SwiGLU
    grouped GEMM with a single group.  The names differ from the expert
    tensors on purpose: these weights are replicated and reduced like every
    other dense parameter.
    """

    def __init__(self, cfg: MoEModelConfig):
        super().__init__()
        h, i = cfg.hidden_size, cfg.intermediate_size
        self.w_gate_up = nn.Parameter(torch.empty(1, 2 * i, h))
        self.w_down = nn.Parameter(torch.empty(1, h, i))
        self.last_aux_loss = None

    def forward(self, x):
        return moe_ops.dense_swiglu_mlp(x, self.w_gate_up, self.w_down)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: MoEModelConfig, layer_idx: int, num_local_slots: int | None = None):
        super().__init__()
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.self_attn = Attention(cfg)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.mlp = DenseMLP(cfg) if cfg.is_dense else MoEBlock(cfg, layer_idx, num_local_slots)

    def forward(self, x, pos, seq_len, docs=None):
        h, m = self.forward_fused(x, None, pos, seq_len, docs)
        return h + m

    def forward_fused(self, x, branch, pos, seq_len, docs=None):
        """The layer on the residual stream x + branch (branch: the previous layer's MLP output, not yet
        added).  Returns (residual after attention, MLP output): each residual add runs inside the
        norm that follows it."""
        h, n = self.input_layernorm.add_norm(x, branch)
        h, n = self.post_attention_layernorm.add_norm(h, self.self_attn(n, pos, seq_len, docs))
        return h, self.mlp(n)


class MoEForCausalLM(nn.Module):
    def __init__(self, cfg: MoEModelConfig, num_local_slots: int | None = None):
        super().__init__()
        self.config = cfg
        self.embed_tokens = nn.Parameter(torch.empty(cfg.vocab_size, cfg.hidden_size))
        self.layers = nn.ModuleList(DecoderLayer(cfg, i, num_local_slots) for i in range(cfg.num_hidden_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.lm_head = None if cfg.tie_word_embeddings else nn.Parameter(torch.empty(cfg.vocab_size, cfg.hidden_size))
        self.gradient_checkpointing = False

    # ------------------------------------------------------------------ init
    @torch.no_grad()
    def init_weights(self, seed: int = 0, expert_init=None):
        """Random init: N(0, initializer_range) for matrices, ones for norms (drawn on the params' device).

        ``expert_init(layer_idx, name, tensor)`` may fill expert tensors (used to
        slice logical experts into physical slots consistently across ranks).
        """
        std = self.config.initializer_range
        gens: dict = {}

        def normal_(t, salt):
            dev = t.device
            g = torch.Generator(device=dev)
            g.manual_seed(seed * 1000003 + salt)
            t.normal_(0.0, std, generator=g)

        normal_(self.embed_tokens, 1)
        if self.lm_head is not None:
            normal_(self.lm_head, 2)
        for li, layer in enumerate(self.layers):
            base = 16 * (li + 1)
            normal_(layer.self_attn.qkv_proj, base + 1)
            normal_(layer.self_attn.o_proj, base + 2)
            if isinstance(layer.mlp, DenseMLP):
                normal_(layer.mlp.w_gate_up, base + 4)
                normal_(layer.mlp.w_down, base + 5)
                continue
            normal_(layer.mlp.gate, base + 3)
            if expert_init is None:
                normal_(layer.mlp.gate_up_proj, base + 4)
                normal_(layer.mlp.down_proj, base + 5)
            else:
                expert_init(li, "gate_up_proj", layer.mlp.gate_up_proj)
                expert_init(li, "down_proj", layer.mlp.down_proj)
        del gens
        return self

    def moe_blocks(self):
        return [layer.mlp for layer in self.layers if isinstance(layer.mlp, MoEBlock)]

    def expert_parameters(self):
        for blk in self.moe_blocks():
            yield blk.gate_up_proj
            yield blk.down_proj

    # --------------------------------------------------------------- forward
    def _anchor(self, device):
        a = getattr(self, "_grad_anchor", None)
        if a is None or a.device != device:
            a = torch.zeros((), device=device, requires_grad=True)
            self._grad_anchor = a
        return a

    def hidden_states(self, input_ids: torch.Tensor, cu_seqlens: torch.Tensor | None = None) -> torch.Tensor:
        """``cu_seqlens``: cumulative document boundaries over the flattened tokens when rows pack
        several documents (positions restart and attention stays inside each document)."""
        b, s = input_ids.shape
        ids = input_ids.reshape(-1)
        x = mp_ops.embedding(ids, self.embed_tokens, self._anchor(ids.device))
        docs = None
        sp = getattr(self, "sp", None)
        if sp is not None and cu_seqlens is not None:
            # cu_seqlens covers the whole sequences of the group (b rows of P*s tokens); attention runs on
            # whole sequences, so the document bounds are those of the full rows, and the positions are
            # this rank's chunk of the full rows' in-document positions
            full = s * sp.size
            docs = attn_ops.doc_bounds(cu_seqlens.to(ids.device), b * full, full)
            pos_full = torch.arange(full, device=ids.device, dtype=torch.int32).repeat(b) - docs[0]
            pos = pos_full.view(b, full)[:, sp.rank * s:(sp.rank + 1) * s].reshape(-1).to(torch.int32).contiguous()
        elif sp is not None:  # this rank's chunk of every sequence starts at position rank * s
            pos = (torch.arange(s, device=ids.device, dtype=torch.int32) + sp.rank * s).repeat(b)
        elif cu_seqlens is None:
            pos = torch.arange(s, device=ids.device, dtype=torch.int32).repeat(b)
        else:
            docs = attn_ops.doc_bounds(cu_seqlens.to(ids.device), b * s, s)
            pos = (torch.arange(s, device=ids.device, dtype=torch.int32).repeat(b) - docs[0]).to(torch.int32)
        branch = None
        for layer in self.layers:
            if self.gradient_checkpointing and self.training:
                x, branch = torch.utils.checkpoint.checkpoint(layer.forward_fused, x, branch, pos, s, docs,
                                                              use_reentrant=False)
            else:
                x, branch = layer.forward_fused(x, branch, pos, s, docs)
        return self.norm.add_norm(x, branch)[1]

    def set_sequence_parallel(self, sp) -> None:
        """Run attention with Ulysses sequence parallelism over ``sp`` (a parallel.ulysses.UlyssesGroup)."""
        self.sp = sp
        for layer in self.layers:
            layer.self_attn.sp = sp

    def forward(self, input_ids: torch.Tensor, labels: torch.Tensor | None = None, loss_denom=None,
                cu_seqlens: torch.Tensor | None = None, shifted_labels: torch.Tensor | None = None):
        """Returns (loss, aux_loss) with labels, else logits [B, S, V].  With ``cu_seqlens`` the last
        token of a document predicts nothing (no loss across document boundaries).  ``shifted_labels``
        (the next-token targets, already shifted) replace ``labels`` -- sequence-parallel ranks pass
        their chunk of the targets of the whole sequence."""
        h = self.hidden_states(input_ids, cu_seqlens)
        w = self.embed_tokens if self.lm_head is None else self.lm_head
        if labels is None and shifted_labels is None:
            logits = mp_ops.linear(h, w)
            return logits.reshape(*input_ids.shape, -1)
        if shifted_labels is not None:
            loss = loss_ops.fused_linear_cross_entropy(h, w, shifted_labels, denom=loss_denom)
            aux = None
            for blk in self.moe_blocks():
                if blk.last_aux_loss is not None:
                    aux = blk.last_aux_loss if aux is None else aux + blk.last_aux_loss
            return loss, aux
        shifted = torch.full_like(labels, loss_ops.IGNORE_INDEX)
        shifted[:, :-1] = labels[:, 1:]
        if cu_seqlens is not None:
            ends = cu_seqlens.to(labels.device).long()[1:] - 1  # last token of every document
            flat = shifted.view(-1)
            flat[ends] = loss_ops.IGNORE_INDEX
        if loss_denom is None:  # targets counted on the host: no device read in the middle of the step
            b, s = labels.shape
            loss_denom = max(b * s - (cu_seqlens.numel() - 1 if cu_seqlens is not None else b), 1)
        loss = loss_ops.fused_linear_cross_entropy(h, w, shifted, denom=loss_denom)
        aux = None
        for blk in self.moe_blocks():
            if blk.last_aux_loss is not None:
                aux = blk.last_aux_loss if aux is None else aux + blk.last_aux_loss
        return loss, aux


def build_model(cfg: MoEModelConfig, num_local_slots: int | None = None, device="cpu", seed: int = 0,
                expert_init=None) -> MoEForCausalLM:
    """Construct directly on ``device`` (no CPU staging of multi-GB weights) and initialise."""
    with torch.device(device):
        model = MoEForCausalLM(cfg, num_local_slots)
    model.to(device)  # buffers built from host data (router bias) follow the parameters
    model.init_weights(seed, expert_init)
    return model


def param_count(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())


def flops_per_token(cfg: MoEModelConfig, seq_len: int) -> float:
    return cfg.flops_per_token(seq_len)


__all__ = ["MoEForCausalLM", "DecoderLayer", "MoEBlock", "Attention", "RMSNorm", "build_model", "param_count",
           "flops_per_token", "math"]
