"""Model configurations for the Qwen3-MoE / OLMoE decoder families and the dense
Qwen3 / Llama families.

The presets carry the shapes named by the benchmark configurations:

* ``tiny_qwen3_moe``  4 layers, hidden 256, 8q/2kv heads x 32, 16 experts top-4,
  moe_intermediate 128, vocab 1024 (CPU/gloo plumbing run);
* ``olmoe_1b_7b``     16 layers, hidden 2048, 16 MHA heads x 128, 64 experts
  top-8, moe_intermediate 1024, vocab 50304;
* ``qwen3_30b_a3b``   48 layers, hidden 2048, 32q/4kv heads x 128, QK-norm,
  128 experts top-8, moe_intermediate 768, vocab 151936.

Dense presets (``num_experts == 0``, SwiGLU MLP of ``intermediate_size``):
``tiny_qwen3_dense``, ``qwen3_8b``, ``llama3_8b``.

``from_hf_config`` maps a HuggingFace ``config.json`` (model_type
``qwen3_moe`` / ``olmoe`` / ``qwen3`` / ``llama``) onto the same dataclass.

Reference parity: model configs under veomni/models/transformers/qwen3_moe and
tests/toy_config/qwen3_moe_toy/config.json.
"""

from __future__ import annotations

import json
import math
import os
from dataclasses import asdict, dataclass, field, replace

import numpy as np


@dataclass
class MoEModelConfig:
    model_type: str = "qwen3_moe"
    vocab_size: int = 151936
    hidden_size: int = 2048
    num_hidden_layers: int = 48
    num_attention_heads: int = 32
    num_key_value_heads: int = 4
    head_dim: int = 128
    moe_intermediate_size: int = 768
    intermediate_size: int = 0  # dense SwiGLU MLP width (dense families: num_experts == 0)
    num_experts: int = 128
    num_experts_per_tok: int = 8
    norm_topk_prob: bool = True
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    # "per_head": RMSNorm over head_dim (Qwen3); "full": over the whole projection (OLMoE); "none"
    qk_norm: str = "per_head"
    router_aux_loss_coef: float = 0.001
    tie_word_embeddings: bool = False
    initializer_range: float = 0.02
    # synthetic routing skew: per-expert fixed bias added to the router logits
    router_bias_zipf_s: float = 0.0
    router_bias_scale: float = 1.0
    router_bias_seed_per_layer: bool = False
    extra: dict = field(default_factory=dict)

    @property
    def is_dense(self) -> bool:
        """Dense decoder (Llama / Qwen3 dense): a SwiGLU MLP in every layer instead of experts."""
        return self.num_experts == 0

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def to_dict(self) -> dict:
        return asdict(self)

    def with_(self, **kw) -> "MoEModelConfig":
        return replace(self, **kw)

    def num_params(self) -> int:
        h, i, e = self.hidden_size, self.moe_intermediate_size, self.num_experts
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        norms = 2 * h + (self.q_size + self.kv_size if self.qk_norm == "full" else 2 * self.head_dim if self.qk_norm == "per_head" else 0)
        layer = attn + norms + (3 * h * self.intermediate_size if self.is_dense else e * h + e * 3 * h * i)
        emb = self.vocab_size * h * (1 if self.tie_word_embeddings else 2)
        return self.num_hidden_layers * layer + emb + h

    def flops_per_token(self, seq_len: int) -> float:
        """Training FLOPs per token (forward + backward = 3x forward), causal attention."""
        h, i, k = self.hidden_size, self.moe_intermediate_size, self.num_experts_per_tok
        proj = 2 * h * (self.q_size + 2 * self.kv_size) + 2 * self.q_size * h
        router = 2 * h * self.num_experts
        experts = 2 * 3 * h * self.intermediate_size if self.is_dense else k * 2 * 3 * h * i
        attn = 2 * 2 * self.q_size * (seq_len / 2)  # QK^T and PV, causal average
        per_layer = proj + router + experts + attn
        head = 2 * h * self.vocab_size
        return 3.0 * (self.num_hidden_layers * per_layer + head)


def zipf_router_bias(num_experts: int, s: float, scale: float = 1.0, seed: int = 0) -> np.ndarray:
    """scale * log of Zipf(s) weights over a seeded permutation of the experts (s = 0 -> zeros)."""
    if s == 0:
        return np.zeros(num_experts, dtype=np.float32)
    ranks = np.arange(1, num_experts + 1, dtype=np.float64)
    w = ranks ** (-s)
    w /= w.sum()
    perm = np.random.default_rng(seed).permutation(num_experts)
    bias = np.empty(num_experts, dtype=np.float64)
    bias[perm] = scale * np.log(w)
    return bias.astype(np.float32)


PRESETS: dict[str, MoEModelConfig] = {
    "tiny_qwen3_moe": MoEModelConfig(
        model_type="qwen3_moe",
        vocab_size=1024,
        hidden_size=256,
        num_hidden_layers=4,
        num_attention_heads=8,
        num_key_value_heads=2,
        head_dim=32,
        moe_intermediate_size=128,
        num_experts=16,
        num_experts_per_tok=4,
        norm_topk_prob=True,
        rope_theta=1_000_000.0,
        rms_norm_eps=1e-6,
        qk_norm="per_head",
        router_bias_zipf_s=1.1,
        router_bias_scale=0.5,
    ),
    # small GPU-kernel-compatible shapes (head_dim 128, hidden % 256 == 0) for tests and smoke runs
    "small_qwen3_moe": MoEModelConfig(
        model_type="qwen3_moe", vocab_size=4096, hidden_size=1024, num_hidden_layers=2, num_attention_heads=8,
        num_key_value_heads=2, head_dim=128, moe_intermediate_size=512, num_experts=16, num_experts_per_tok=4,
        norm_topk_prob=True, rope_theta=1_000_000.0, rms_norm_eps=1e-6, qk_norm="per_head",
        router_bias_zipf_s=1.0, router_bias_scale=0.5,
    ),
    "small_olmoe": MoEModelConfig(
        model_type="olmoe", vocab_size=4096, hidden_size=1024, num_hidden_layers=2, num_attention_heads=8,
        num_key_value_heads=8, head_dim=128, moe_intermediate_size=512, num_experts=16, num_experts_per_tok=4,
        norm_topk_prob=False, rope_theta=10_000.0, rms_norm_eps=1e-5, qk_norm="full", router_aux_loss_coef=0.01,
        router_bias_zipf_s=1.0, router_bias_scale=0.5, router_bias_seed_per_layer=True,
    ),
    "olmoe_1b_7b": MoEModelConfig(
        model_type="olmoe",
        vocab_size=50304,
        hidden_size=2048,
        num_hidden_layers=16,
        num_attention_heads=16,
        num_key_value_heads=16,
        head_dim=128,
        moe_intermediate_size=1024,
        num_experts=64,
        num_experts_per_tok=8,
        norm_topk_prob=False,
        rope_theta=10_000.0,
        rms_norm_eps=1e-5,
        qk_norm="full",
        router_aux_loss_coef=0.01,
        router_bias_zipf_s=1.0,
        router_bias_scale=0.5,
        router_bias_seed_per_layer=True,
    ),
    "qwen3_30b_a3b": MoEModelConfig(
        model_type="qwen3_moe",
        vocab_size=151936,
        hidden_size=2048,
        num_hidden_layers=48,
        num_attention_heads=32,
        num_key_value_heads=4,
        head_dim=128,
        moe_intermediate_size=768,
        num_experts=128,
        num_experts_per_tok=8,
        norm_topk_prob=True,
        rope_theta=1_000_000.0,
        rms_norm_eps=1e-6,
        qk_norm="per_head",
        router_aux_loss_coef=0.001,
        router_bias_zipf_s=1.0,
        router_bias_scale=1.0,
    ),
}


# dense decoder families (same attention; SwiGLU MLP instead of experts)
PRESETS.update({
    "tiny_qwen3_dense": MoEModelConfig(
        model_type="qwen3", vocab_size=1024, hidden_size=256, num_hidden_layers=2, num_attention_heads=8,
        num_key_value_heads=2, head_dim=32, intermediate_size=512, num_experts=0, num_experts_per_tok=0,
        router_aux_loss_coef=0.0),
    "qwen3_8b": MoEModelConfig(
        model_type="qwen3", vocab_size=151936, hidden_size=4096, num_hidden_layers=36, num_attention_heads=32,
        num_key_value_heads=8, head_dim=128, intermediate_size=12288, num_experts=0, num_experts_per_tok=0,
        router_aux_loss_coef=0.0),
    "llama3_8b": MoEModelConfig(
        model_type="llama", vocab_size=128256, hidden_size=4096, num_hidden_layers=32, num_attention_heads=32,
        num_key_value_heads=8, head_dim=128, intermediate_size=14336, num_experts=0, num_experts_per_tok=0,
        rope_theta=500000.0, rms_norm_eps=1e-5, qk_norm="none", router_aux_loss_coef=0.0),
})


def get_preset(name: str, **overrides) -> MoEModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; available: {sorted(PRESETS)}")
    return PRESETS[name].with_(**overrides)


def from_hf_config(path_or_dict) -> MoEModelConfig:
    """Build a config from a HuggingFace config.json (qwen3_moe / olmoe)."""
    if isinstance(path_or_dict, (str, os.PathLike)):
        p = os.path.join(path_or_dict, "config.json") if os.path.isdir(path_or_dict) else path_or_dict
        with open(p) as f:
            d = json.load(f)
    else:
        d = dict(path_or_dict)
    mt = d.get("model_type", "qwen3_moe")
    heads = d["num_attention_heads"]
    hd = d.get("head_dim") or d["hidden_size"] // heads
    if mt in ("qwen3", "llama"):
        return MoEModelConfig(
            model_type=mt, vocab_size=d["vocab_size"], hidden_size=d["hidden_size"],
            num_hidden_layers=d["num_hidden_layers"], num_attention_heads=heads,
            num_key_value_heads=d.get("num_key_value_heads", heads), head_dim=hd,
            intermediate_size=d["intermediate_size"], num_experts=0, num_experts_per_tok=0,
            rope_theta=float(d.get("rope_theta", 10000.0)), rms_norm_eps=float(d.get("rms_norm_eps", 1e-6)),
            qk_norm="per_head" if mt == "qwen3" else "none", router_aux_loss_coef=0.0,
            tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
            initializer_range=float(d.get("initializer_range", 0.02)))
    if mt in ("qwen3_moe", "qwen3_vl_moe_text"):
        qk = "per_head"
    elif mt == "olmoe":
        qk = "full"
    else:
        raise ValueError(f"unsupported model_type {mt!r}")
    return MoEModelConfig(
        model_type="olmoe" if mt == "olmoe" else "qwen3_moe",
        vocab_size=d["vocab_size"],
        hidden_size=d["hidden_size"],
        num_hidden_layers=d["num_hidden_layers"],
        num_attention_heads=heads,
        num_key_value_heads=d.get("num_key_value_heads", heads),
        head_dim=hd,
        moe_intermediate_size=d.get("moe_intermediate_size", d.get("intermediate_size")),
        num_experts=d.get("num_experts", d.get("num_local_experts")),
        num_experts_per_tok=d["num_experts_per_tok"],
        norm_topk_prob=bool(d.get("norm_topk_prob", mt != "olmoe")),
        rope_theta=float(d.get("rope_theta", 10000.0)),
        rms_norm_eps=float(d.get("rms_norm_eps", 1e-6)),
        qk_norm=qk,
        router_aux_loss_coef=float(d.get("router_aux_loss_coef", 0.001)),
        tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
        initializer_range=float(d.get("initializer_range", 0.02)),
    )


def log2_ceil(x: int) -> int:
    return int(math.ceil(math.log2(max(x, 1))))
