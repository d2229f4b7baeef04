"""Single-backend op table: every hot op and the sm_100a kernel that implements it.

One implementation per op (no multi-backend dispatch on hot paths).
``resolve`` checks the device's compute capability and that the compiled
extension exports the entry point, and fails loudly otherwise; ``table``
lists the bindings for documentation and tests.

Reference parity: veomni/ops/kernel_registry.py:36-172 (KernelSpec, resolve
with hardware requirements) and ops/config/registry.py (per-model binding).
"""

from __future__ import annotations

import dataclasses


@dataclasses.dataclass(frozen=True)
class KernelSpec:
    op: str  # logical op name
    entry: str  # extension entry point
    min_cc: tuple[int, int] = (10, 0)
    note: str = ""


_TABLE = [
    KernelSpec("linear", "dense_gemm", note="tcgen05 GEMM, CTA pairs, TMA-store epilogue"),
    KernelSpec("moe_experts_fc1", "moe_fc1_swiglu", note="grouped GEMM + SwiGLU + routing scale"),
    KernelSpec("moe_experts_fc2", "moe_grouped_gemm"),
    KernelSpec("moe_experts_dgrad", "moe_fc2_dgrad_dswiglu"),
    KernelSpec("moe_experts_wgrad", "moe_wgrad", note="fp32 TMA reduce-add into main_grad"),
    KernelSpec("router", "router_topk_fwd", note="softmax + top-k (+ bias), counts"),
    KernelSpec("moe_dispatch_plan", "moe_plan"),
    KernelSpec("attention", "attn_fwd", note="causal GQA flash attention, tcgen05"),
    KernelSpec("attention_backward", "attn_bwd"),
    KernelSpec("rms_norm", "rmsnorm_fwd"),
    KernelSpec("qk_norm_rope", "qkv_rope_fwd"),
    KernelSpec("cross_entropy", "ce_fwd_bwd"),
    KernelSpec("adamw", "adamw_step"),
    KernelSpec("ep_dispatch", "p2p_put_rows", note="peer-memory stores over NVLink"),
    KernelSpec("replica_grad_reduce", "p2p_sum_f32"),
    KernelSpec("state_migration", "p2p_pull"),
]


def table() -> list[KernelSpec]:
    return list(_TABLE)


def resolve(op: str):
    """The extension function implementing ``op`` on the current GPU (raises if unavailable)."""
    import torch

    from ._ext import kernels

    spec = next((s for s in _TABLE if s.op == op), None)
    if spec is None:
        raise KeyError(f"unknown op {op!r}")
    if not torch.cuda.is_available():
        raise RuntimeError(f"{op}: needs a CUDA device with compute capability >= {spec.min_cc}")
    cc = torch.cuda.get_device_capability()
    if cc < spec.min_cc:
        raise RuntimeError(f"{op}: compute capability {cc} < required {spec.min_cc}")
    fn = getattr(kernels(), spec.entry, None)
    if fn is None:
        raise RuntimeError(f"{op}: the kernel extension does not export {spec.entry}")
    return fn
