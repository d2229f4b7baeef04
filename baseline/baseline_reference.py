"""Reference arm of bench.py: the unmodified reference (installed in baseline/_ref) on the same metric.

Drives the reference through its public API and stock code path, in the
order its BaseTrainer uses: ``init_parallel_state`` (FSDP2 data parallel +
expert parallel = world size), ``configure_hiermoe`` (its defaults: HierMoE off; with
``--ref-hiermoe dedup`` at N > 1 its token-deduplicated dispatch/combine on, direct all-to-all,
expert swap off),
``build_foundation_model`` (meta init) -> ``build_parallelize_model`` (FSDP2,
mixed precision, gradient checkpointing as in its trainer default) ->
``build_optimizer`` (fused AdamW) and, per step, forward/backward of every
micro-batch, ``veomni_clip_grad_norm`` and ``optimizer.step``.

Model: the reference has no expert-parallel OLMoE implementation, so its
Qwen3-MoE implementation is configured at the OLMoE-1B-7B shape (16 layers,
hidden 2048, 16 MHA heads x 128, 64 experts top-8, moe_intermediate 1024,
vocab 50304), or at the Qwen3-30B-A3B shape (``--model qwen3_30b_a3b``: 48
layers, 32 q / 4 kv heads, 128 experts top-8, moe_intermediate 768, vocab
151936); MoE kernels ``fused_triton`` (its default), attention through
PyTorch SDPA, other ops eager (liger_kernel is not installed here).  The
reference exposes no router-bias hook, so its routing is not skewed.

On one GPU the reference's parallelizer skips FSDP, which is where its
mixed-precision policy lives: with the policy switched on it only upcasts the
model to fp32, which its fused MoE kernels reject.  The one-GPU arm therefore
builds the model in bf16 with the policy off (bf16 parameters and AdamW
states) and initialises on cuda (meta init is rejected without FSDP).

Timing and output follow bench.py: W warm-up steps, K device-timed steps
(CUDA events, max over ranks), then K end-to-end steps with pinned-host
inputs and a loss read per step.
"""

from __future__ import annotations

import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def _unavailable(reason: str) -> int:
    print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)
    return 0


# The two benchmark shapes, as Qwen3-MoE configurations of the reference's own model implementation.
SHAPES = {
    "olmoe_1b_7b": dict(vocab=50304, hidden=2048, layers=16, heads=16, kv=16, hd=128, experts=64, k=8, inter=1024,
                        norm_topk=False, theta=10000.0, eps=1e-5, aux=0.01),
    "qwen3_30b_a3b": dict(vocab=151936, hidden=2048, layers=48, heads=32, kv=4, hd=128, experts=128, k=8,
                          inter=768, norm_topk=True, theta=1000000.0, eps=1e-6, aux=0.001),
}


def _config_dir(vocab, hidden, layers, heads, kv, hd, experts, k, inter, norm_topk, theta, eps, aux):
    d = tempfile.mkdtemp(prefix="ref_moe_shape_")
    cfg = {
        "architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe", "vocab_size": vocab,
        "hidden_size": hidden, "intermediate_size": inter, "moe_intermediate_size": inter,
        "num_hidden_layers": layers, "num_attention_heads": heads, "num_key_value_heads": kv, "head_dim": hd,
        "num_experts": experts, "num_experts_per_tok": k, "norm_topk_prob": norm_topk, "decoder_sparse_step": 1,
        "mlp_only_layers": [], "rope_theta": theta, "rms_norm_eps": eps, "max_position_embeddings": 4096,
        "tie_word_embeddings": False, "router_aux_loss_coef": aux, "output_router_logits": True,
        "attention_bias": False, "attention_dropout": 0.0, "hidden_act": "silu", "initializer_range": 0.02,
        "torch_dtype": "bfloat16", "use_cache": False,
    }
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    return d


def main(args) -> int:
    if not os.path.isdir(os.path.join(REF, "veomni")):
        return _unavailable("reference not installed in baseline/_ref")
    if args.model not in SHAPES:
        return _unavailable(f"reference arm is defined for {sorted(SHAPES)} (got {args.model})")
    shape = SHAPES[args.model]
    # the reference trainer's default is activation recomputation on; --ref-no-recompute measures it off
    ckpt = not getattr(args, "ref_no_recompute", False)
    sys.path.insert(0, REF)
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if not dist.is_initialized():
        if world == 1:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", str(29600 + os.getpid() % 1000))
            os.environ.setdefault("RANK", "0")
            os.environ.setdefault("WORLD_SIZE", "1")
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600))
    try:
        from veomni.arguments.arguments_types import HierMoEConfig, MixedPrecisionConfig, OpsImplementationConfig
        from veomni.distributed.clip_grad_norm import veomni_clip_grad_norm
        from veomni.distributed.moe.hiermoe.state import configure_hiermoe
        from veomni.distributed.parallel_state import get_parallel_state, init_parallel_state
        from veomni.distributed.torch_parallelize import build_parallelize_model
        from veomni.models import build_foundation_model
        from veomni.optim import build_optimizer
    except Exception as e:  # missing optional deps etc.
        return _unavailable(f"reference import failed: {type(e).__name__}: {e}")

    init_parallel_state(dp_size=world, dp_shard_size=world, extra_parallel_sizes=(world,),
                        extra_parallel_names=("ep",), dp_mode="fsdp2")
    ps = get_parallel_state()
    hier = getattr(args, "ref_hiermoe", "off") == "dedup" and world > 1
    hcfg = (HierMoEConfig(enable=True, token_dedup=True, communication_mode="direct", expert_swap=False)
            if hier else HierMoEConfig())
    configure_hiermoe(hcfg, ep_group=ps.ep_group if getattr(ps, "ep_enabled", False) else None,
                      ep_fsdp_size=ps.ep_fsdp_size if getattr(ps, "ep_enabled", False) else 1,
                      activation_checkpointing_enabled=ckpt, fsdp_offload_enabled=False,
                      gradient_bytes_per_element=4)
    ops = OpsImplementationConfig(attn_implementation="sdpa", moe_implementation="fused_triton",
                                  cross_entropy_loss_implementation="eager", rms_norm_implementation="eager",
                                  swiglu_mlp_implementation="eager", rotary_pos_emb_implementation="eager")
    cfg_dir = _config_dir(**shape)
    # its parallelizer accepts meta init only when FSDP is on (world size > 1)
    init_device = "meta" if world > 1 else "cuda"
    # Without FSDP its mixed-precision switch only upcasts the model to fp32, which its fused
    # MoE kernels reject (bf16/fp16 only); on one GPU the model is therefore built in bf16 with
    # the switch off (bf16 parameters and optimizer states).
    mp_on = world > 1
    model = build_foundation_model(config_path=cfg_dir, weights_path=None,
                                   torch_dtype="float32" if mp_on else "bfloat16",
                                   init_device=init_device, ops_implementation=ops)
    model = build_parallelize_model(model, init_device=init_device, weights_path=None, enable_reshard_after_forward=True,
                                    mixed_precision=MixedPrecisionConfig(enable=mp_on),
                                    enable_gradient_checkpointing=ckpt,
                                    basic_modules=list(getattr(model, "_no_split_modules", None) or []),
                                    enable_forward_prefetch=True)
    model.train()
    opt = build_optimizer(model, lr=3e-4, weight_decay=0.1, fused=True)

    seq, bpg, mb = args.seq, args.batch_per_gpu, args.micro_batch
    g = torch.Generator().manual_seed(rank)
    pool = [torch.randint(0, shape["vocab"], (bpg, seq), generator=g).pin_memory() for _ in range(2)]
    dev = [p.cuda() for p in pool]

    def step(ids, read_loss):
        losses = []
        for i in range(0, bpg, mb):
            x = ids[i:i + mb].cuda(non_blocking=True)
            out = model(input_ids=x, labels=x, use_cache=False)
            loss = out.loss
            (loss / max(1, bpg // mb)).backward()
            losses.append(loss.detach())
        veomni_clip_grad_norm(model, 1.0)
        opt.step()
        opt.zero_grad()
        loss = torch.stack(losses).mean()
        return float(loss.item()) if read_loss else loss

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(pool[0], True)
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        step(dev[i % 2], False)
    e.record()
    barrier()
    ms = s.elapsed_time(e) / args.steps
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    last = None
    for i in range(args.steps):
        last = step(pool[i % 2], True)
    e2.record()
    barrier()
    ms_e2e = s2.elapsed_time(e2) / args.steps
    t = torch.tensor([ms, ms_e2e], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e = t.tolist()
    tokens = bpg * seq * world
    if rank == 0:
        print(json.dumps({
            "impl": "reference", "metric": "MoE train tokens/s", "value": round(tokens / (ms / 1e3), 1),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic uniform token ids (seeded), random-init weights",
            "config": {"model": (f"reference Qwen3-MoE implementation at the {args.model} shape "
                                 f"({shape['layers']}L, H{shape['hidden']}, {shape['heads']}q/{shape['kv']}kv heads, "
                                 f"{shape['experts']}E top{shape['k']}, I{shape['inter']}, V{shape['vocab']}); "
                                 "no router bias"), "global_batch": bpg * world, "seq_len": seq,
                       "precision": "fsdp2 mixed precision (fp32 masters, bf16 compute)" if mp_on
                       else "bf16 parameters and optimizer states (no FSDP on one GPU)",
                       "micro_batch": mb, "parallelism": f"fsdp{world}+ep{world}",
                       "ops": "moe fused_triton, attention sdpa, gradient checkpointing "
                              + ("on (its trainer default)" if ckpt else "off"),
                       "hiermoe": ("token-deduplicated dispatch/combine (direct all-to-all, no expert swap)"
                                   if hier else "off (its trainer default)")},
            "e2e": {"value": round(tokens / (ms_e2e / 1e3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": pool[0].numel() * 8, "d2h_bytes_per_step": 4, "last_loss": last},
        }), flush=True)
    if world > 1:
        dist.barrier()
    dist.destroy_process_group()
    return 0


