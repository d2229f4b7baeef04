"""TextTrainer: argument-driven wrapper around :class:`Trainer` for ``tasks/train_text.py``.

Maps the YAML/CLI arguments onto a TrainConfig, resolves the PlaceMoE runtime
configuration from ``VEOMNI_PLACEMOE_CONFIG`` (initial artifact loaded at
startup, hot-update controller attached when enabled), captures routes for
the planner when asked, logs, and checkpoints.

Reference parity: veomni/trainer/text_trainer.py:35 and the train loop of
veomni/trainer/base.py:820-863.
"""

from __future__ import annotations

import os
import time

import torch
import torch.distributed as dist

from ..arguments.parser import Arguments, save_args
from ..data.synthetic import SyntheticTokens
from ..models.config import from_hf_config, get_preset
from ..placemoe.runtime.config import PlaceMoERuntimeConfig
from .base import TrainConfig, Trainer


class TextTrainer:
    def __init__(self, args: Arguments):
        self.args = args
        t = args.train
        world = int(os.environ.get("WORLD_SIZE", "1"))
        per_rank = max(1, t.global_batch_size // world)
        mcfg = (from_hf_config(args.model.config_path) if args.model.config_path else get_preset(args.model.preset))
        if args.model.overrides:
            mcfg = mcfg.with_(**args.model.overrides)
        self.placemoe = PlaceMoERuntimeConfig.from_environment()
        from ..parallel.hiermoe_state import configure_hiermoe

        # fail fast on invalid MoE-parallel settings, before any model is built
        self.hiermoe = configure_hiermoe(t.hiermoe, ep_size=world, ranks_per_node=int(os.environ.get(
            "LOCAL_WORLD_SIZE", str(world))), activation_checkpointing_enabled=t.gradient_checkpointing,
            has_artifact=bool(self.placemoe.initial_artifact))
        cfg = TrainConfig(
            model=args.model.preset, seq_len=args.data.max_seq_len, batch_per_rank=per_rank,
            micro_batch_size=min(t.micro_batch_size, per_rank), lr=t.lr, betas=tuple(t.betas), eps=t.eps,
            weight_decay=t.weight_decay, max_grad_norm=t.max_grad_norm, optimizer=t.optimizer,
            lr_scheduler=t.lr_decay_style, min_lr_ratio=t.lr_min_ratio, muon_lr=t.muon_lr,
            muon_momentum=t.muon_momentum,
            warmup_steps=int(t.lr_warmup_ratio * t.max_steps), total_steps=t.max_steps, seed=t.seed,
            redundant_slots_per_rank=t.hiermoe.redundant_slot_increment_per_device,
            placemoe_artifact=self.placemoe.initial_artifact, capture_routes=t.hiermoe.capture_routes,
            gradient_checkpointing=t.gradient_checkpointing,
            device="cuda" if torch.cuda.is_available() else "cpu", log_interval=t.log_interval,
            output_dir=t.output_dir, save_steps=t.save_steps, ep_transport=t.hiermoe.transport,
        )
        self.trainer = Trainer(cfg, mcfg)
        self.data = SyntheticTokens(mcfg.vocab_size, per_rank, args.data.max_seq_len, seed=args.data.seed,
                                    rank=self.trainer.rank)
        from ..placemoe.oracle import OracleCapture

        self.oracle = OracleCapture(self.trainer.model)  # planner inputs on request (environment)
        self.recorder = None
        if t.hiermoe.capture_routes or t.hiermoe.route_capture_steps:
            from ..parallel.route_capture import RouteRecorder

            root = t.hiermoe.route_root or os.path.join(t.output_dir, "routes")
            self.recorder = RouteRecorder(self.trainer.model, root)
        if self.placemoe.hot_update.enabled:
            from ..parallel.hot_update import HotUpdateManager

            self.trainer.hot_update = HotUpdateManager(self.trainer, self.placemoe)
        if t.load_checkpoint_path:
            from ..checkpoint import load_checkpoint

            load_checkpoint(self.trainer, t.load_checkpoint_path)
        if self.trainer.rank == 0:
            save_args(args, t.output_dir)
        from .callbacks import CallbackList, EnvironmentMeterCallback, RouterMonitorCallback

        world = self.trainer.world
        self.callbacks = CallbackList([
            RouterMonitorCallback(t.log_interval),
            EnvironmentMeterCallback(per_rank * args.data.max_seq_len * world,
                                     mcfg.flops_per_token(args.data.max_seq_len), t.log_interval,
                                     os.path.join(t.output_dir, "metrics.jsonl")),
        ])

    def train(self):
        t = self.args.train
        tr = self.trainer
        t0 = time.perf_counter()
        self.callbacks.on_train_begin(tr)
        for step in range(tr.global_step, t.max_steps):
            if self.recorder is not None:
                self.recorder.enabled = step < max(t.hiermoe.route_capture_steps, 0) or t.hiermoe.capture_routes
            self.oracle.before_step(step)
            loss = tr.train_step(next(self.data))
            if self.recorder is not None and self.recorder.enabled:
                self.recorder.record_step(step)
            self.oracle.after_step(step)
            if tr.rank == 0 and (step % max(1, t.log_interval) == 0 or step == t.max_steps - 1):
                gn = tr.metrics.get("grad_norm")
                gn = float(gn) if gn is not None else float("nan")
                print(f"step {step + 1}/{t.max_steps} loss {loss:.4f} grad_norm {gn:.3f} "
                      f"lr {tr.lr_at(step):.3e} elapsed {time.perf_counter() - t0:.1f}s", flush=True)
            if t.save_steps and (step + 1) % t.save_steps == 0:
                from ..checkpoint import save_checkpoint

                save_checkpoint(tr, os.path.join(t.output_dir, "checkpoints"))
            self.callbacks.on_step_end(tr, step, loss)
        self.callbacks.on_train_end(tr)
        if dist.is_initialized():
            dist.barrier()
        return tr
