"""Trainer: setup -> build model -> parallelize -> optimizer -> train steps.

Step structure (same order as the reference's BaseTrainer.train_step):

    for each micro-batch: forward (loss / world + aux) -> backward
    replica-gradient sync (copies of one expert summed)
    dense gradient reduction (one bucket, one collective)
    global grad norm (each logical expert counted once) -> clip coefficient on device
    fused AdamW (clip applied in-kernel, bf16 compute copies rewritten)
    zero grads -> placement hot update at the step boundary (if configured)

Everything between the input copy and the loss read stays on the device: the
clip coefficient is a device scalar fed to the optimizer kernel, MoE dispatch
plans are built by kernels (single GPU), so a step has exactly one host
synchronisation, the loss read.

Reference parity: veomni/trainer/base.py:239-331 (_setup), :452-535, :695-727
(forward_backward_step), :755-811 (train_step), :820-863 (train).
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from ..models.config import MoEModelConfig, get_preset
from ..models.moe_decoder import build_model
from ..ops import check_device_error
from ..ops import moe as moe_ops
from ..ops import mp as mp_ops
from ..optim import build_lr_scheduler, build_optimizer
from ..parallel.p2p_ep import EPCapacityExceeded
from ..parallel.data_parallel import (expert_init_from_full, expert_topology, parallelize_model,
                                      redundant_slot_weights, sync_replica_gradients)
from ..placemoe.artifacts import load_artifact


@dataclass
class TrainConfig:
    model: str = "olmoe_1b_7b"
    model_overrides: dict = field(default_factory=dict)
    seq_len: int = 4096
    batch_per_rank: int = 8  # sequences per rank per step
    micro_batch_size: int = 2  # sequences per micro-batch
    lr: float = 3e-4
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    weight_decay: float = 0.1
    max_grad_norm: float = 1.0
    warmup_steps: int = 0
    total_steps: int = 100
    optimizer: str = "adamw"  # "adamw" | "muon" (Muon for hidden matrices, AdamW for the rest)
    lr_scheduler: str = "cosine"  # "constant" | "linear" | "cosine" after linear warmup
    min_lr_ratio: float = 0.1
    muon_lr: float = 0.02
    muon_momentum: float = 0.95
    # "auto": shard dense masters / moments / reduced gradients over the ranks (peer-memory
    # reduce-scatter + all-gather) when N > 1 on CUDA with AdamW; "on" / "off" force it
    dense_sharding: str = "auto"
    seed: int = 0
    redundant_slots_per_rank: int = 0
    placemoe_artifact: str = ""  # schema-v2 artifact loaded at startup
    capture_routes: bool = False
    ep_transport: str = "auto"
    recompute_expert_rows: bool = False  # drop dispatched expert inputs after forward, re-gather in backward  # "auto" | "p2p" | "nccl"
    ulysses_size: int = 1  # sequence-parallel ranks per group (consecutive ranks; they share one batch)
    gradient_checkpointing: bool = False
    activation_offload: bool = False  # saved activations to pinned host memory (utils/offload.py)
    device: str = "cuda"
    log_interval: int = 10
    output_dir: str = ""
    save_steps: int = 0


def init_distributed(backend: str | None = None, timeout_s: int = 600):
    """Initialise torch.distributed from the torchrun environment (no-op for a single process)."""
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1:
        return 0, 1
    from datetime import timedelta

    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    dist.init_process_group(backend=backend, timeout=timedelta(seconds=timeout_s))
    return dist.get_rank(), dist.get_world_size()


class Trainer:
    def __init__(self, cfg: TrainConfig, model_cfg: MoEModelConfig | None = None):
        self.cfg = cfg
        self.rank, self.world = init_distributed()
        if cfg.device == "cuda":
            self.device = torch.device("cuda", torch.cuda.current_device() if torch.cuda.is_available() else 0)
        else:
            self.device = torch.device(cfg.device)
        self.model_cfg = model_cfg or get_preset(cfg.model, **cfg.model_overrides)
        plans = None
        # dense families hold no experts: a placeholder topology of one slot per rank
        topology = expert_topology(self.model_cfg.num_experts or self.world, self.world,
                                   cfg.redundant_slots_per_rank)
        if cfg.placemoe_artifact:
            _, topology, plans = load_artifact(cfg.placemoe_artifact)
            if topology.ep_size != self.world or topology.num_experts != self.model_cfg.num_experts:
                raise ValueError("PlaceMoE artifact topology does not match the run")
        self.topology = topology
        init = expert_init_from_full(self.model_cfg, topology, plans, self.rank, cfg.seed)
        self.model = build_model(self.model_cfg, topology.slots_per_rank, self.device, cfg.seed, init)
        self.model.gradient_checkpointing = cfg.gradient_checkpointing
        for blk in self.model.moe_blocks():
            blk.keep_expert_rows = not cfg.recompute_expert_rows
        self.model.train()
        self.pstate = parallelize_model(self.model, plans=plans, topology=topology, device=self.device,
                                        capture_routes=cfg.capture_routes, transport=cfg.ep_transport)
        self.optimizer = build_optimizer(self.model, cfg.optimizer, lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                                         weight_decay=cfg.weight_decay, muon_lr=cfg.muon_lr,
                                         muon_momentum=cfg.muon_momentum)
        self.lr_schedule = build_lr_scheduler(cfg.lr_scheduler, cfg.lr, cfg.warmup_steps, cfg.total_steps,
                                              cfg.min_lr_ratio)
        # peer-memory exchange for replica gradients and migration (CUDA, peer-memory EP transport)
        self.peer_exchange = None
        self.replica_sync = None
        if self.world > 1 and self.device.type == "cuda" and hasattr(self.pstate.ep, "replica_sync"):
            from ..parallel.p2p_sync import PeerExchange, ReplicaGradSync

            nbytes = max(p.numel() * 4 for p in self.model.expert_parameters())
            self.peer_exchange = PeerExchange(None, self.device, nbytes)
            self.replica_sync = ReplicaGradSync(self.peer_exchange)
            self.pstate.ep.replica_sync = self.replica_sync
        self.sp = None
        if cfg.ulysses_size > 1:
            from ..parallel.ulysses import build_ulysses_groups

            mc = self.model_cfg
            if mc.num_key_value_heads % cfg.ulysses_size or mc.num_attention_heads % cfg.ulysses_size:
                raise ValueError("attention heads must split over the sequence-parallel ranks")
            if cfg.seq_len % cfg.ulysses_size:
                raise ValueError("seq_len must split over the sequence-parallel ranks")
            widest = cfg.micro_batch_size * cfg.seq_len // cfg.ulysses_size * mc.q_size
            self.sp = build_ulysses_groups(cfg.ulysses_size, self.device, widest)
            self.model.set_sequence_parallel(self.sp)
        self.dense_shards = None
        if self._want_dense_sharding():
            self._setup_dense_shards()
        self._norm_table = None
        self.global_step = 0
        self.hot_update = None  # set by placement runtime (hot updates)
        self.metrics: dict = {}

    # ------------------------------------------------------------- sharding
    def _want_dense_sharding(self) -> bool:
        mode = self.cfg.dense_sharding
        if mode not in ("auto", "on", "off"):
            raise ValueError("dense_sharding must be 'auto', 'on' or 'off'")
        if mode == "on" and self.cfg.optimizer != "adamw":
            raise ValueError("dense sharding is built for AdamW (Muon needs whole matrices)")
        if mode == "off" or self.world == 1 or self.cfg.optimizer != "adamw":
            return False
        return mode == "on" or (self.device.type == "cuda" and self.replica_sync is not None)

    def _setup_dense_shards(self) -> None:
        """AdamW over shards of the dense matrices; small fp32-read parameters stay replicated."""
        from ..ops.optim import FusedAdamW
        from ..optim import MultiOptimizer
        from ..parallel.data_parallel import DenseGradBucket, is_expert_param
        from ..parallel.dense_shard import ShardedDenseAdamW, shardable

        cfg = self.cfg
        named = list(self.model.named_parameters())
        shard = [p for n, p in named if not is_expert_param(n) and shardable(n, p)]
        rep = [p for n, p in named if not is_expert_param(n) and not shardable(n, p)]
        experts = [p for n, p in named if is_expert_param(n)]
        self.dense_shards = ShardedDenseAdamW(shard, lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                                              weight_decay=cfg.weight_decay)
        if self.pstate.dense_bucket is not None:
            self.pstate.dense_bucket = DenseGradBucket(rep, self.device) if rep else None
        self.optimizer = MultiOptimizer({
            "experts": FusedAdamW(experts + rep, lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                                  weight_decay=cfg.weight_decay),
            "dense": self.dense_shards})

    # ------------------------------------------------------------------ utils
    def lr_at(self, step: int) -> float:
        return self.lr_schedule(step)

    def _grad_sq_norm(self) -> torch.Tensor:
        """Squared global grad norm (device scalar); redundant expert copies are excluded."""
        kn = mp_ops.kernels()
        if self._norm_table is None:
            grads, weights = [], []
            for blk in self.model.moe_blocks():
                w = redundant_slot_weights(blk, blk.placement)
                for p in (blk.gate_up_proj, blk.down_proj):
                    mg = mp_ops.main_grad(p)
                    for j in range(p.shape[0]):
                        grads.append(mg[j])
                        weights.append(w[j])
            if self.pstate.dense_bucket is not None:
                grads.append(self.pstate.dense_bucket.flat)
                weights.append(1.0)
            if self.dense_shards is not None:  # disjoint slices: each counted once over the ranks
                grads.append(self.dense_shards.grad_shard)
                weights.append(1.0)
            self._norm_table = kn.sq_norm_build_table(grads, weights)
        out = torch.zeros((), device=self.device, dtype=torch.float32)
        kn.sq_norm(self._norm_table[0], self._norm_table[1], out)
        if self.world > 1:
            # the replicated dense part is counted once per rank -> keep one copy
            dsq = self.pstate.dense_bucket.flat.float().pow(2).sum() if self.pstate.dense_bucket is not None else None
            if dsq is not None:
                out = out - dsq
            dist.all_reduce(out)
            if dsq is not None:
                out = out + dsq
        return out

    # ------------------------------------------------------------------- step
    def forward_backward(self, input_ids: torch.Tensor, cu_seqlens: torch.Tensor | None = None) -> torch.Tensor:
        from ..utils.offload import ActivationOffload

        with ActivationOffload(enabled=self.cfg.activation_offload and self.device.type == "cuda"):
            if self.sp is not None:
                # every rank of the SP group holds the same sequences: take this rank's chunk of the tokens and
                # of the next-token targets of the whole sequence; the loss divisor is the group's target
                # count over P, so the mean of the P chunk losses is the loss of the whole batch.  Packed rows:
                # the last token of every document predicts nothing, and attention (on whole sequences after
                # the exchange) stays inside each document.
                from ..ops.loss import IGNORE_INDEX

                b, s = input_ids.shape
                p, r = self.sp.size, self.sp.rank
                chunk = s // p
                targets = torch.full_like(input_ids, IGNORE_INDEX)
                targets[:, :-1] = input_ids[:, 1:]
                n_targets = b * (s - 1)
                if cu_seqlens is not None:
                    ends = cu_seqlens.to(targets.device).long()[1:] - 1
                    targets.view(-1)[ends] = IGNORE_INDEX
                    n_targets = b * s - (cu_seqlens.numel() - 1)
                sl = slice(r * chunk, (r + 1) * chunk)
                loss, aux = self.model(input_ids[:, sl].contiguous(), shifted_labels=targets[:, sl].contiguous(),
                                       loss_denom=n_targets / p, cu_seqlens=cu_seqlens)
            elif cu_seqlens is None:
                loss, aux = self.model(input_ids, labels=input_ids)
            else:
                loss, aux = self.model(input_ids, labels=input_ids, cu_seqlens=cu_seqlens)
        total = loss / self.world
        if aux is not None:
            total = total + aux / self.world
        total.backward()
        ep = self.pstate.ep if self.pstate is not None else None
        if hasattr(ep, "wait_wgrads"):
            # the last MoE layer's weight gradients may still read its receive slab, which the next
            # micro-batch's dispatch refills (peers store into it once this rank reaches that dispatch)
            ep.wait_wgrads()
        return loss.detach()

    def train_step(self, input_ids: torch.Tensor, *, read_loss: bool = True, cu_seqlens: torch.Tensor | None = None):
        """One optimizer step over ``input_ids`` [batch_per_rank, seq] (host or device tensor).

        ``cu_seqlens`` (packed rows): cumulative document boundaries over the flattened tokens;
        every row boundary is a document boundary (``data.pack_documents``).
        """
        cfg = self.cfg
        ids = input_ids.to(self.device, non_blocking=True)
        mb = max(1, cfg.micro_batch_size)
        n_micro = max(1, ids.shape[0] // mb)
        cus = [None] * n_micro
        if cu_seqlens is not None:  # split the document boundaries by micro-batch
            cu = cu_seqlens.to(torch.int64).cpu()
            seq = ids.shape[1]
            for i in range(n_micro):
                lo, hi = i * mb * seq, (i + 1) * mb * seq
                part = cu[(cu >= lo) & (cu <= hi)] - lo
                cus[i] = part.to(torch.int32).to(self.device)
        ep = self.pstate.ep
        rsync = self.replica_sync
        for attempt in range(4):
            losses = []
            for i in range(n_micro):
                if rsync is not None:  # replicas are reduced during the last micro-batch's backward
                    rsync.armed = i == n_micro - 1
                if cus[i] is None:
                    losses.append(self.forward_backward(ids[i * mb:(i + 1) * mb]))
                else:
                    losses.append(self.forward_backward(ids[i * mb:(i + 1) * mb], cus[i]))
            if rsync is not None:
                rsync.armed = False
            if not hasattr(ep, "check_capacity"):
                break
            try:
                ep.check_capacity()  # one host read per step: did any rank overflow its expert buffers?
                if self.device.type == "cuda":
                    # a peer wait that ran out (sticky status) or a kernel check: raise now, not
                    # after further steps on stale data
                    check_device_error()
                break
            except EPCapacityExceeded:
                if attempt == 3:
                    raise
                # recompute the step with larger expert buffers (gradients restart from zero)
                if rsync is not None:
                    rsync.wait()
                self._zero_all_grads()
                if hasattr(ep, "grow_capacity"):  # size for the rows the step needed (plus a margin)
                    ep.grow_capacity()
                else:
                    ep.capacity_factor = min(float(self.world), ep.capacity_factor * 2)
                self.metrics["ep_capacity_factor"] = ep.capacity_factor
        loss = torch.stack(losses).mean()
        self.optimizer_step()
        self.global_step += 1
        if self.hot_update is not None:
            self.hot_update.on_step_end(self)
        if not read_loss:
            return loss
        value = float(loss.item())
        if self.device.type == "cuda" and not hasattr(ep, "check_capacity"):
            check_device_error()  # the loss read already synchronised: one more small read
        return value

    def optimizer_step(self):
        cfg = self.cfg
        # gradients of micro-batches were accumulated; average them
        nmb = max(1, cfg.batch_per_rank // max(1, cfg.micro_batch_size))
        if self.replica_sync is not None:
            self.replica_sync.wait()  # replicas were reduced over peer memory during the backward
        moe_ops.settle_stale_grads(self.model.expert_parameters())
        if self.world > 1:
            if self.replica_sync is None:  # else reduced over peer memory during the backward
                sync_replica_gradients(self.model, self.pstate.placements)
            if self.pstate.dense_bucket is not None:
                self.pstate.dense_bucket.reduce()
            if self.dense_shards is not None and self.device.type == "cuda":
                self.dense_shards.reduce_scatter()
        if self.device.type == "cuda":
            sq = self._grad_sq_norm()
            norm = sq.sqrt() / nmb
            clip = torch.clamp(cfg.max_grad_norm / (norm + 1e-6), max=1.0) if cfg.max_grad_norm > 0 else \
                torch.ones((), device=self.device)
            self.optimizer.grad_scale = (clip / nmb).reshape(1).contiguous()
            self.metrics["grad_norm"] = norm
        else:
            from ..parallel.data_parallel import is_expert_param

            for p in self.model.parameters():
                if p.grad is not None:
                    p.grad.div_(nmb)
            sharded = set()
            dense_sq = torch.zeros((), dtype=torch.float64)
            if self.dense_shards is not None:
                # local gradients into the flat bucket, reduce-scatter, norm of the owned slices
                for p in self.dense_shards.params:
                    sharded.add(id(p))
                    if p.grad is not None:
                        p.main_grad.copy_(p.grad)
                    else:
                        p.main_grad.zero_()
                self.dense_shards.reduce_scatter()
                dense_sq = self.dense_shards.grad_shard.double().pow(2).sum()
                dist.all_reduce(dense_sq)
            if self.world > 1:
                for n, p in self.model.named_parameters():
                    if p.grad is not None and not is_expert_param(n) and id(p) not in sharded:
                        dist.all_reduce(p.grad)
            if cfg.max_grad_norm > 0:
                # global norm: dense once, each logical expert once (owner copies)
                dense_sq = dense_sq + sum(p.grad.double().pow(2).sum() for n, p in self.model.named_parameters()
                                          if p.grad is not None and not is_expert_param(n) and id(p) not in sharded)
                exp_sq = torch.zeros((), dtype=torch.float64)
                for blk in self.model.moe_blocks():
                    w = redundant_slot_weights(blk, blk.placement)
                    for p in (blk.gate_up_proj, blk.down_proj):
                        if p.grad is not None:
                            per = p.grad.double().pow(2).flatten(1).sum(1)
                            exp_sq = exp_sq + (per * torch.tensor(w, dtype=torch.float64)).sum()
                if self.world > 1:
                    dist.all_reduce(exp_sq)
                norm = float((dense_sq + exp_sq).sqrt())
                self.metrics["grad_norm"] = norm
                coef = min(1.0, cfg.max_grad_norm / (norm + 1e-6))
                if coef < 1.0:
                    for p in self.model.parameters():
                        if p.grad is not None:
                            p.grad.mul_(coef)
                if self.dense_shards is not None:
                    self.dense_shards.grad_scale = torch.tensor(coef, dtype=torch.float32)
        mult = self.lr_schedule.multiplier(self.global_step)
        for g in self.optimizer.param_groups:
            g.setdefault("initial_lr", g["lr"])
            g["lr"] = g["initial_lr"] * mult  # each group keeps its own base rate (Muon vs AdamW)
        self.optimizer.step()
        self.zero_grad()

    def _zero_all_grads(self):
        for p in self.model.parameters():
            p.grad = None
            g = getattr(p, "main_grad", None)
            if g is not None:
                g.zero_()
                p._main_grad_stale = False

    def zero_grad(self):
        expert = {id(p) for p in self.model.expert_parameters()}
        for p in self.model.parameters():
            p.grad = None
            g = getattr(p, "main_grad", None)
            if g is not None and self.pstate.dense_bucket is None and id(p) not in expert:
                g.zero_()
        if self.pstate.dense_bucket is not None:
            self.pstate.dense_bucket.zero()
        if self.dense_shards is not None:
            self.dense_shards.zero_grad()
        # expert gradients (the bulk) are overwritten by the step's first weight-gradient GEMM
        moe_ops.mark_grads_stale(self.model.expert_parameters())

    def train(self, data_iter, steps: int | None = None, log=print):
        steps = steps or self.cfg.total_steps
        t0 = time.perf_counter()
        for s in range(steps):
            batch = next(data_iter)
            loss = self.train_step(batch)
            if self.rank == 0 and log and (s % max(1, self.cfg.log_interval) == 0 or s == steps - 1):
                log(f"step {self.global_step} loss {loss:.4f} ({time.perf_counter() - t0:.1f}s)")
        return self
