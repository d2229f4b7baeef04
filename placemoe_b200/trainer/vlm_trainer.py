"""VLMTrainer: MoE text decoder + a compact vision tower for ``tasks/train_vlm.py``.

The vision tower patchifies images (``patch x patch x 3`` pixels -> hidden)
with two projection layers (patch embed, merger MLP) on the same tcgen05
GEMMs, and the resulting visual tokens replace the first positions of each
sequence (the positions an image placeholder occupies in Qwen-VL style
inputs).  Synthetic data: uniform token ids plus N(0, 1) pixels.  Visual
positions carry no language-model labels.

Reference parity: veomni/trainer/vlm_trainer.py (VLMTrainer) -- the reference
trains full Qwen-VL vision towers; this one keeps the decoder/MoE/placement
path identical and uses a minimal tower.
"""

from __future__ import annotations

import time

import torch
import torch.nn as nn

from ..arguments.parser import Arguments
from ..ops import loss as loss_ops
from ..ops import mp as mp_ops
from .text_trainer import TextTrainer


class VisionTower(nn.Module):
    def __init__(self, hidden: int, patch: int = 14, channels: int = 3):
        super().__init__()
        self.patch = patch
        d_in = patch * patch * channels
        self.patch_embed = nn.Parameter(torch.empty(hidden, d_in))
        self.merger_fc1 = nn.Parameter(torch.empty(hidden, hidden))
        self.merger_fc2 = nn.Parameter(torch.empty(hidden, hidden))
        for p in self.parameters():
            nn.init.normal_(p, std=0.02)

    def forward(self, pixels: torch.Tensor) -> torch.Tensor:
        # pixels [B, N, patch*patch*3] -> [B, N, hidden]
        x = mp_ops.linear(pixels, self.patch_embed)
        x = torch.nn.functional.gelu(mp_ops.linear(x, self.merger_fc1).float()).to(x.dtype)
        return mp_ops.linear(x, self.merger_fc2)


class VLMTrainer(TextTrainer):
    def __init__(self, args: Arguments, num_image_tokens: int = 256):
        super().__init__(args)
        tr = self.trainer
        self.n_img = num_image_tokens
        with torch.device(tr.device):
            self.vision = VisionTower(tr.model_cfg.hidden_size)
        self.vision.to(tr.device)
        tr.optimizer.add_param_group({"params": list(self.vision.parameters()), **{
            k: v for k, v in tr.optimizer.defaults.items()}})
        tr.optimizer.reset_tables()
        g = torch.Generator().manual_seed(1234 + tr.rank)
        self._pix = lambda b: torch.randn(b, self.n_img, 14 * 14 * 3, generator=g)
        model = tr.model
        vision = self.vision
        n_img = self.n_img

        def forward_backward(input_ids):
            b, s = input_ids.shape
            pixels = self._pix(b).to(tr.device, non_blocking=True)
            img = vision(pixels)  # [B, n_img, H]
            ids = input_ids.reshape(-1)
            x = mp_ops.embedding(ids, model.embed_tokens, model._anchor(ids.device)).view(b, s, -1)
            x = torch.cat([img.to(x.dtype), x[:, n_img:]], dim=1).reshape(b * s, -1)
            pos = torch.arange(s, device=ids.device, dtype=torch.int32).repeat(b)
            for layer in model.layers:
                x = layer(x, pos, s)
            h = model.norm(x)
            labels = torch.full_like(input_ids, loss_ops.IGNORE_INDEX)
            labels[:, n_img:-1] = input_ids[:, n_img + 1:]
            w = model.embed_tokens if model.lm_head is None else model.lm_head
            loss = loss_ops.fused_linear_cross_entropy(h, w, labels)
            aux = None
            for blk in model.moe_blocks():
                if blk.last_aux_loss is not None:
                    aux = blk.last_aux_loss if aux is None else aux + blk.last_aux_loss
            total = loss / tr.world + (aux / tr.world if aux is not None else 0.0)
            total.backward()
            return loss.detach()

        tr.forward_backward = forward_backward
        # vision tower gradients join the dense bucket reduction
        if tr.pstate.dense_bucket is not None:
            from ..parallel.data_parallel import DenseGradBucket

            dense = tr.pstate.dense_bucket.params + list(self.vision.parameters())
            tr.pstate.dense_bucket = DenseGradBucket(dense, tr.device)
            tr._norm_table = None

    def train(self):
        t = self.args.train
        tr = self.trainer
        t0 = time.perf_counter()
        for step in range(tr.global_step, t.max_steps):
            loss = tr.train_step(next(self.data))
            if tr.rank == 0 and (step % max(1, t.log_interval) == 0 or step == t.max_steps - 1):
                print(f"[vlm] step {step + 1}/{t.max_steps} loss {loss:.4f} elapsed {time.perf_counter() - t0:.1f}s",
                      flush=True)
        return tr


__all__ = ["VLMTrainer", "VisionTower"]
