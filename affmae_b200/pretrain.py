"""One AFF-small MAE pretraining step on the affmae_b200 operators (config 5).

Mirrors the reference's training loop (pretrain.py:47-110, 260-290): AdamW
(lr 5e-4, weight decay 0.05 on weight matrices only, betas 0.883 / 0.935),
gradient-norm clipping at 5.0, mixed precision (bf16 autocast here, so no
loss scaler).  Data parallelism is plain DistributedDataParallel over NCCL:
one process per GPU, gradients all-reduced in buckets while the backward
pass is still running.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .mae import AFFMaskedAutoEncoder, MAEConfig


def param_groups(model: nn.Module, weight_decay: float):
    decay, no_decay = [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        (no_decay if p.dim() == 1 or name.endswith(".bias") else decay).append(p)
    return [{"params": decay, "weight_decay": weight_decay}, {"params": no_decay, "weight_decay": 0.0}]


def make_optimizer(model: nn.Module, lr: float = 5e-4, weight_decay: float = 0.05,
                   betas=(0.883, 0.935)) -> torch.optim.Optimizer:
    return torch.optim.AdamW(param_groups(model, weight_decay), lr=lr, betas=betas,
                             fused=torch.cuda.is_available())


def wrap_ddp(model: nn.Module) -> nn.Module:
    """DistributedDataParallel over the default process group (NCCL on GPUs):
    gradients are averaged in buckets as the backward pass produces them."""
    dev = next(model.parameters()).device
    return nn.parallel.DistributedDataParallel(
        model, device_ids=[dev.index] if dev.type == "cuda" else None, broadcast_buffers=False,
        gradient_as_bucket_view=True)


def build(cfg: MAEConfig = MAEConfig(), device="cuda", ddp: bool = False, seed: int = 0):
    """Model (random init from `seed`, identical on every rank), optimizer."""
    torch.manual_seed(seed)
    model = AFFMaskedAutoEncoder(cfg).to(device)
    if ddp:
        model = wrap_ddp(model)
    return model, make_optimizer(model)


def train_step(model: nn.Module, opt: torch.optim.Optimizer, images: torch.Tensor,
               clip: float = 5.0, **kw) -> torch.Tensor:
    """Forward (bf16 autocast), backward, clip, update.  Returns the loss."""
    with torch.autocast(device_type=images.device.type, dtype=torch.bfloat16):
        loss, _ = model(images, **kw)
    loss.backward()
    torch.nn.utils.clip_grad_norm_(model.parameters(), clip)
    opt.step()
    opt.zero_grad(set_to_none=True)
    return loss.detach()


def synthetic_images(batch: int, size: int, seed: int, device="cuda") -> torch.Tensor:
    """N(0,1) single-channel images, normalised per image (the benchmark's
    stand-in for the reference's EM image shards)."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((batch, 1, size, size), device=device, generator=g)
    mu = x.mean(dim=(1, 2, 3), keepdim=True)
    sd = x.std(dim=(1, 2, 3), keepdim=True)
    return (x - mu) / (sd + 1e-6)
