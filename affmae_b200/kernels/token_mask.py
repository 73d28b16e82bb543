"""Token-mask multiply of the patch stem (the masking glue of the reference's
AFFPatchEmbed, src/layers/aff.py:591-639, and of the image masking before it).

``apply_token_mask(x, token_mask)`` returns ``x * upsample(token_mask)`` for a
channels-last feature map ``x`` (logical [B, C, h, w], memory [B, h, w, C])
and a [B, th, tw] token mask with h / th = w / tw an integer, without
materialising the upsampled mask; its gradient is the same product.
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from .. import _native as nat


def _apply(x, tm8, th, tw):
    B, C, h, w = x.shape
    xc = x.contiguous(memory_format=torch.channels_last) if C > 1 else x.contiguous()
    out = torch.empty_like(xc)
    nat.call("affb_token_mask_apply", nat.ptr(xc), nat.dcode(xc), B, h, w, C, nat.ptr(tm8), th, tw,
             nat.ptr(out), nat.stream(x.device))
    return out


class TokenMaskFunction(Function):
    @staticmethod
    def forward(ctx, x, token_mask):
        nat.require_cuda(x, token_mask)
        tm8 = (token_mask != 0).to(torch.uint8).contiguous()
        th, tw = tm8.shape[-2:]
        ctx.save_for_backward(tm8)
        return _apply(x, tm8, th, tw)

    @staticmethod
    def backward(ctx, g):
        (tm8,) = ctx.saved_tensors
        th, tw = tm8.shape[-2:]
        return _apply(g, tm8, th, tw), None


def apply_token_mask(x, token_mask):
    """x [B,C,h,w] (channels-last when C > 1), token_mask [B,th,tw] (nonzero = keep)."""
    return TokenMaskFunction.apply(x, token_mask)
