"""Per-head splits and merges around the neighbourhood attention.

ClusterAttention (src/layers/attention.py:126-207) views its q projection
[B, N, H*d] and kv projection [B, N, H*2d] per head, permutes them to the
operator's [B, H, N, d] (``.permute(0, 2, 1, 3).contiguous()``) and permutes
the output back to [B, N, H*d].  ``split_heads`` / ``merge_heads`` do those
moves (and their gradients) with one strided 16-byte copy kernel each
(``affb_head_copy``) instead of PyTorch's general permute copies.
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from .. import _native as nat


def _copy(src, s_strides, dst, d_strides, B, N, H, d, src_off=0, dst_off=0):
    esz = src.element_size()
    nat.call("affb_head_copy", nat.ptr(src) + src_off * esz, *s_strides, nat.ptr(dst) + dst_off * esz, *d_strides,
             esz, B, N, H, d, nat.stream(src.device))


class SplitHeadsFunction(Function):
    """x [B, N, H*parts*d] laid out per token as [H, parts, d] -> `parts`
    tensors [B, H, N, d] (part p of every head)."""

    @staticmethod
    def forward(ctx, x, H, parts):
        nat.require_cuda(x)
        x = x.contiguous()
        B, N, W = x.shape
        d = W // (H * parts)
        assert d * H * parts == W, "last dimension must be heads * parts * head_dim"
        outs = []
        for p in range(parts):
            o = torch.empty((B, H, N, d), device=x.device, dtype=x.dtype)
            _copy(x, (N * W, W, parts * d), o, (H * N * d, d, N * d), B, N, H, d, src_off=p * d)
            outs.append(o)
        ctx.meta = (B, N, H, d, parts)
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        B, N, H, d, parts = ctx.meta
        W = H * parts * d
        ref = next(g for g in grads if g is not None)
        full = all(g is not None for g in grads)
        dx = (torch.empty if full else torch.zeros)((B, N, W), device=ref.device, dtype=ref.dtype)
        for p, g in enumerate(grads):
            if g is None:
                continue
            g = g.to(ref.dtype).contiguous()
            _copy(g, (H * N * d, d, N * d), dx, (N * W, W, parts * d), B, N, H, d, dst_off=p * d)
        return dx, None, None


class MergeHeadsFunction(Function):
    """o [B, H, N, d] -> [B, N, H*d]."""

    @staticmethod
    def forward(ctx, o):
        nat.require_cuda(o)
        o = o.contiguous()
        B, H, N, d = o.shape
        y = torch.empty((B, N, H * d), device=o.device, dtype=o.dtype)
        _copy(o, (H * N * d, d, N * d), y, (N * H * d, H * d, d), B, N, H, d)
        ctx.meta = (B, N, H, d)
        return y

    @staticmethod
    def backward(ctx, g):
        B, N, H, d = ctx.meta
        g = g.contiguous()
        do = torch.empty((B, H, N, d), device=g.device, dtype=g.dtype)
        _copy(g, (N * H * d, H * d, d), do, (H * N * d, d, N * d), B, N, H, d)
        return do


def split_heads(x: torch.Tensor, heads: int, parts: int = 1):
    """Returns `parts` tensors [B, H, N, d] (a single tensor when parts == 1)."""
    outs = SplitHeadsFunction.apply(x, heads, parts)
    return outs[0] if parts == 1 else outs


def merge_heads(o: torch.Tensor) -> torch.Tensor:
    return MergeHeadsFunction.apply(o)
