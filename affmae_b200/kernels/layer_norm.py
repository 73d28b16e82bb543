"""Fused residual + dropout + LayerNorm (the elementwise fusion around the
operators in the model; no counterpart module among the reference kernels).

``fused_layer_norm(x, weight, bias, eps, delta=None, p=0.0, out32=True,
out16=False)`` computes ``LayerNorm(x + dropout_p(delta))`` in one pass and
returns it as fp32 (the residual stream) and/or bf16 (the input of the next
Linear under bf16 autocast, produced without a separate cast), in that order.
The backward takes the gradients of both outputs at once and returns those
of x, delta, weight and bias.  The dropout mask is regenerated from a seed
drawn from the CPU generator, so it follows ``torch.manual_seed``.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd import Function

from .. import _native as nat

_OK = (torch.float32, torch.bfloat16)


class FusedLayerNormFunction(Function):
    @staticmethod
    def forward(ctx, x, delta, weight, bias, eps, p, out32, out16):
        C = x.shape[-1]
        R = x.numel() // C
        dev = x.device
        xc = x.contiguous()
        dc = delta.contiguous() if delta is not None else None
        seed = int(torch.randint(0, 2 ** 31 - 1, (1,)).item()) if (dc is not None and p > 0) else 0
        s = torch.empty(x.shape, device=dev, dtype=torch.float32) if dc is not None else None
        mean = torch.empty(R, device=dev, dtype=torch.float32)
        rstd = torch.empty(R, device=dev, dtype=torch.float32)
        y32 = torch.empty(x.shape, device=dev, dtype=torch.float32) if out32 else None
        y16 = torch.empty(x.shape, device=dev, dtype=torch.bfloat16) if out16 else None
        w = weight.detach().float().contiguous()
        b = bias.detach().float().contiguous()
        nat.call("affb_layer_norm_fwd", nat.ptr(xc), nat.dcode(xc), nat.ptr(dc),
                 nat.dcode(dc) if dc is not None else 0, float(p), seed, nat.ptr(w), nat.ptr(b), float(eps),
                 R, C, nat.ptr(s), nat.ptr(mean), nat.ptr(rstd), nat.ptr(y32), nat.ptr(y16), nat.stream(dev))
        ctx.save_for_backward(s if s is not None else xc, mean, rstd, w)
        ctx.meta = (None if dc is None else dc.dtype, float(p), seed, x.dtype, out32, out16, weight.dtype,
                    bias.dtype, R, C)
        outs = [t for t in (y32, y16) if t is not None]
        return tuple(outs) if len(outs) > 1 else outs[0]

    @staticmethod
    def backward(ctx, *grads):
        s, mean, rstd, w = ctx.saved_tensors
        ddt, p, seed, xdt, out32, out16, wdt, bdt, R, C = ctx.meta
        g32 = grads[0] if out32 else None
        g16 = grads[-1] if out16 else None
        g32 = g32.float().contiguous() if g32 is not None else None
        g16 = g16.to(torch.bfloat16).contiguous() if g16 is not None else None
        dev = s.device
        if g32 is None and g16 is None:
            g32 = torch.zeros(s.shape, device=dev, dtype=torch.float32)
        dx = torch.empty(s.shape, device=dev, dtype=s.dtype)
        dd = torch.empty(s.shape, device=dev, dtype=ddt) if ddt is not None else None
        dg = torch.zeros(C, device=dev, dtype=torch.float32)
        db = torch.zeros(C, device=dev, dtype=torch.float32)
        nat.call("affb_layer_norm_bwd", nat.ptr(g32), nat.ptr(g16), nat.ptr(s), nat.dcode(s), nat.ptr(mean),
                 nat.ptr(rstd), nat.ptr(w), p, seed, R, C, nat.ptr(dx), nat.ptr(dd),
                 nat.dcode(dd) if dd is not None else 0, nat.ptr(dg), nat.ptr(db), nat.stream(dev))
        return dx.to(xdt), dd, dg.to(wdt), db.to(bdt), None, None, None, None


class ResidualNormFunction(Function):
    """(s, y) = (x + row_scale * delta, LayerNorm(s)) for the pre-norm blocks:
    s (fp32) is the residual stream kept by the caller, y (bf16) feeds the
    next Linear; row_scale [G] (or None) multiplies delta per group of
    R / G consecutive rows (stochastic depth per sample)."""

    @staticmethod
    def forward(ctx, x, delta, row_scale, weight, bias, eps):
        C = x.shape[-1]
        R = x.numel() // C
        dev = x.device
        xc, dc = x.contiguous(), delta.contiguous()
        rs = row_scale.float().contiguous() if row_scale is not None else None
        rps = R // rs.numel() if rs is not None else 1
        s = torch.empty(x.shape, device=dev, dtype=torch.float32)
        mean = torch.empty(R, device=dev, dtype=torch.float32)
        rstd = torch.empty(R, device=dev, dtype=torch.float32)
        y16 = torch.empty(x.shape, device=dev, dtype=torch.bfloat16)
        w = weight.detach().float().contiguous()
        b = bias.detach().float().contiguous()
        nat.call("affb_layer_norm_res_fwd", nat.ptr(xc), nat.dcode(xc), nat.ptr(dc), nat.dcode(dc), 0.0, 0,
                 nat.ptr(rs), rps, nat.ptr(w), nat.ptr(b), float(eps), R, C, nat.ptr(s), nat.ptr(mean),
                 nat.ptr(rstd), None, nat.ptr(y16), nat.stream(dev))
        ctx.save_for_backward(s, mean, rstd, w, rs)
        ctx.meta = (dc.dtype, x.dtype, weight.dtype, bias.dtype, R, C, rps)
        return s, y16

    @staticmethod
    def backward(ctx, ds, dy16):
        s, mean, rstd, w, rs = ctx.saved_tensors
        ddt, xdt, wdt, bdt, R, C, rps = ctx.meta
        dev = s.device
        ds = ds.float().contiguous() if ds is not None else None
        if dy16 is None:
            dy16 = torch.zeros(s.shape, device=dev, dtype=torch.bfloat16)
        dy16 = dy16.to(torch.bfloat16).contiguous()
        dx = torch.empty(s.shape, device=dev, dtype=torch.float32)
        dd = torch.empty(s.shape, device=dev, dtype=ddt)
        dg = torch.zeros(C, device=dev, dtype=torch.float32)
        db = torch.zeros(C, device=dev, dtype=torch.float32)
        nat.call("affb_layer_norm_res_bwd", None, nat.ptr(dy16), nat.ptr(ds), nat.ptr(s), nat.ptr(mean),
                 nat.ptr(rstd), nat.ptr(w), 0.0, 0, nat.ptr(rs), rps, R, C, nat.ptr(dx), nat.ptr(dd),
                 nat.dcode(dd), nat.ptr(dg), nat.ptr(db), nat.stream(dev))
        return dx.to(xdt), dd, None, dg.to(wdt), db.to(bdt), None


def fused_layer_norm(x, weight, bias, eps=1e-5, delta=None, p=0.0, out32=True, out16=False):
    nat.require_cuda(x, weight, bias)
    assert x.dtype in _OK and (delta is None or (delta.dtype in _OK and x.dtype == torch.float32))
    assert out32 or out16
    return FusedLayerNormFunction.apply(x, delta, weight, bias, eps, p, out32, out16)


class FusedLayerNorm(nn.LayerNorm):
    """nn.LayerNorm whose forward optionally adds ``dropout_p(delta)`` first and
    returns the fp32 result and/or its bf16 copy.  Falls back to PyTorch ops
    off the GPU, outside bf16 autocast or for other dtypes (the bf16 output is
    then the fp32 result itself)."""

    def forward(self, x, delta=None, p=0.0, out32=True, out16=False):
        p = p if self.training else 0.0
        fused = (x.is_cuda and x.shape[-1] <= 1536 and x.dtype in _OK and
                 (delta is None or (delta.dtype in _OK and x.dtype == torch.float32)) and
                 torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16)
        if fused:
            return fused_layer_norm(x, self.weight, self.bias, self.eps, delta, p, out32, out16)
        s = x if delta is None else x + F.dropout(delta, p, self.training)
        y = F.layer_norm(s, self.normalized_shape, self.weight, self.bias, self.eps)
        if out32 and out16:
            return y, y
        return y

    def residual(self, x, delta, row_scale=None):
        """(s, y): s = x + row_scale * delta (row_scale [B] per sample of x
        [B, ..., C], or None), y = LayerNorm(s) in bf16 under bf16 autocast
        (fp32 otherwise).  One pass on the GPU under bf16 autocast, where s is
        fp32 whatever the dtype of x."""
        fused = (x.is_cuda and x.shape[-1] <= 1536 and x.dtype in _OK and delta.dtype in _OK and
                 torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16)
        if fused:
            nat.require_cuda(x, delta, self.weight, self.bias)
            return ResidualNormFunction.apply(x, delta, row_scale, self.weight, self.bias, self.eps)
        if row_scale is not None:
            delta = delta * row_scale.view((-1,) + (1,) * (delta.dim() - 1)).to(delta.dtype)
        s = x + delta
        return s, F.layer_norm(s, self.normalized_shape, self.weight, self.bias, self.eps)
