"""Relative-position bias of ClusterAttention (src/layers/attention.py:72-125).

* ``pos_bias_gather(pe_table [T,H], pe_idx [B,N,M]) -> bias [B,H,N,M]`` with
  ``bias[b,h,n,m] = pe_table[pe_idx[b,n,m], h]``: the reference's
  ``index_select`` + ``view`` + ``permute`` + ``contiguous`` in one kernel, and
  its backward as one scatter-add into the table gradient;
* ``rel_pos_bias(weight [H,5], bias [H], pe_idx, dtype)``: the same bias for a
  ``Linear(5 -> H)`` over the reference's relative-position table, evaluated
  per element without forming the table; its backward reduces straight into
  the Linear's weight and bias gradients.
"""
from __future__ import annotations

import torch
from torch.autograd import Function
from torch.amp import custom_fwd, custom_bwd

from .. import _native as nat


class PosBiasGatherFunction(Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, pe_table, pe_idx):
        nat.require_cuda(pe_table, pe_idx)
        T, H = pe_table.shape
        B, N, M = pe_idx.shape
        tab = pe_table.contiguous()
        idx = pe_idx.to(torch.int64).contiguous()
        out = torch.empty((B, H, N, M), device=tab.device, dtype=tab.dtype)
        nat.call("affb_pos_bias_fwd", nat.ptr(tab), nat.ptr(idx), nat.dcode(tab), T, H, B, N, M,
                 nat.ptr(out), nat.stream(tab.device))
        ctx.save_for_backward(idx)
        ctx.meta = (T, H, tab.dtype)
        return out

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dbias):
        (idx,) = ctx.saved_tensors
        T, H, dt = ctx.meta
        B, N, M = idx.shape
        g = dbias.to(dt).contiguous()
        dtab = torch.zeros((T, H), device=g.device, dtype=torch.float32)
        nat.call("affb_pos_bias_bwd", nat.ptr(g), nat.ptr(idx), nat.dcode(g), T, H, B, N, M,
                 nat.ptr(dtab), nat.stream(g.device))
        return dtab.to(dt), None


def pos_bias_gather(pe_table, pe_idx):
    return PosBiasGatherFunction.apply(pe_table, pe_idx)


class RelPosBiasFunction(Function):
    @staticmethod
    def forward(ctx, weight, bias, pe_idx, dtype):
        nat.require_cuda(weight, bias, pe_idx)
        H = weight.shape[0]
        B, N, M = pe_idx.shape
        w = weight.detach().float().contiguous()
        b = bias.detach().float().contiguous()
        idx = pe_idx.to(torch.int64).contiguous()
        out = torch.empty((B, H, N, M), device=w.device, dtype=dtype)
        nat.call("affb_rel_bias_fwd", nat.ptr(w), nat.ptr(b), nat.ptr(idx), nat.dcode(out), H, B, N, M,
                 nat.ptr(out), nat.stream(w.device))
        ctx.save_for_backward(idx)
        ctx.meta = (H, weight.dtype, bias.dtype)
        return out

    @staticmethod
    def backward(ctx, dout):
        (idx,) = ctx.saved_tensors
        H, wdt, bdt = ctx.meta
        B, N, M = idx.shape
        g = dout.contiguous()
        if g.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            g = g.float()
        dw = torch.zeros((H, 5), device=g.device, dtype=torch.float32)
        db = torch.zeros((H,), device=g.device, dtype=torch.float32)
        nat.call("affb_rel_bias_bwd", nat.ptr(g), nat.ptr(idx), nat.dcode(g), H, B, N, M, nat.ptr(dw),
                 nat.ptr(db), nat.stream(g.device))
        return dw.to(wdt), db.to(bdt), None, None


def rel_pos_bias(weight, bias, pe_idx, dtype=torch.float32):
    """weight [H,5], bias [H] (a Linear(5 -> H) over the relative-position
    table), pe_idx [B,N,M] -> bias [B,H,N,M] in `dtype`."""
    return RelPosBiasFunction.apply(weight, bias, pe_idx, dtype)
