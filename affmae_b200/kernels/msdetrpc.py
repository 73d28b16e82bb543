"""Double-weighted neighbour gather (mirrors src/layers/kernels/msdetrpc.py).

``MSDETRPCFunction.apply(nn_idx [B,N,M,K], nn_weight [B,N,M,K], attn [B,N,M],
val [B,Nv,C]) -> [B,N,C]`` with
``out[b,n,c] = sum_m attn[b,n,m] * sum_k w[b,n,m,k] * val[b, idx[b,n,m,k], c]``;
backward returns ``(None, d_nn_weight, d_attn, d_val)`` (msdetrpc.py:372-390).
"""
from __future__ import annotations

import torch
from torch.autograd import Function
from torch.amp import custom_fwd, custom_bwd

from .. import _native as nat


def launch_msdetrpc_forward(nn_idx, nn_weight, attn, val):
    B, N, M, K = nn_idx.shape
    _, Nv, C = val.shape
    dt = val.dtype
    out = torch.empty((B, N, C), device=val.device, dtype=dt)
    nat.call("affb_msdetrpc_fwd", nat.ptr(nn_idx), nat.ptr(nn_weight.to(dt).contiguous()),
             nat.ptr(attn.to(dt).contiguous()), nat.ptr(val), nat.dcode(val), B, N, M, K, Nv, C,
             nat.ptr(out), nat.stream(val.device))
    return out


def launch_msdetrpc_backward(d_feat, nn_idx, nn_weight, attn, val):
    B, N, M, K = nn_idx.shape
    _, Nv, C = val.shape
    dt = val.dtype
    dev = val.device
    d_nw = torch.empty((B, N, M, K), device=dev, dtype=dt)
    d_att = torch.empty((B, N, M), device=dev, dtype=dt)
    d_val = torch.zeros((B, Nv, C), device=dev, dtype=torch.float32)
    nat.call("affb_msdetrpc_bwd", nat.ptr(d_feat.to(dt).contiguous()), nat.ptr(nn_idx),
             nat.ptr(nn_weight.to(dt).contiguous()), nat.ptr(attn.to(dt).contiguous()),
             nat.ptr(val), nat.dcode(val), B, N, M, K, Nv, C, nat.ptr(d_nw), nat.ptr(d_att),
             nat.ptr(d_val), nat.stream(dev))
    return d_nw, d_att, nat.cast_from_f32(d_val, dt)


class MSDETRPCFunction(Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, nn_idx, nn_weight, attn, val):
        nat.require_cuda(nn_idx, nn_weight, attn, val)
        nn_idx = nn_idx.to(torch.int32).contiguous()
        val = val.contiguous()
        out = launch_msdetrpc_forward(nn_idx, nn_weight, attn, val)
        ctx.save_for_backward(nn_idx, nn_weight, attn, val)
        return out

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, d_out):
        nn_idx, nn_weight, attn, val = ctx.saved_tensors
        d_nw, d_att, d_val = launch_msdetrpc_backward(d_out, nn_idx, nn_weight, attn, val)
        return None, d_nw.to(nn_weight.dtype), d_att.to(attn.dtype), d_val
