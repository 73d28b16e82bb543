"""Shepard weights of given neighbours (mirrors src/layers/kernels/mssample.py).

``mssample(sampling_locs [B,N,D], kv_pos [B,Nkv,D], nb_idx [B,N,K], power, D=2)``
returns ``nn_weights [B,N,K,1] = softmax_k(-P * sqrt(d2 + 1e-6))`` (note the
epsilon inside the square root, unlike the fused kernels), P = max(power, 1e-6);
backward returns ``(d_sampling_locs, d_kv_pos, None, d_power, None)``
(mssample.py:402-448).
"""
from __future__ import annotations

import torch
from torch.autograd import Function
from torch.amp import custom_fwd, custom_bwd

from .. import _native as nat


def mssample_forward(sampling_locs, kv_pos, nb_idx, power, D=2):
    B, N, _ = sampling_locs.shape
    Nkv = kv_pos.shape[1]
    K = nb_idx.shape[-1]
    dev = sampling_locs.device
    w = torch.empty((B, N, K), device=dev, dtype=torch.float32)
    nat.call("affb_mssample_fwd", nat.ptr(nat.f32(sampling_locs)), nat.ptr(nat.f32(kv_pos)),
             nat.ptr(nb_idx.to(torch.int32).contiguous()), nat.ptr(nat.scalar_dev(power, dev)),
             B, N, Nkv, K, D, nat.ptr(w), nat.stream(dev))
    return w.to(sampling_locs.dtype).unsqueeze(-1)


def mssample_backward(dout, sampling_locs, kv_pos, nb_idx, power, nn_weights, D=2):
    B, N, _ = sampling_locs.shape
    Nkv = kv_pos.shape[1]
    K = nb_idx.shape[-1]
    dev = sampling_locs.device
    d_sl = torch.empty((B, N, D), device=dev, dtype=torch.float32)
    d_kv = torch.zeros((B, Nkv, D), device=dev, dtype=torch.float32)
    d_pow = torch.zeros((1,), device=dev, dtype=torch.float32)
    nat.call("affb_mssample_bwd", nat.ptr(nat.f32(dout.reshape(B, N, K))),
             nat.ptr(nat.f32(sampling_locs)), nat.ptr(nat.f32(kv_pos)),
             nat.ptr(nb_idx.to(torch.int32).contiguous()), nat.ptr(nat.scalar_dev(power, dev)),
             nat.ptr(nat.f32(nn_weights.reshape(B, N, K))), B, N, Nkv, K, D, nat.ptr(d_sl),
             nat.ptr(d_kv), nat.ptr(d_pow), nat.stream(dev))
    return d_sl.to(sampling_locs.dtype), d_kv.to(kv_pos.dtype), d_pow[0]


class MSSampleFunction(Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, sampling_locs, kv_pos, nb_idx, power, D=2):
        nat.require_cuda(sampling_locs, kv_pos, nb_idx)
        nb_idx = nb_idx.to(torch.int32).contiguous()
        nn_weights = mssample_forward(sampling_locs, kv_pos, nb_idx, power, D)
        ctx.save_for_backward(sampling_locs, kv_pos, nb_idx, power, nn_weights)
        ctx.D = D
        return nn_weights

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dout):
        sampling_locs, kv_pos, nb_idx, power, nn_weights = ctx.saved_tensors
        d_sl, d_kv, d_pow = mssample_backward(dout, sampling_locs, kv_pos, nb_idx, power,
                                              nn_weights, ctx.D)
        d_p = d_pow.reshape(power.shape).to(power.dtype) if torch.is_tensor(power) else None
        return d_sl, d_kv, None, d_p, None


def mssample(sampling_locs, kv_pos, nb_idx, power, D=2):
    return MSSampleFunction.apply(sampling_locs, kv_pos, nb_idx, power, D)
