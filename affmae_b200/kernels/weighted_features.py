"""Importance-weighted gather (mirrors src/layers/kernels/weighted_features.py).

``weighted_features(weights [B,No,M,IC], feat [B,N,C], nbhd_idx [B,No,M])``
returns ``out [B,No,IC,C]`` with ``out[b,i,ic,c] = sum_m w[b,i,m,ic] *
feat[b, idx[b,i,m], c]``; gradients ``(d_weights, d_feat, None)`` as in
``WeightedFeaturesFunction`` (weighted_features.py:401-429).  The output has
the dtype of ``feat``; weights are read in that dtype too.
"""
from __future__ import annotations

import torch
from torch.autograd import Function
from torch.amp import custom_fwd, custom_bwd

from .. import _native as nat


def weighted_features_fwd(weights, feat, nbhd_idx):
    B, No, M, IC = weights.shape
    _, N, C = feat.shape
    dt = feat.dtype
    w = weights.to(dt).contiguous()
    f = feat.contiguous()
    idx = nbhd_idx.to(torch.int32).contiguous()
    out = torch.empty((B, No, IC, C), device=feat.device, dtype=dt)
    nat.call("affb_weighted_features_fwd", nat.ptr(w), nat.ptr(f), nat.ptr(idx), nat.dcode(f),
             B, No, M, IC, N, C, nat.ptr(out), nat.stream(feat.device))
    return out


def weighted_features_bwd(dout, weights, feat, nbhd_idx):
    B, No, M, IC = weights.shape
    _, N, C = feat.shape
    dt = feat.dtype
    w = weights.to(dt).contiguous()
    f = feat.contiguous()
    g = dout.to(dt).contiguous()
    idx = nbhd_idx.to(torch.int32).contiguous()
    dw = torch.empty((B, No, M, IC), device=feat.device, dtype=dt)
    dfeat = torch.zeros((B, N, C), device=feat.device, dtype=torch.float32)
    nat.call("affb_weighted_features_bwd", nat.ptr(g), nat.ptr(w), nat.ptr(f), nat.ptr(idx),
             nat.dcode(f), B, No, M, IC, N, C, nat.ptr(dw), nat.ptr(dfeat),
             nat.stream(feat.device))
    return dw, nat.cast_from_f32(dfeat, dt)


class WeightedFeaturesFunction(Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, weights, feat, nbhd_idx):
        assert weights.is_cuda and feat.is_cuda and nbhd_idx.is_cuda
        nbhd_idx = nbhd_idx.to(torch.int32).contiguous()
        out = weighted_features_fwd(weights, feat, nbhd_idx)
        ctx.save_for_backward(weights, feat, nbhd_idx)
        return out

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dout):
        weights, feat, nbhd_idx = ctx.saved_tensors
        dw, dfeat = weighted_features_bwd(dout, weights, feat, nbhd_idx)
        return dw.to(weights.dtype), dfeat.to(feat.dtype), None


def weighted_features(weights, feat, nbhd_idx):
    return WeightedFeaturesFunction.apply(weights, feat, nbhd_idx)


def weighted_features_ref(weights, feat, nbhd_idx):
    """Plain PyTorch formula of the op (reference weighted_features.py:440-457)."""
    B, N_out, M, IC = weights.shape
    _, N, C = feat.shape
    gathered = feat.gather(dim=1, index=nbhd_idx.reshape(B, N_out * M)[..., None].expand(-1, -1, C))
    gathered = gathered.reshape(B, N_out, M, C)
    return (weights[..., None] * gathered[:, :, :, None, :]).sum(dim=2)


def weighted_features_triton(weights, feat, nbhd_idx):
    """Forward launcher of the reference (weighted_features.py:114): [B,No,IC,C]."""
    return weighted_features_fwd(weights, feat, nbhd_idx)


def weighted_features_triton_backward(dout, weights, feat, nbhd_idx):
    """Backward launcher of the reference (weighted_features.py:348): (d_weights, d_feat)."""
    dw, dfeat = weighted_features_bwd(dout, weights, feat, nbhd_idx)
    return dw.to(weights.dtype), dfeat.to(feat.dtype)
