"""Weighted neighbour gather (mirrors src/layers/kernels/weighted_gather.py).

``weighted_gather(nbhd_idx [B,N,M], weights [B,N,M], feat [B,N_old,C])``
returns ``[B,N,C]`` with ``out[b,n,c] = sum_k w[b,n,k] * feat[b, idx[b,n,k], c]``;
gradients ``(None, d_weights, d_feat)`` as in ``WeightedGatherFunction``
(weighted_gather.py:329-359).  Runs on the weighted-features kernels with IC = 1.
"""
from __future__ import annotations

import torch
from torch.autograd import Function
from torch.amp import custom_fwd, custom_bwd

from .weighted_features import weighted_features_fwd, weighted_features_bwd


def launch_weighted_gather_fwd_kernel(nbhd_idx, weights, feat):
    return weighted_features_fwd(weights.unsqueeze(-1), feat, nbhd_idx).squeeze(2)


def launch_weighted_gather_bwd_kernel(dout, nbhd_idx, weights, feat):
    dw, dfeat = weighted_features_bwd(dout.unsqueeze(2), weights.unsqueeze(-1), feat, nbhd_idx)
    return dw.squeeze(-1), dfeat


class WeightedGatherFunction(Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, nbhd_idx, weights, feat):
        assert nbhd_idx.is_cuda and weights.is_cuda and feat.is_cuda, "All inputs must be CUDA tensors."
        nbhd_idx = nbhd_idx.to(torch.int32).contiguous()
        out = launch_weighted_gather_fwd_kernel(nbhd_idx, weights, feat)
        ctx.save_for_backward(nbhd_idx, weights, feat)
        return out

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dout):
        nbhd_idx, weights, feat = ctx.saved_tensors
        dw, dfeat = launch_weighted_gather_bwd_kernel(dout, nbhd_idx, weights, feat)
        return None, dw.to(weights.dtype), dfeat.to(feat.dtype)


def weighted_gather(nbhd_idx, weights, feat):
    return WeightedGatherFunction.apply(nbhd_idx, weights, feat)
