"""Fused KNN + Shepard deformable attention (mirrors src/layers/kernels/fused_deform_attn.py).

Public API as in the reference:
  * ``fused_knn_deformable_self_attention(pos, offsets, attn_weights, values, power, D=2)``
    (fused_deform_attn.py:4063) / ``FusedKNNDeformSelfAttnFunction`` (:3981);
  * ``fused_knn_deformable_cross_attention(query_pos, kv_pos, offsets, attn_weights,
    values, power, D=2)`` (:4095) / ``FusedKNNDeformCrossAttnFunction`` (:4020);
  * ``fused_deformable_attention(sampling_locs, kv_pos, nb_idx, power, attn_weights,
    values, D=2, use_heuristics=None)`` (:694) / ``FusedDeformAttnFunction`` (:654);
  * the ``*_forward_save`` / ``*_backward`` helpers (:2530-2925).

Geometry (positions, offsets, attention weights) is computed in fp32, as the
reference kernels do after loading; ``values`` keep their dtype and the output
has the dtype of ``values``.  ``power`` is read on the device (the reference
calls ``power.item()``, a host synchronisation, in every wrapper).
The 4 nearest neighbours are found through a per-call spatial grid instead of
the reference's scan over all kv positions; the selected indices are the same.
"""
from __future__ import annotations

import torch
from torch.autograd import Function
from torch.amp import custom_fwd, custom_bwd

from .. import _native as nat


def workspace_bytes(B: int, Nkv: int) -> int:
    return int(nat.lib().affb_deform_workspace_bytes(B, Nkv))


def fused_knn_deform_cross_attn_forward_save(query_pos, kv_pos, offsets, attn_weights, values,
                                             power, D=2, save_dist=True):
    """Returns (out [B,Nq,H,C], knn_idx [B,Nq,H,4,4] int32, knn_dist_sq [B,Nq,H,4,4] fp32).

    ``save_dist=False`` (used by the autograd Functions) skips writing the
    squared distances and returns None for them; the backward recomputes them
    from the positions bit for bit."""
    assert D == 2, "Currently only D=2 is supported"
    B, Nq, _ = query_pos.shape
    Nkv = kv_pos.shape[1]
    _, _, H, K, _ = offsets.shape
    assert K == 4, "Currently only K=4 sampling points supported"
    C = values.shape[-1]
    nat.require_cuda(query_pos, kv_pos, offsets, attn_weights, values)
    dev = values.device
    qp, kp = nat.f32(query_pos), nat.f32(kv_pos)
    off, aw = nat.f32(offsets), nat.f32(attn_weights)
    val = values.contiguous()
    pw = nat.scalar_dev(power, dev)
    out = torch.empty((B, Nq, H, C), device=dev, dtype=values.dtype)
    knn_idx = torch.empty((B, Nq, H, K, 4), device=dev, dtype=torch.int32)
    knn_d2 = torch.empty((B, Nq, H, K, 4), device=dev, dtype=torch.float32) if save_dist else None
    ws = torch.empty(workspace_bytes(B, Nkv), device=dev, dtype=torch.uint8)
    nat.call("affb_deform_knn_fwd", nat.ptr(qp), nat.ptr(kp), nat.ptr(off), nat.ptr(aw),
             nat.ptr(val), nat.ptr(pw), nat.dcode(val), B, Nq, Nkv, H, C, nat.ptr(out),
             nat.ptr(knn_idx), nat.ptr(knn_d2), nat.ptr(ws), nat.stream(dev))
    return out, knn_idx, knn_d2


def fused_knn_deform_self_attn_forward_save(pos, offsets, attn_weights, values, power, D=2, save_dist=True):
    return fused_knn_deform_cross_attn_forward_save(pos, pos, offsets, attn_weights, values, power, D, save_dist)


def _deform_backward(dout, query_pos, kv_pos, offsets, attn_weights, values, power, knn_idx,
                     knn_dist_sq, self_attn):
    B, Nq, _ = query_pos.shape
    Nkv = kv_pos.shape[1]
    _, _, H, K, _ = offsets.shape
    C = values.shape[-1]
    dev = values.device
    qp, kp = nat.f32(query_pos), nat.f32(kv_pos)
    off, aw = nat.f32(offsets), nat.f32(attn_weights)
    val = values.contiguous()
    g = dout.to(values.dtype).contiguous()
    pw = nat.scalar_dev(power, dev)
    d_off = torch.empty((B, Nq, H, K, 2), device=dev, dtype=torch.float32)
    d_aw = torch.empty((B, Nq, H, K), device=dev, dtype=torch.float32)
    d_qpos = torch.zeros((B, Nq, 2), device=dev, dtype=torch.float32)
    d_kvpos = d_qpos if self_attn else torch.zeros((B, Nkv, 2), device=dev, dtype=torch.float32)
    d_val = torch.zeros((B, Nkv, H, C), device=dev, dtype=torch.float32)
    d_pow = torch.zeros((1,), device=dev, dtype=torch.float32)
    nat.call("affb_deform_knn_bwd", nat.ptr(qp), nat.ptr(kp), nat.ptr(off), nat.ptr(aw),
             nat.ptr(val), nat.ptr(pw), nat.ptr(knn_idx.contiguous()),
             nat.ptr(None if knn_dist_sq is None else knn_dist_sq.contiguous()), nat.ptr(g), nat.dcode(val), B, Nq, Nkv, H, C,
             nat.ptr(d_off), nat.ptr(d_aw), nat.ptr(d_qpos), nat.ptr(d_kvpos), nat.ptr(d_val),
             nat.ptr(d_pow), nat.stream(dev))
    return d_qpos, d_kvpos, d_off, d_aw, nat.cast_from_f32(d_val, values.dtype), d_pow


def fused_knn_deform_cross_attn_backward(dout, query_pos, kv_pos, offsets, attn_weights, values,
                                         power, knn_idx, knn_dist_sq, D=2):
    """Returns d_query_pos, d_kv_pos, d_offsets, d_attn_weights, d_values, d_power."""
    dq, dkv, doff, daw, dval, dpow = _deform_backward(dout, query_pos, kv_pos, offsets,
                                                      attn_weights, values, power, knn_idx,
                                                      knn_dist_sq, self_attn=False)
    return (dq.to(query_pos.dtype), dkv.to(kv_pos.dtype), doff.to(offsets.dtype),
            daw.to(attn_weights.dtype), dval, dpow)


def fused_knn_deform_self_attn_backward(dout, pos, offsets, attn_weights, values, power, knn_idx,
                                        knn_dist_sq, D=2):
    """Returns d_pos, d_offsets, d_attn_weights, d_values, d_power."""
    dpos, _, doff, daw, dval, dpow = _deform_backward(dout, pos, pos, offsets, attn_weights,
                                                      values, power, knn_idx, knn_dist_sq,
                                                      self_attn=True)
    return dpos.to(pos.dtype), doff.to(offsets.dtype), daw.to(attn_weights.dtype), dval, dpow


def _power_grad(d_pow, power):
    if torch.is_tensor(power):
        return d_pow.reshape(power.shape).to(power.dtype)
    return None


class FusedKNNDeformSelfAttnFunction(Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, pos, offsets, attn_weights, values, power, D=2):
        out, knn_idx, _ = fused_knn_deform_self_attn_forward_save(
            pos, offsets, attn_weights, values, power, D, save_dist=False)
        ctx.save_for_backward(pos, offsets, attn_weights, values, power, knn_idx)
        return out

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dout):
        pos, offsets, attn_weights, values, power, knn_idx = ctx.saved_tensors
        dpos, doff, daw, dval, dpow = fused_knn_deform_self_attn_backward(
            dout, pos, offsets, attn_weights, values, power, knn_idx, None)
        return dpos, doff, daw, dval, _power_grad(dpow, power), None


class FusedKNNDeformCrossAttnFunction(Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, query_pos, kv_pos, offsets, attn_weights, values, power, D=2):
        out, knn_idx, _ = fused_knn_deform_cross_attn_forward_save(
            query_pos, kv_pos, offsets, attn_weights, values, power, D, save_dist=False)
        ctx.save_for_backward(query_pos, kv_pos, offsets, attn_weights, values, power, knn_idx)
        return out

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dout):
        query_pos, kv_pos, offsets, attn_weights, values, power, knn_idx = ctx.saved_tensors
        dq, dkv, doff, daw, dval, dpow = fused_knn_deform_cross_attn_backward(
            dout, query_pos, kv_pos, offsets, attn_weights, values, power, knn_idx, None)
        return dq, dkv, doff, daw, dval, _power_grad(dpow, power), None


def fused_knn_deformable_self_attention(pos, offsets, attn_weights, values, power, D=2):
    """pos [B,N,2], offsets [B,N,H,4,2], attn_weights [B,N,H,4], values [B,N,H,C] -> [B,N,H,C]."""
    return FusedKNNDeformSelfAttnFunction.apply(pos, offsets, attn_weights, values, power, D)


def fused_knn_deformable_cross_attention(query_pos, kv_pos, offsets, attn_weights, values, power, D=2):
    """query_pos [B,Nq,2], kv_pos [B,Nkv,2], offsets [B,Nq,H,4,2], attn_weights [B,Nq,H,4],
    values [B,Nkv,H,C] -> [B,Nq,H,C]."""
    return FusedKNNDeformCrossAttnFunction.apply(query_pos, kv_pos, offsets, attn_weights, values,
                                                 power, D)


# ------------------------------------------ deformable attention, given nb_idx
def fused_deform_attn_forward(sampling_locs, kv_pos, nb_idx, power, attn_weights, values, D=2,
                              use_heuristics=False):
    B, N, _ = sampling_locs.shape
    _, Nkv, C = values.shape
    K = nb_idx.shape[-1]
    dev = values.device
    nat.require_cuda(sampling_locs, kv_pos, nb_idx, attn_weights, values)
    out = torch.empty((B, N, C), device=dev, dtype=values.dtype)
    nat.call("affb_deform_nbidx_fwd", nat.ptr(nat.f32(sampling_locs)), nat.ptr(nat.f32(kv_pos)),
             nat.ptr(nb_idx.to(torch.int32).contiguous()), nat.ptr(nat.scalar_dev(power, dev)),
             nat.ptr(nat.f32(attn_weights)), nat.ptr(values.contiguous()), nat.dcode(values),
             B, N, Nkv, K, D, C, nat.ptr(out), nat.stream(dev))
    return out


def fused_deform_attn_backward(dout, sampling_locs, kv_pos, nb_idx, power, attn_weights, values,
                               D=2, use_heuristics=False):
    B, N, _ = sampling_locs.shape
    _, Nkv, C = values.shape
    K = nb_idx.shape[-1]
    dev = values.device
    d_sl = torch.empty((B, N, D), device=dev, dtype=torch.float32)
    d_kv = torch.zeros((B, Nkv, D), device=dev, dtype=torch.float32)
    d_pow = torch.zeros((1,), device=dev, dtype=torch.float32)
    d_aw = torch.empty((B, N), device=dev, dtype=torch.float32)
    d_val = torch.zeros((B, Nkv, C), device=dev, dtype=torch.float32)
    vals = values.contiguous()
    nat.call("affb_deform_nbidx_bwd", nat.ptr(nat.f32(sampling_locs)), nat.ptr(nat.f32(kv_pos)),
             nat.ptr(nb_idx.to(torch.int32).contiguous()), nat.ptr(nat.scalar_dev(power, dev)),
             nat.ptr(nat.f32(attn_weights)), nat.ptr(vals),
             nat.ptr(dout.to(values.dtype).contiguous()), nat.dcode(vals), B, N, Nkv, K, D, C,
             nat.ptr(d_sl), nat.ptr(d_kv), nat.ptr(d_pow), nat.ptr(d_aw), nat.ptr(d_val),
             nat.stream(dev))
    return (d_sl.to(sampling_locs.dtype), d_kv.to(kv_pos.dtype), d_pow[0],
            d_aw.to(attn_weights.dtype), nat.cast_from_f32(d_val, values.dtype))


class FusedDeformAttnFunction(Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, sampling_locs, kv_pos, nb_idx, power, attn_weights, values, D=2,
                use_heuristics=None):
        nb_idx = nb_idx.to(torch.int32).contiguous()
        out = fused_deform_attn_forward(sampling_locs, kv_pos, nb_idx, power, attn_weights,
                                        values, D)
        ctx.save_for_backward(sampling_locs, kv_pos, nb_idx, power, attn_weights, values)
        ctx.D = D
        return out

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dout):
        sampling_locs, kv_pos, nb_idx, power, attn_weights, values = ctx.saved_tensors
        d_sl, d_kv, d_pow, d_attn, d_val = fused_deform_attn_backward(
            dout, sampling_locs, kv_pos, nb_idx, power, attn_weights, values, ctx.D)
        return d_sl, d_kv, None, _power_grad(d_pow, power), d_attn, d_val, None, None


def fused_deformable_attention(sampling_locs, kv_pos, nb_idx, power, attn_weights, values, D=2,
                               use_heuristics=None):
    """sampling_locs [B,N,D], kv_pos [B,Nkv,D], nb_idx [B,N,K], attn_weights [B,N],
    values [B,Nkv,C] -> [B,N,C]."""
    return FusedDeformAttnFunction.apply(sampling_locs, kv_pos, nb_idx, power, attn_weights,
                                         values, D, use_heuristics)


# ------------------------------------------- public helpers of the reference
USE_HEURISTICS = True


def set_use_heuristics(value: bool):
    """The reference's switch between autotuning and launch heuristics
    (fused_deform_attn.py:721).  These kernels have fixed launch shapes; the
    flag is kept for callers that set it and has no effect."""
    global USE_HEURISTICS
    USE_HEURISTICS = bool(value)


def fused_knn_deform_self_attn_forward(pos, offsets, attn_weights, values, power, D=2, use_heuristics=True):
    """Forward only (fused_deform_attn.py:2387): out [B,N,H,C], nothing saved."""
    out, _, _ = fused_knn_deform_cross_attn_forward_save(pos, pos, offsets, attn_weights, values, power, D,
                                                         save_dist=False)
    return out


def fused_knn_deform_cross_attn_forward(query_pos, kv_pos, offsets, attn_weights, values, power, D=2,
                                        use_heuristics=True):
    """Forward only (fused_deform_attn.py:2460): out [B,Nq,H,C], nothing saved."""
    out, _, _ = fused_knn_deform_cross_attn_forward_save(query_pos, kv_pos, offsets, attn_weights, values, power,
                                                         D, save_dist=False)
    return out


def compute_softmax_weights(knn_dist_sq, power):
    """The reference's helper over saved squared distances
    (fused_deform_attn.py:3608): softmax_j(-max(power, 1e-6) * d2_j)."""
    p = torch.clamp(power, min=1e-6)
    return torch.softmax(-p * knn_dist_sq, dim=-1)
