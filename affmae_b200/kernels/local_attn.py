"""Neighbourhood (cluster) flash attention (mirrors src/layers/kernels/local_attn.py).

Public API as in the reference: ``launch_flash_nbhood_attn_fwd``
(local_attn.py:609), ``launch_flash_nbhood_attn_bwd`` (:711) and
``FlashLocalAttentionFunction`` (:843), same arguments, shapes and returns.

Differences that are deliberate:
  * inputs keep their dtype (fp32, fp16 or bf16); the reference casts to fp16
    under autocast and rounds O through fp16 even for fp32 inputs;
  * a [B,1,N,M] mask is read per batch element instead of being expanded to
    [B,H,N,M];
  * O, dQ, dK and dV are written directly, without zero-initialised fp32 buffers.
"""
from __future__ import annotations

import torch
from torch.autograd import Function
from torch.amp import custom_fwd, custom_bwd

from .. import _native as nat


def _prep_mask(mask, B, H, N, M):
    if mask is None or mask.numel() == 0:
        return None, 1
    if mask.dim() == 3:
        mask = mask.unsqueeze(1)
    assert mask.shape[0] == B and mask.shape[2] == N and mask.shape[3] == M and mask.shape[1] in (1, H), \
        f"mask must have shape [B, 1 or H, N, M] (mask shape: {tuple(mask.shape)})"
    if mask.dtype == torch.bool:
        m = mask.contiguous().view(torch.uint8)
    else:
        m = (mask > 0).to(torch.uint8).contiguous()
    return m, mask.shape[1]


def launch_flash_nbhood_attn_fwd(q, k, v, member_index, sm_scale, bias=None, mask=None,
                                 blank_k=None, blank_v=None, exp2=False, return_plan=False):
    """Forward: returns (o [B,H,N,D] in q.dtype, lse [B,H,N] fp32).

    ``return_plan=True`` also returns the tiles' cluster unions the forward
    built (a byte tensor, or None off the tensor-core path), which
    ``launch_flash_nbhood_attn_bwd(..., plan=...)`` reuses for the same lists."""
    assert q.shape == k.shape and k.shape == v.shape, "q, k, v must have the same shape"
    assert q.dim() == 4, "q, k, v must have 4 dimensions"
    assert q.shape[-1] % 8 == 0, "head_dim must be a multiple of 8"
    B, H, N, D = q.shape
    M = member_index.shape[-1]
    assert M % 8 == 0, "neighbor_size must be a multiple of 8"
    nat.require_cuda(q, k, v, member_index)
    dt = q.dtype
    q = q.contiguous()
    k = k.to(dt).contiguous()
    v = v.to(dt).contiguous()
    mi = member_index.to(torch.int32).contiguous()
    if bias is not None and bias.numel() > 0:
        assert bias.shape == (B, H, N, M), "bias must have shape [batch_size, n_heads, seq_len, neighbor_size]"
        bias = bias.to(dt).contiguous()
    else:
        bias = None
    if blank_k is not None and blank_v is not None and blank_k.numel() > 0 and blank_v.numel() > 0:
        assert blank_k.shape == (H, D), "blank_k must have shape [n_heads, head_dim]"
        assert blank_v.shape == (H, D), "blank_v must have shape [n_heads, head_dim]"
        blank_k = blank_k.to(dt).contiguous()
        blank_v = blank_v.to(dt).contiguous()
    else:
        blank_k = blank_v = None
    m8, mh = _prep_mask(mask, B, H, N, M)
    o = torch.empty_like(q)
    lse = torch.empty((B, H, N), device=q.device, dtype=torch.float32)
    plan = None
    if return_plan:
        pb = int(nat.lib().affb_nbhd_tile_plan_bytes(nat.dcode(q), B, N, D, M))
        plan = torch.empty((pb,), device=q.device, dtype=torch.uint8) if pb > 0 else None
    if plan is not None:
        nat.call("affb_nbhd_attn_fwd_plan", nat.ptr(q), nat.ptr(k), nat.ptr(v), nat.ptr(mi), nat.ptr(bias),
                 nat.ptr(m8), mh, nat.ptr(blank_k), nat.ptr(blank_v), nat.dcode(q), B, H, N, D, M,
                 float(sm_scale), nat.ptr(o), nat.ptr(lse), nat.ptr(plan), plan.numel(), nat.stream(q.device))
    else:
        nat.call("affb_nbhd_attn_fwd", nat.ptr(q), nat.ptr(k), nat.ptr(v), nat.ptr(mi), nat.ptr(bias),
                 nat.ptr(m8), mh, nat.ptr(blank_k), nat.ptr(blank_v), nat.dcode(q), B, H, N, D, M,
                 float(sm_scale), nat.ptr(o), nat.ptr(lse), nat.stream(q.device))
    if return_plan:
        return o, lse, plan
    return o, lse


def launch_flash_nbhood_attn_bwd(q, k, v, member_index, sm_scale, o, lse, do, bias=None,
                                 mask=None, blank_k=None, blank_v=None, exp2=False, plan=None):
    """Backward: returns (dq, dk, dv, dbias | None, dblank_k | None, dblank_v | None).
    ``plan``: the forward's tile plan for the same lists and mask (optional)."""
    assert not exp2, "EXP2 is not supported in backward pass"
    assert q.shape == k.shape == v.shape == o.shape == do.shape
    assert q.dim() == 4
    B, H, N, D = q.shape
    M = member_index.shape[-1]
    dt = q.dtype
    nat.require_cuda(q, k, v, o, do, lse, member_index)
    q = q.contiguous()
    k = k.to(dt).contiguous()
    v = v.to(dt).contiguous()
    o = o.to(dt).contiguous()
    do = do.to(dt).contiguous()
    lse = lse.to(torch.float32).contiguous()
    mi = member_index.to(torch.int32).contiguous()
    has_bias = bias is not None and bias.numel() > 0
    if has_bias:
        assert bias.shape == (B, H, N, M)
        bias = bias.to(dt).contiguous()
    else:
        bias = None
    has_blank = blank_k is not None and blank_v is not None
    if has_blank:
        assert blank_k.shape == (H, D) and blank_v.shape == (H, D)
        blank_k = blank_k.to(dt).contiguous()
        blank_v = blank_v.to(dt).contiguous()
    m8, mh = _prep_mask(mask, B, H, N, M)
    dev = q.device
    dq = torch.empty_like(q)
    dk = torch.empty_like(q)
    dv = torch.empty_like(q)
    dbias = torch.empty((B, H, N, M), device=dev, dtype=dt) if has_bias else None
    dbk = torch.zeros((H, D), device=dev, dtype=torch.float32) if has_blank else None
    dbv = torch.zeros((H, D), device=dev, dtype=torch.float32) if has_blank else None
    wsb = int(nat.lib().affb_nbhd_attn_bwd_workspace_bytes(nat.dcode(q), B, H, N, D, M))
    ws = torch.empty((max(wsb, 1),), device=dev, dtype=torch.uint8)
    common = [nat.ptr(q), nat.ptr(k), nat.ptr(v), nat.ptr(o), nat.ptr(do),
              nat.ptr(lse), nat.ptr(mi), nat.ptr(bias), nat.ptr(m8), mh,
              nat.ptr(blank_k) if has_blank else None, nat.ptr(blank_v) if has_blank else None,
              nat.dcode(q), B, H, N, D, M, float(sm_scale), nat.ptr(dq), nat.ptr(dk),
              nat.ptr(dv), nat.ptr(dbias), nat.ptr(dbk), nat.ptr(dbv)]
    if plan is not None:
        nat.call("affb_nbhd_attn_bwd_plan", *common, nat.ptr(plan), plan.numel(), nat.ptr(ws), wsb, nat.stream(dev))
    else:
        nat.call("affb_nbhd_attn_bwd", *common, nat.ptr(ws), wsb, nat.stream(dev))
    if has_blank:
        dbk = dbk.to(dt)
        dbv = dbv.to(dt)
    return dq, dk, dv, dbias, dbk, dbv


class FlashLocalAttentionFunction(Function):
    """Neighbourhood attention with optional bias, mask and per-head blank token.

    forward(Q, K, V [B,H,N,D], member_idx [B,N,M], bias [B,H,N,M] | None,
            mask [B,1|H,N,M] | None, blank_k, blank_v [H,D] | None, softmax_scale)
    backward returns (dQ, dK, dV, None, dbias, None, dblank_k, dblank_v, None).
    """

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, Q, K, V, member_idx, bias, mask, blank_k, blank_v, softmax_scale):
        has_bias = bias is not None and bias.numel() > 0
        has_blank = blank_k is not None and blank_v is not None
        has_mask = mask is not None and mask.numel() > 0
        member_idx = member_idx.to(torch.int32).contiguous()
        out, lse, plan = launch_flash_nbhood_attn_fwd(
            Q, K, V, member_idx, softmax_scale, bias=bias if has_bias else None,
            mask=mask if has_mask else None, blank_k=blank_k if has_blank else None,
            blank_v=blank_v if has_blank else None, return_plan=True)
        ctx.save_for_backward(Q, K, V, member_idx, bias if has_bias else None,
                              mask if has_mask else None, blank_k if has_blank else None,
                              blank_v if has_blank else None, out, lse, plan)
        ctx.scale = softmax_scale
        ctx.flags = (has_bias, has_blank, has_mask)
        return out

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, grad_output):
        Q, K, V, member_idx, bias, mask, blank_k, blank_v, out, lse, plan = ctx.saved_tensors
        has_bias, has_blank, has_mask = ctx.flags
        dq, dk, dv, dbias, dbk, dbv = launch_flash_nbhood_attn_bwd(
            Q, K, V, member_idx, ctx.scale, out, lse, grad_output,
            bias=bias if has_bias else None, mask=mask if has_mask else None,
            blank_k=blank_k if has_blank else None, blank_v=blank_v if has_blank else None, plan=plan)
        dq, dk, dv = dq.to(Q.dtype), dk.to(K.dtype), dv.to(V.dtype)
        if has_bias:
            dbias = dbias.to(bias.dtype)
        if has_blank:
            dbk, dbv = dbk.to(blank_k.dtype), dbv.to(blank_v.dtype)
        else:
            dbk = dbv = None
        return dq, dk, dv, None, dbias, None, dbk, dbv, None
