"""The hot-path operators registered with the PyTorch dispatcher (namespace
``affb200``), on top of the same C ABI the ``kernels`` package calls.

The reference's operators are plain Python functions around Triton launches,
invisible to the dispatcher.  Registering them as custom ops gives every
operator a schema (``torch.ops.affb200.<name>``), a fake (meta) implementation
for shape propagation under FakeTensor / ``torch.compile`` tracing, and, for
the differentiable ones, an autograd formula that calls the backward op:

  knn                     knn(query, ref, k) -> int64 [B,M,k]  (src/layers/kernels/knn.py:1615)
  nbhd_attn_fwd / _bwd    FlashLocalAttentionFunction (local_attn.py:843-936)
  weighted_features_fwd / _bwd
                          WeightedFeaturesFunction (weighted_features.py:401-429)
  deform_cross_fwd / _bwd FusedKNNDeformCrossAttnFunction (fused_deform_attn.py:4020-4056)

Optional tensors are passed as ``None``; optional gradients come back as
empty tensors (a custom op returns tensors only).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor
from torch.library import custom_op

from .kernels import fused_deform_attn as _fd
from .kernels import knn as _knn
from .kernels import local_attn as _la
from .kernels import weighted_features as _wf

_EMPTY = (0,)


def _none_if_empty(t: Optional[Tensor]) -> Optional[Tensor]:
    return None if t is None or t.numel() == 0 else t


# ------------------------------------------------------------------- KNN --
@custom_op("affb200::knn", mutates_args=())
def knn(query: Tensor, ref: Tensor, k: int) -> Tensor:
    D = query.shape[-1]
    _knn._check(query, ref, k, D)
    return _knn._knn_int64(query, ref, k, D)


@knn.register_fake
def _(query, ref, k):
    return query.new_empty((query.shape[0], query.shape[1], k), dtype=torch.int64)


# ------------------------------------------------ neighbourhood attention --
@custom_op("affb200::nbhd_attn_fwd", mutates_args=())
def nbhd_attn_fwd(q: Tensor, k: Tensor, v: Tensor, member_idx: Tensor, bias: Optional[Tensor],
                  mask: Optional[Tensor], blank_k: Optional[Tensor], blank_v: Optional[Tensor],
                  scale: float) -> tuple[Tensor, Tensor]:
    return _la.launch_flash_nbhood_attn_fwd(q, k, v, member_idx, scale, bias=bias, mask=mask, blank_k=blank_k,
                                            blank_v=blank_v)


@nbhd_attn_fwd.register_fake
def _(q, k, v, member_idx, bias, mask, blank_k, blank_v, scale):
    B, H, N, _ = q.shape
    return torch.empty_like(q), q.new_empty((B, H, N), dtype=torch.float32)


@custom_op("affb200::nbhd_attn_bwd", mutates_args=())
def nbhd_attn_bwd(q: Tensor, k: Tensor, v: Tensor, member_idx: Tensor, scale: float, o: Tensor, lse: Tensor,
                  dout: Tensor, bias: Optional[Tensor], mask: Optional[Tensor], blank_k: Optional[Tensor],
                  blank_v: Optional[Tensor]) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    dq, dk, dv, dbias, dbk, dbv = _la.launch_flash_nbhood_attn_bwd(
        q, k, v, member_idx, scale, o, lse, dout, bias=bias, mask=mask, blank_k=blank_k, blank_v=blank_v)
    e = q.new_empty(_EMPTY)
    return dq, dk, dv, (dbias if dbias is not None else e), (dbk if dbk is not None else e), \
        (dbv if dbv is not None else e)


@nbhd_attn_bwd.register_fake
def _(q, k, v, member_idx, scale, o, lse, dout, bias, mask, blank_k, blank_v):
    e = q.new_empty(_EMPTY)
    return (torch.empty_like(q), torch.empty_like(q), torch.empty_like(q),
            torch.empty_like(bias) if bias is not None else e,
            torch.empty_like(blank_k) if blank_k is not None else e,
            torch.empty_like(blank_v) if blank_v is not None else e)


def _attn_setup(ctx, inputs, output):
    q, k, v, member_idx, bias, mask, blank_k, blank_v, scale = inputs
    o, lse = output
    ctx.save_for_backward(q, k, v, member_idx, bias, mask, blank_k, blank_v, o, lse)
    ctx.scale = scale


def _attn_backward(ctx, grad_o, grad_lse):
    q, k, v, member_idx, bias, mask, blank_k, blank_v, o, lse = ctx.saved_tensors
    dq, dk, dv, dbias, dbk, dbv = nbhd_attn_bwd(q, k, v, member_idx, ctx.scale, o, lse, grad_o.contiguous(),
                                                bias, mask, blank_k, blank_v)
    return dq, dk, dv, None, _none_if_empty(dbias), None, _none_if_empty(dbk), _none_if_empty(dbv), None


nbhd_attn_fwd.register_autograd(_attn_backward, setup_context=_attn_setup)


# ------------------------------------------------------ weighted features --
@custom_op("affb200::weighted_features_fwd", mutates_args=())
def weighted_features_fwd(weights: Tensor, feat: Tensor, nbhd_idx: Tensor) -> Tensor:
    return _wf.weighted_features_fwd(weights, feat, nbhd_idx)


@weighted_features_fwd.register_fake
def _(weights, feat, nbhd_idx):
    B, No, _, IC = weights.shape
    return feat.new_empty((B, No, IC, feat.shape[-1]))


@custom_op("affb200::weighted_features_bwd", mutates_args=())
def weighted_features_bwd(dout: Tensor, weights: Tensor, feat: Tensor, nbhd_idx: Tensor) -> tuple[Tensor, Tensor]:
    return _wf.weighted_features_bwd(dout, weights, feat, nbhd_idx)


@weighted_features_bwd.register_fake
def _(dout, weights, feat, nbhd_idx):
    return weights.new_empty(weights.shape, dtype=feat.dtype), torch.empty_like(feat)


def _wf_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _wf_backward(ctx, grad):
    weights, feat, nbhd_idx = ctx.saved_tensors
    dw, dfeat = weighted_features_bwd(grad.contiguous(), weights, feat, nbhd_idx)
    return dw.to(weights.dtype), dfeat.to(feat.dtype), None


weighted_features_fwd.register_autograd(_wf_backward, setup_context=_wf_setup)


# ----------------------------------------- fused KNN deformable attention --
@custom_op("affb200::deform_cross_fwd", mutates_args=())
def deform_cross_fwd(query_pos: Tensor, kv_pos: Tensor, offsets: Tensor, attn_weights: Tensor, values: Tensor,
                     power: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    return _fd.fused_knn_deform_cross_attn_forward_save(query_pos, kv_pos, offsets, attn_weights, values, power)


@deform_cross_fwd.register_fake
def _(query_pos, kv_pos, offsets, attn_weights, values, power):
    B, Nq, H, K, _ = offsets.shape
    return (values.new_empty((B, Nq, H, values.shape[-1])),
            offsets.new_empty((B, Nq, H, K, 4), dtype=torch.int32),
            offsets.new_empty((B, Nq, H, K, 4), dtype=torch.float32))


@custom_op("affb200::deform_cross_bwd", mutates_args=())
def deform_cross_bwd(dout: Tensor, query_pos: Tensor, kv_pos: Tensor, offsets: Tensor, attn_weights: Tensor,
                     values: Tensor, power: Tensor, knn_idx: Tensor, knn_d2: Tensor
                     ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    dq, dkv, doff, daw, dval, dpow = _fd.fused_knn_deform_cross_attn_backward(
        dout, query_pos, kv_pos, offsets, attn_weights, values, power, knn_idx, knn_d2)
    return dq, dkv, doff, daw, dval, dpow.reshape(power.shape).to(power.dtype)


@deform_cross_bwd.register_fake
def _(dout, query_pos, kv_pos, offsets, attn_weights, values, power, knn_idx, knn_d2):
    return (torch.empty_like(query_pos), torch.empty_like(kv_pos), torch.empty_like(offsets),
            torch.empty_like(attn_weights), torch.empty_like(values), torch.empty_like(power))


def _deform_setup(ctx, inputs, output):
    _, knn_idx, knn_d2 = output
    ctx.save_for_backward(*inputs, knn_idx, knn_d2)


def _deform_backward(ctx, grad_out, grad_idx, grad_d2):
    query_pos, kv_pos, offsets, attn_weights, values, power, knn_idx, knn_d2 = ctx.saved_tensors
    return deform_cross_bwd(grad_out.contiguous(), query_pos, kv_pos, offsets, attn_weights, values, power,
                            knn_idx, knn_d2)


deform_cross_fwd.register_autograd(_deform_backward, setup_context=_deform_setup)
