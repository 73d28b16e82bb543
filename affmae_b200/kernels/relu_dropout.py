"""ReLU followed by dropout in one pass (the decoder feed-forward network's
``dropout3(relu(linear1(x)))``, reference src/layers/decoder.py:138-141).

``relu_dropout(x, p, training)`` equals ``F.dropout(F.relu(x), p, training)``
in distribution: the mask is a counter-based function of (seed, element
index) with the seed drawn from the CPU generator (so it follows
``torch.manual_seed``), and the backward recomputes nothing: the gradient
passes where the output is positive.  No mask tensor is written.
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from .. import _native as nat


class ReluDropoutFunction(Function):
    @staticmethod
    def forward(ctx, x, p):
        nat.require_cuda(x)
        xc = x.contiguous()
        seed = int(torch.randint(0, 2 ** 31 - 1, (1,)).item()) if p > 0 else 0
        y = torch.empty_like(xc)
        nat.call("affb_relu_dropout_fwd", nat.ptr(xc), nat.dcode(xc), xc.numel(), float(p), seed, nat.ptr(y),
                 nat.stream(x.device))
        ctx.save_for_backward(y)
        ctx.p = float(p)
        return y

    @staticmethod
    def backward(ctx, g):
        (y,) = ctx.saved_tensors
        gc = g.to(y.dtype).contiguous()
        dx = torch.empty_like(y)
        nat.call("affb_relu_dropout_bwd", nat.ptr(gc), nat.ptr(y), nat.dcode(y), y.numel(), ctx.p, nat.ptr(dx),
                 nat.stream(y.device))
        return dx, None


def relu_dropout(x: torch.Tensor, p: float, training: bool = True) -> torch.Tensor:
    return ReluDropoutFunction.apply(x, p if training else 0.0)
