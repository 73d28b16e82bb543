"""Elementwise fusions of the model around the operators.

ReLU + dropout in one pass (affb_relu_dropout_fwd / _bwd) against the
PyTorch formula relu(x) * keep / (1 - p), with the keep mask taken from the
host copy of the same counter-based stream (affb_dropout_keep_mask); the
sine position embedding (affb_sine_embed) against the PyTorch sequence of
the reference's PositionEmbeddingSine (decoder.py:16-62)."""
import ctypes

import numpy as np
import pytest
import torch

from affmae_b200 import _native as nat


def _keep(seed, p, n):
    keep = np.empty(n, dtype=np.uint8)
    nat.call("affb_dropout_keep_mask", seed, p, 0, n, keep.ctypes.data_as(ctypes.c_void_p))
    return torch.from_numpy(keep.astype(bool))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n", [4096 * 8, 1000 * 7 + 3])   # vector and scalar paths
@pytest.mark.parametrize("p", [0.0, 0.1, 0.5])
def test_relu_dropout_matches_formula(cuda, dtype, n, p):
    g = torch.Generator().manual_seed(n)
    x = torch.randn(n, generator=g).to(cuda, dtype)
    dy = torch.randn(n, generator=g).to(cuda, dtype)
    seed = 1234567
    y = torch.empty_like(x)
    nat.call("affb_relu_dropout_fwd", nat.ptr(x), nat.dcode(x), n, p, seed, nat.ptr(y), nat.stream(x.device))
    keep = _keep(seed, p, n).to(cuda) if p > 0 else torch.ones(n, dtype=torch.bool, device=cuda)
    scale = 1.0 / (1.0 - p)
    ref = torch.where(keep & (x.float() > 0), x.float() * torch.tensor(scale, dtype=torch.float32), 0.0).to(dtype)
    assert torch.equal(y, ref)
    if p > 0:
        assert abs(keep.float().mean().item() - (1 - p)) < 0.02
    dx = torch.empty_like(x)
    nat.call("affb_relu_dropout_bwd", nat.ptr(dy), nat.ptr(y), nat.dcode(y), n, p, nat.ptr(dx),
             nat.stream(x.device))
    dref = torch.where(y.float() > 0, dy.float() * torch.tensor(scale, dtype=torch.float32), 0.0).to(dtype)
    assert torch.equal(dx, dref)


@pytest.mark.gpu
def test_relu_dropout_function_autograd(cuda):
    """The autograd Function: p = 0 is exactly F.relu with its gradient; in
    training the surviving fraction is 1 - p and gradients pass where the
    output is positive."""
    from affmae_b200.kernels.relu_dropout import relu_dropout
    x = torch.randn(64, 768, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    y = relu_dropout(x, 0.0)
    y.backward(torch.ones_like(y))
    x2 = x.detach().clone().requires_grad_(True)
    torch.nn.functional.relu(x2).backward(torch.ones_like(x2))
    assert torch.equal(y, torch.relu(x.detach())) and torch.equal(x.grad, x2.grad)
    x.grad = None
    torch.manual_seed(0)
    y = relu_dropout(x, 0.1)
    pos = x.detach() > 0
    kept = (y != 0) & pos
    assert abs(kept.sum().item() / pos.sum().item() - 0.9) < 0.02
    y.sum().backward()
    assert torch.equal(x.grad != 0, y != 0)


def _sine_torch(pos, dim):
    """The reference's PositionEmbeddingSine(dim / 2, normalize=True) sequence
    (decoder.py:34-56) in PyTorch ops."""
    import math
    half = dim // 2
    x = pos[..., 0] / (pos[..., 0].max() + 1e-6) * (2 * math.pi)
    y = pos[..., 1] / (pos[..., 1].max() + 1e-6) * (2 * math.pi)
    dim_t = torch.arange(half, dtype=torch.float32, device=pos.device)
    dim_t = 10000 ** (2 * dim_t.div(2, rounding_mode="floor") / half)
    px, py = x[..., None] / dim_t, y[..., None] / dim_t
    px = torch.cat((px[..., 0::2].sin(), px[..., 1::2].cos()), -1)
    py = torch.cat((py[..., 0::2].sin(), py[..., 1::2].cos()), -1)
    return torch.cat((px, py), -1)


@pytest.mark.gpu
@pytest.mark.parametrize("dim", [64, 384])
def test_sine_embedding_kernel_matches_torch(cuda, dim):
    from affmae_b200.mae import sine_embedding
    g = torch.Generator().manual_seed(dim)
    pos = (torch.rand((3, 517, 2), generator=g) * 255).round().to(cuda)
    ref = _sine_torch(pos, dim)
    out = sine_embedding(pos, dim)
    assert (out - ref).abs().max().item() < 1e-6
    assert (sine_embedding(pos, dim, torch.bfloat16).float() - ref).abs().max().item() < 4e-3  # half a bf16 ulp
