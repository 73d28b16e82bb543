"""The operators as dispatcher-registered torch custom ops (``torch.ops.affb200``):
schemas and fake (meta) implementations on the CPU, equality with the
``kernels`` API and autograd through the registered backward on the GPU."""
import pytest
import torch

from conftest import rel_err


def test_ops_are_registered_with_schemas():
    import affmae_b200.ops  # noqa: F401
    for name in ("knn", "nbhd_attn_fwd", "nbhd_attn_bwd", "weighted_features_fwd", "weighted_features_bwd",
                 "deform_cross_fwd", "deform_cross_bwd"):
        op = getattr(torch.ops.affb200, name)
        assert "affb200::" + name in str(op.default._schema)


def test_fake_shapes_without_a_gpu():
    """Shape propagation needs no device: FakeTensor mode runs the fake impls."""
    import affmae_b200.ops  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        q = torch.empty((2, 4, 64, 32), dtype=torch.bfloat16)
        mi = torch.empty((2, 64, 48), dtype=torch.int32)
        bias = torch.empty((2, 4, 64, 48), dtype=torch.bfloat16)
        o, lse = torch.ops.affb200.nbhd_attn_fwd(q, q, q, mi, bias, None, None, None, 0.17)
        assert o.shape == q.shape and lse.shape == (2, 4, 64) and lse.dtype == torch.float32
        g = torch.ops.affb200.nbhd_attn_bwd(q, q, q, mi, 0.17, o, lse, o, bias, None, None, None)
        assert g[3].shape == bias.shape and g[4].numel() == 0
        idx = torch.ops.affb200.knn(torch.empty((2, 10, 2)), torch.empty((2, 30, 2)), 5)
        assert idx.shape == (2, 10, 5) and idx.dtype == torch.int64
        out = torch.ops.affb200.weighted_features_fwd(torch.empty((2, 7, 48, 4)), torch.empty((2, 30, 96)),
                                                      torch.empty((2, 7, 48), dtype=torch.int32))
        assert out.shape == (2, 7, 4, 96)


@pytest.mark.gpu
def test_ops_match_kernels_api_and_autograd(cuda):
    import affmae_b200.ops  # noqa: F401
    from affmae_b200.kernels.knn import knn
    from affmae_b200.kernels.local_attn import FlashLocalAttentionFunction
    from affmae_b200.workloads import nbhd_attention_inputs
    g = torch.Generator().manual_seed(0)
    p = (torch.rand((2, 500, 2), generator=g) * 30).to(cuda)
    assert torch.equal(torch.ops.affb200.knn(p, p, 16), knn(p, p, 16))
    inp = nbhd_attention_inputs(B=1, side=32, dtype=torch.bfloat16, seed=2, device=cuda)
    names = ("q", "k", "v", "bias", "blank_k", "blank_v")
    a = [inp[n].clone().requires_grad_() for n in names]
    b = [inp[n].clone().requires_grad_() for n in names]
    o1, _ = torch.ops.affb200.nbhd_attn_fwd(a[0], a[1], a[2], inp["member_idx"], a[3], None, a[4], a[5],
                                            inp["scale"])
    o2 = FlashLocalAttentionFunction.apply(b[0], b[1], b[2], inp["member_idx"], b[3], None, b[4], b[5],
                                           inp["scale"])
    assert torch.equal(o1, o2)
    o1.backward(inp["dout"])
    o2.backward(inp["dout"])
    for x, y in zip(a, b):
        assert rel_err(x.grad.float(), y.grad.float()) < 1e-6
