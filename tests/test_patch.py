"""patch_reference() rebinds the reference's operator names (host logic, no GPU)."""
import sys
import types

from affmae_b200 import patch
import importlib
knn, local_attn, weighted_features = (importlib.import_module(f"affmae_b200.kernels.{n}") for n in ("knn", "local_attn", "weighted_features"))


def _mod(name, **attrs):
    m = types.ModuleType(name)
    for k, v in attrs.items():
        setattr(m, k, v)
    sys.modules[name] = m
    return m


def test_patch_reference_rebinds_kernel_and_layer_names():
    old = lambda *a: None  # noqa: E731
    names = ["fakesrc", "fakesrc.layers", "fakesrc.layers.kernels", "fakesrc.layers.kernels.knn",
             "fakesrc.layers.kernels.local_attn", "fakesrc.layers.attention", "fakesrc.layers.aff"]
    try:
        _mod("fakesrc"); _mod("fakesrc.layers"); _mod("fakesrc.layers.kernels")
        kk = _mod("fakesrc.layers.kernels.knn", knn=old, knn_forward=old, KNNFunction=old)
        la = _mod("fakesrc.layers.kernels.local_attn", FlashLocalAttentionFunction=old)
        att = _mod("fakesrc.layers.attention", triton_knn=old, FlashLocalAttentionFunction=old)
        aff = _mod("fakesrc.layers.aff", triton_knn=old, weighted_features=old, unrelated=old)
        done = patch.patch_reference("fakesrc")
        assert kk.knn is knn.knn and kk.knn_forward is knn.knn_forward and kk.KNNFunction is knn.KNNFunction
        assert la.FlashLocalAttentionFunction is local_attn.FlashLocalAttentionFunction
        assert att.triton_knn is knn.knn
        assert att.FlashLocalAttentionFunction is local_attn.FlashLocalAttentionFunction
        assert aff.weighted_features is weighted_features.weighted_features
        assert aff.unrelated is old
        assert len(done) >= 7
    finally:
        for n in names:
            sys.modules.pop(n, None)


def test_patch_reference_on_the_real_reference_tree():
    """patch_reference() on the reference's own modules (imported from the
    checkout named by AFFMAE_REFERENCE, with the same stubs as the fixture
    generators: the GPU-driver query of kernels/util.py and the unused
    pykeops / timm / fvcore imports): every operator name the layer modules
    use is rebound to this package, and the modules' classes are untouched."""
    import os
    import pytest
    root = os.environ.get("AFFMAE_REFERENCE")
    if not root:
        pytest.skip("AFFMAE_REFERENCE (a checkout of the reference) is not set")
    sys.path.insert(0, str(__import__("pathlib").Path(__file__).resolve().parent / "golden"))
    saved = {k: v for k, v in sys.modules.items() if k == "src" or k.startswith("src.")}
    try:
        from make_module_golden import load_attention
        import importlib
        load_attention(root)
        att = importlib.import_module("src.layers.attention")
        aff = importlib.import_module("src.layers.aff")
        done = patch.patch_reference("src")
        from affmae_b200.kernels import fused_deform_attn, msdetrpc
        assert att.FlashLocalAttentionFunction is local_attn.FlashLocalAttentionFunction
        assert att.launch_flash_nbhood_attn_fwd is local_attn.launch_flash_nbhood_attn_fwd
        assert att.fused_knn_deformable_cross_attention is fused_deform_attn.fused_knn_deformable_cross_attention
        assert att.fused_knn_deformable_self_attention is fused_deform_attn.fused_knn_deformable_self_attention
        assert att.fused_deformable_attention is fused_deform_attn.fused_deformable_attention
        assert att.MSDETRPCFunction is msdetrpc.MSDETRPCFunction
        assert att.triton_knn is knn.knn
        assert aff.triton_knn is knn.knn and aff.weighted_features is weighted_features.weighted_features
        kmod = importlib.import_module("src.layers.kernels.local_attn")
        assert kmod.FlashLocalAttentionFunction is local_attn.FlashLocalAttentionFunction
        assert att.ClusterAttention.__module__ == "src.layers.attention"
        assert len(done) >= 10
    finally:
        for k in [k for k in sys.modules if k == "src" or k.startswith("src.")]:
            del sys.modules[k]
        sys.modules.update(saved)
