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
