"""Rebind the reference's kernel operators to the affmae_b200 implementations.

``patch_reference()`` walks the already-imported modules of an AFFMAE source
tree (``src.layers.kernels.*``, ``src.layers.attention``, ``src.layers.aff``,
``src.utils.geometry``) and replaces every public operator name with the
affmae_b200 object of the same name, so the reference's modules
(``ClusterAttention``, ``Deformable{Self,Cross}Attention``, ``BasicLayer``,
``ClusterMerging``) call the sm_100a kernels without any code change.
"""
from __future__ import annotations

import importlib
import sys

_k = lambda n: importlib.import_module(f"{__package__}.kernels.{n}")  # noqa: E731
fused_deform_attn, knn, local_attn, msdetrpc, mssample, weighted_features, weighted_gather = (
    _k(n) for n in ("fused_deform_attn", "knn", "local_attn", "msdetrpc", "mssample",
                    "weighted_features", "weighted_gather"))

# reference module -> replacement module
_MODULES = {
    "knn": knn,
    "local_attn": local_attn,
    "weighted_features": weighted_features,
    "weighted_gather": weighted_gather,
    "fused_deform_attn": fused_deform_attn,
    "msdetrpc": msdetrpc,
    "mssample": mssample,
}

# names imported into the reference's layer modules (attention.py:11-18, aff.py:16-17)
_ALIASES = {
    "triton_knn": knn.knn,
    "knn": knn.knn,
    "knn_triton": knn.knn_triton,
    "FlashLocalAttentionFunction": local_attn.FlashLocalAttentionFunction,
    "launch_flash_nbhood_attn_fwd": local_attn.launch_flash_nbhood_attn_fwd,
    "launch_flash_nbhood_attn_bwd": local_attn.launch_flash_nbhood_attn_bwd,
    "weighted_features": weighted_features.weighted_features,
    "weighted_gather": weighted_gather.weighted_gather,
    "MSDETRPCFunction": msdetrpc.MSDETRPCFunction,
    "mssample": mssample.mssample,
    "fused_deformable_attention": fused_deform_attn.fused_deformable_attention,
    "fused_knn_deformable_self_attention": fused_deform_attn.fused_knn_deformable_self_attention,
    "fused_knn_deformable_cross_attention": fused_deform_attn.fused_knn_deformable_cross_attention,
}


def _public(mod):
    return {n: getattr(mod, n) for n in dir(mod) if not n.startswith("_")}


def patch_reference(prefix: str = "src") -> list[str]:
    """Patch every imported module under ``prefix``; returns the patched names."""
    patched = []
    for name, mod in list(sys.modules.items()):
        if mod is None or not (name == prefix or name.startswith(prefix + ".")):
            continue
        leaf = name.rsplit(".", 1)[-1]
        repl = _MODULES.get(leaf) if ".kernels." in name or name.endswith(".kernels." + leaf) else None
        if repl is not None:
            for attr, obj in _public(repl).items():
                if hasattr(mod, attr) and callable(obj):
                    setattr(mod, attr, obj)
                    patched.append(f"{name}.{attr}")
        for attr, obj in _ALIASES.items():
            if attr in vars(mod) and vars(mod)[attr] is not obj and callable(vars(mod)[attr]):
                if repl is None or not hasattr(repl, attr):
                    setattr(mod, attr, obj)
                    patched.append(f"{name}.{attr}")
    return patched
