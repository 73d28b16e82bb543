"""Drop-in replacements for the reference's ``src/layers/kernels`` operators.

Every module here mirrors the reference module of the same name (same public
functions, ``torch.autograd.Function`` classes, argument order, shapes and
return tuples) and runs on the sm_100a kernels of ``libaffmae_b200.so``.
"""
from .mssample import mssample, MSSampleFunction
from .local_attn import FlashLocalAttentionFunction
from .msdetrpc import MSDETRPCFunction
from .fused_deform_attn import fused_deformable_attention, FusedDeformAttnFunction

__all__ = [
    "mssample",
    "MSSampleFunction",
    "FlashLocalAttentionFunction",
    "MSDETRPCFunction",
    "fused_deformable_attention",
    "FusedDeformAttnFunction",
]
