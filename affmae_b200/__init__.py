"""affmae_b200: B200 (sm_100a) kernels for AFFMAE's custom-kernel hot path.

``affmae_b200.kernels`` mirrors the reference's ``src/layers/kernels`` package
operator by operator; ``affmae_b200.patch.patch_reference()`` rebinds those
names inside an imported reference tree so its modules run on these kernels.
"""
from . import _native  # noqa: F401

__version__ = "0.1.0"
