"""CPU oracle: a restatement of the reference's algorithms for the hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this package; it is
used by ``tests/``, by ``__graft_entry__.smoke()`` as the checker, and by
``bench.py`` for the timed CPU baseline (``cpu_baseline`` and the
``--impl reference`` arm).

Each function cites the reference file:line it restates.  The restatement is
pinned against the reference's own Triton kernels, executed on the CPU under
``TRITON_INTERPRET=1`` at small shapes; the resulting golden vectors live in
``tests/golden/`` together with the script that generated them.
"""
from .ops import (  # noqa: F401
    knn,
    nbhd_attn_fwd,
    nbhd_attn_bwd,
    nbhd_attn_formula,
    nbhd_blank_grads,
    weighted_features_fwd,
    weighted_features_bwd,
    deform_knn_fwd,
    deform_knn_bwd,
    deform_nbidx_fwd,
    deform_nbidx_bwd,
    msdetrpc_fwd,
    msdetrpc_bwd,
    mssample_fwd,
    mssample_bwd,
    pos_bias_fwd,
    pos_bias_bwd,
)
