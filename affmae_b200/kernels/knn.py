"""K-nearest neighbours over 2/3/4-D points (mirrors src/layers/kernels/knn.py).

Public API as in the reference: ``knn`` (knn.py:1615), ``knn_triton``
(:1585), ``KNNFunction`` (:1543) and ``knn_forward`` (:1368).  One exact
rule serves every K (the reference switches to cdist+topk for K > 8): fp32
squared distances with separately rounded products and sums, ascending, ties
broken by the lower index.  Large 2-D searches (GRID_MIN_POINTS reference
points, GRID_MIN_PAIRS query-point pairs) go through a uniform grid (same
result as the brute-force scan, which serves 3-D / 4-D and small searches).
"""
from __future__ import annotations

import torch
from torch.autograd import Function
from torch.amp import custom_fwd

from .. import _native as nat


def _check(query, ref, k, D):
    nat.require_cuda(query, ref)
    assert query.dim() == 3 and ref.dim() == 3, "Expected 3D tensors [B, N, D]"
    assert query.shape[0] == ref.shape[0], "Batch sizes must match"
    assert query.shape[2] == ref.shape[2] == D, \
        f"Expected D={D}, got query D={query.shape[2]}, ref D={ref.shape[2]}"
    assert D in [2, 3, 4], f"D must be 2, 3, or 4, got {D}"
    assert k <= ref.shape[1], f"k={k} exceeds number of reference points N={ref.shape[1]}"


GRID_MIN_POINTS = 128     # 2-D searches use the grid when the reference set has at least
GRID_MIN_PAIRS = 1 << 21  # this many points and queries x points reaches this (else the
                          # brute-force scan is cheaper than building the grid)


def _knn_int64(query, ref, k, D):
    if query.dtype != ref.dtype or query.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        query, ref = query.float(), ref.float()
    query = query.contiguous()
    ref = ref.contiguous()
    B, M, _ = query.shape
    N = ref.shape[1]
    out = torch.empty((B, M, k), dtype=torch.int64, device=query.device)
    if D == 2 and N >= GRID_MIN_POINTS and M * N >= GRID_MIN_PAIRS:
        # fp32 copies are exact for fp16 / bf16 points, so distances are unchanged
        q32, r32 = nat.f32(query), nat.f32(ref)
        wsb = int(nat.lib().affb_knn2d_workspace_bytes(B, N))
        ws = torch.empty((wsb,), dtype=torch.uint8, device=query.device)
        nat.call("affb_knn2d", nat.ptr(q32), nat.ptr(r32), B, M, N, int(k), nat.ptr(out), nat.ptr(ws), wsb,
                 nat.stream(query.device))
        return out
    nat.call("affb_knn", nat.ptr(query), nat.ptr(ref), nat.dcode(query), B, M, N, D, int(k),
             nat.ptr(out), nat.stream(query.device))
    return out


def knn_forward(query, ref, k, D=2, use_v2=True, use_heuristic=True):
    """Indices [B, M, k] (int32) of the k nearest ``ref`` points of each query."""
    _check(query, ref, k, D)
    return _knn_int64(query, ref, k, D).to(torch.int32)


class KNNFunction(Function):
    """Forward-only autograd Function (KNN indices carry no gradient)."""

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, query, ref, k, D=2):
        with torch.no_grad():
            q, r = query.detach(), ref.detach()
            _check(q, r, k, D)
            return _knn_int64(q, r, k, D)

    @staticmethod
    def backward(ctx, grad_output):
        return None, None, None, None


def knn_triton(query, ref, k, D=2):
    """Same contract as the reference's ``knn_triton``: int64 indices [B, M, k]."""
    return KNNFunction.apply(query, ref, k, D)


def knn(query, database, k, return_dist=False, D=None):
    """knn_keops-compatible entry point; optionally also returns squared distances."""
    if D is None:
        D = query.shape[-1]
    indices = knn_triton(query, database, k, D=D)
    if return_dist:
        B, M, K = indices.shape
        nbr = database.gather(dim=1, index=indices.view(B, M * K, 1).expand(-1, -1, D)).view(B, M, K, D)
        distances = ((query.unsqueeze(2) - nbr) ** 2).sum(dim=-1)
        return indices, distances
    return indices


def knn_pytorch_large(query, ref, k):
    """Same contract as the reference's cdist + topk path (knn.py:1312): int64
    indices [B, M, k] of the k nearest ``ref`` points, here from the exact
    kernel (ties by lower index; the reference's topk leaves their order open)."""
    D = query.shape[-1]
    _check(query, ref, k, D)
    return _knn_int64(query, ref, k, D)


def knn_large_k_fallback(query, ref, k):
    """The reference's large-K entry (knn.py:1336); the same exact kernel."""
    return knn_pytorch_large(query, ref, k)
