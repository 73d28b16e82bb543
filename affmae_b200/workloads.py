"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (the reference trains on EM image shards that are
not available here; these generators stand in for them).

  * ``nbhd_attention_inputs``: config 3 — neighbourhood attention over a
    0.5-masked 96x96 token grid, clusters of 8 tokens in space-filling-curve
    order, each token attending the members of its 6 nearest clusters (the
    neighbourhood construction of BasicLayer.forward, src/layers/aff.py:426-465),
    with a relative-position bias from a Linear(5 -> H) over the reference's
    relative-position table (src/utils/pos_embed.py:9-24, attention.py:110-124).
  * ``deform_inputs``: config 4 — one level of multi-scale deformable
    attention in level-0 token units.
  * ``knn_points``: config 2 — jittered 96x96 stride-4 lattice.

Curve order: tokens are clustered by the reference's own space-filling scan
of grid anchors (src/utils/geometry.py:170-319, restated bit-exactly in
``affmae_b200.mae.curve_clusters``).  ``order="morton"`` gives the Z-order
curve used by earlier benchmark lines, kept so both can be compared.
"""
from __future__ import annotations

import math

import torch

from .kernels.knn import knn
from .kernels.pos_bias import pos_bias_gather

REL_POS_WIDTH = 1024 // 8 - 1          # pos_embed.py:8
TABLE_WIDTH = 2 * REL_POS_WIDTH + 1   # 255


def relative_position_table() -> torch.Tensor:
    """[T*T, 5] = (dx, dy, r, dy/r, dx/r), zero where r = 0 (pos_embed.py:12-22)."""
    hs = torch.arange(TABLE_WIDTH).float() - REL_POS_WIDTH
    ys, xs = torch.meshgrid(hs, hs, indexing="ij")
    r = (ys ** 2 + xs ** 2) ** 0.5
    t = torch.stack([xs, ys, r, ys / r, xs / r], dim=2)
    t[~torch.isfinite(t)] = 0
    return t.reshape(-1, 5)


def _morton(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    def spread(v):
        v = v.long() & 0xFFFF
        v = (v | (v << 8)) & 0x00FF00FF
        v = (v | (v << 4)) & 0x0F0F0F0F
        v = (v | (v << 2)) & 0x33333333
        v = (v | (v << 1)) & 0x55555555
        return v
    return spread(x) | (spread(y) << 1)


def clustered_tokens(B: int, side: int, keep: float, seed: int, device,
                     order: str = "curve") -> torch.Tensor:
    """Positions [B, N, 2] (fp32 grid coordinates) of the kept tokens of a
    side x side grid, in cluster order.  N = round(side*side*keep).
    ``order``: "curve" = the reference's anchor scan (geometry.py:170-319),
    "morton" = Z-order."""
    g = torch.Generator().manual_seed(seed)
    n_all = side * side
    n = int(round(n_all * keep))
    ys, xs = torch.meshgrid(torch.arange(side), torch.arange(side), indexing="ij")
    grid = torch.stack([xs.reshape(-1), ys.reshape(-1)], -1)
    out = torch.empty((B, n, 2))
    for b in range(B):
        sel = torch.randperm(n_all, generator=g)[:n]
        out[b] = grid[sel].float()
    if order == "morton":
        for b in range(B):
            o = torch.argsort(_morton(out[b, :, 0].long(), out[b, :, 1].long()))
            out[b] = out[b][o]
        return out.to(device)
    if order != "curve":
        raise ValueError(f"unknown cluster order {order!r}")
    from .mae import curve_clusters   # the model module imports this one
    pos, _, _, _ = curve_clusters(out, 8, side, side)
    return pos.to(device)


def neighbourhoods(pos: torch.Tensor, cluster: int = 8, nbhd: int = 48):
    """member_idx [B,N,nbhd] int32 and pe_idx [B,N,nbhd] int64 as in BasicLayer.forward
    (aff.py:426-465): clusters of `cluster` consecutive tokens, KNN from each
    token to the cluster means, members of the nearest clusters."""
    B, N, _ = pos.shape
    k = math.ceil(N / cluster)
    assert N == k * cluster, "token count must be a multiple of the cluster size"
    nnc = min(int(round(nbhd / cluster)), k)
    means = pos.view(B, k, cluster, 2).mean(2)
    if pos.is_cuda:
        nearest = knn(pos, means, nnc)                               # [B,N,nnc]
    else:  # host-side input generation only (e.g. for the CPU timing arm)
        d = torch.cdist(pos.double(), means.double())
        nearest = torch.argsort(d, dim=-1, stable=True)[..., :nnc]
    member = (nearest[..., None] * cluster + torch.arange(cluster, device=pos.device)).reshape(B, N, nnc * cluster)
    bidx = torch.arange(B, device=pos.device)[:, None, None]
    pos_nb = pos[bidx, member]                                        # [B,N,M,2]
    rel = (pos_nb - (pos[:, :, None, :] - REL_POS_WIDTH)).clamp(0, TABLE_WIDTH - 1)
    pe_idx = (rel[..., 1] * TABLE_WIDTH + rel[..., 0]).long()
    return member.to(torch.int32).contiguous(), pe_idx


def nbhd_attention_inputs(B=32, side=96, keep=0.5, H=4, d=32, nbhd=48, dtype=torch.bfloat16,
                          seed=0, device="cuda", order="curve"):
    """Config 3 inputs: dict(q, k, v [B,H,N,d], member_idx [B,N,M] int32, bias [B,H,N,M],
    blank_k, blank_v [H,d], dout [B,H,N,d], scale)."""
    pos = clustered_tokens(B, side, keep, seed, device, order)
    member, pe_idx = neighbourhoods(pos, 8, nbhd)
    N = pos.shape[1]
    g = torch.Generator(device="cpu").manual_seed(seed + 1)

    def rnd(*shape, std=1.0):
        return (torch.randn(shape, generator=g) * std).to(device=device, dtype=dtype)

    table = relative_position_table()
    w = torch.randn((H, 5), generator=g) * 0.02
    bvec = torch.randn((H,), generator=g) * 0.02
    pe_table = (table @ w.T + bvec).to(device=device, dtype=dtype)   # Linear(5 -> H)
    if pe_table.is_cuda:
        bias = pos_bias_gather(pe_table, pe_idx)
    else:
        Bn, Nn, Mn = pe_idx.shape
        bias = pe_table[pe_idx.reshape(-1)].view(Bn, Nn, Mn, H).permute(0, 3, 1, 2)
    s = d ** -0.5
    return dict(q=rnd(B, H, N, d, std=s), k=rnd(B, H, N, d, std=s), v=rnd(B, H, N, d, std=s),
                member_idx=member, bias=bias.contiguous(), blank_k=rnd(H, d, std=0.2),
                blank_v=rnd(H, d, std=0.2), dout=rnd(B, H, N, d), scale=s, pos=pos)


def tile_union(member_idx: torch.Tensor, tile: int, cluster: int = 8) -> float:
    """Mean number of distinct key clusters listed by a tile of ``tile``
    consecutive queries (lists of whole clusters, [B,N,M]): the keys a
    query-tiled kernel computes per tile are cluster x this, against M listed
    per query."""
    B, N, M = member_idx.shape
    clu = (member_idx[..., ::cluster] // cluster).long()
    n = (N // tile) * tile
    c = clu[:, :n].reshape(B * (n // tile), tile * (M // cluster))
    s = c.sort(dim=1).values
    distinct = 1 + (s[:, 1:] != s[:, :-1]).sum(1)
    return distinct.double().mean().item()

def nbhd_attention_bytes(B, H, N, d, M, elem=2):
    """Algorithmic (interface) bytes of one forward and one backward call."""
    T = B * H * N * d * elem
    idx = B * N * M * 4
    bias = B * H * N * M * elem
    lse = B * H * N * 4
    fwd = 4 * T + lse + idx + bias
    bwd = 5 * T + lse + idx + bias + 3 * T + bias
    return fwd, bwd


def knn_points(B=8, side=96, stride=4, jitter=True, seed=0, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    ys, xs = torch.meshgrid(torch.arange(side).float(), torch.arange(side).float(), indexing="ij")
    grid = torch.stack([xs, ys], -1).reshape(1, -1, 2) * stride
    pos = grid.expand(B, -1, -1).clone()
    if jitter:
        pos = pos + torch.rand(pos.shape, generator=g) - 0.5
    return pos.to(device)


def deform_inputs(B=16, side=96, level_side=96, H=8, C=32, dtype=torch.bfloat16, seed=0,
                  device="cuda"):
    """One level of config 4 in level-0 token units: queries on the side x side
    lattice, kv positions on a level_side lattice ((i+0.5)*s - 0.5), reference
    points r ~ U[0,1]^2 -> r*side - 0.5, offsets N(0, 0.05)*side, weights
    softmaxed over 12 level-points (the slice of this level is passed)."""
    g = torch.Generator().manual_seed(seed)
    s = side / level_side
    ii = torch.arange(level_side).float()
    ys, xs = torch.meshgrid(ii, ii, indexing="ij")
    kv = (torch.stack([xs, ys], -1).reshape(1, -1, 2) + 0.5) * s - 0.5
    kv = kv.expand(B, -1, -1).contiguous()
    Nq = side * side
    qpos = torch.rand((B, Nq, 2), generator=g) * side - 0.5
    off = torch.randn((B, Nq, H, 4, 2), generator=g) * 0.05 * side
    logits = torch.randn((B, Nq, H, 12), generator=g)
    aw = torch.softmax(logits, -1)[..., :4].contiguous()
    val = torch.randn((B, kv.shape[1], H, C), generator=g)
    dout = torch.randn((B, Nq, H, C), generator=g)
    to = lambda t, dt=torch.float32: t.to(device=device, dtype=dt)
    return dict(query_pos=to(qpos), kv_pos=to(kv), offsets=to(off), attn_weights=to(aw),
                values=to(val, dtype), power=torch.tensor(1.0, device=device), dout=to(dout, dtype))


def deform_levels_inputs(B=16, side=96, level_sides=(96, 48, 24), H=8, C=32, dtype=torch.bfloat16,
                         seed=0, device="cuda"):
    """All levels of config 4 in level-0 token units: one query set, per level l
    a kv lattice of level_sides[l]^2 points ((i+0.5)*s_l - 0.5), offsets
    N(0, 0.05)*side, and the level's 4-point slice of a softmax over the
    4*len(level_sides) (level, point) pairs of each head.  Returns
    dict(query_pos, power, dout, levels=[dict(kv_pos, offsets, attn_weights, values)])."""
    g = torch.Generator().manual_seed(seed)
    L = len(level_sides)
    Nq = side * side
    qpos = torch.rand((B, Nq, 2), generator=g) * side - 0.5
    aw_all = torch.softmax(torch.randn((B, Nq, H, 4 * L), generator=g), -1)
    to = lambda t, dt=torch.float32: t.to(device=device, dtype=dt)
    levels = []
    for li, ls in enumerate(level_sides):
        s = side / ls
        ii = torch.arange(ls).float()
        ys, xs = torch.meshgrid(ii, ii, indexing="ij")
        kv = ((torch.stack([xs, ys], -1).reshape(1, -1, 2) + 0.5) * s - 0.5).expand(B, -1, -1).contiguous()
        off = torch.randn((B, Nq, H, 4, 2), generator=g) * 0.05 * side
        val = torch.randn((B, kv.shape[1], H, C), generator=g)
        levels.append(dict(kv_pos=to(kv), offsets=to(off),
                           attn_weights=to(aw_all[..., 4 * li:4 * li + 4].contiguous()),
                           values=to(val, dtype)))
    dout = torch.randn((B, Nq, H, C), generator=g)
    return dict(query_pos=to(qpos), power=torch.tensor(1.0, device=device), dout=to(dout, dtype),
                levels=levels)


def deform_levels_bytes(B, Nq, level_n, H, C, elem):
    """Interface bytes of one forward and one backward over all levels (config 4):
    values, offsets, weights, query positions, output; the backward reads
    dout and the inputs and writes every gradient."""
    nkv = sum(level_n)
    L = len(level_n)
    val = B * nkv * H * C * elem
    off = B * Nq * H * 4 * L * 2 * elem
    aw = B * Nq * H * 4 * L * elem
    qp = B * Nq * 2 * 4
    out = B * Nq * H * C * elem
    fwd = val + off + aw + qp + out
    bwd = out + val + off + aw + qp + val + off + aw + qp + B * nkv * 2 * 4
    return fwd, bwd
