"""AFF-small masked autoencoder on the affmae_b200 operators (the config 5
pretraining workload).

The network follows the reference's AFFMaskedAutoEncoder
(src/models/aff_mae.py:26-160) with its AFF encoder (src/layers/aff.py) and
cross-attention pixel decoder (src/layers/decoder.py); every custom-kernel op
on its path runs on this package's CUDA kernels:

  * tokens are grouped into clusters of 8 along a space-filling scan of grid
    anchors (``curve_clusters``; reference src/utils/geometry.py:170-319), each
    token attends the members of its 6 nearest clusters (KNN kernel) with a
    relative-position bias evaluated in-kernel from the Linear(5 -> H) weights
    (relative-bias kernels) and a blank token (neighbourhood-attention kernels);
  * adaptive downsampling keeps the tokens with the highest learned
    importance and merges each kept token's neighbourhood with
    position-dependent weights (weighted-features kernels);
  * the decoder's deformable self/cross attention runs on the fused
    KNN-Shepard deformable kernels.

Dense layers (Linear, GELU, convolutions) are PyTorch modules; the
LayerNorms of the encoder blocks, stage outputs, merging and decoder blocks
run on the fused residual + dropout + LayerNorm kernels.
Deliberate differences from the reference: tokens are masked with uniform
random noise (the reference's Perlin-noise masking depends on the
``perlin_noise`` package), and the unused ``global_norm`` / ``global_linear``
layers of the reference's merging module are not created (they never receive
gradients, which data-parallel training would reject).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native as nat
from .kernels.fused_deform_attn import (fused_knn_deformable_cross_attention,
                                        fused_knn_deformable_self_attention)
from .kernels.head_layout import merge_heads, split_heads
from .kernels.knn import knn
from .kernels.layer_norm import FusedLayerNorm
from .kernels.local_attn import FlashLocalAttentionFunction
from .kernels.pos_bias import pos_bias_gather, rel_pos_bias
from .kernels.relu_dropout import relu_dropout
from .kernels.token_mask import apply_token_mask
from .kernels.weighted_features import weighted_features
from .workloads import REL_POS_WIDTH, TABLE_WIDTH, relative_position_table


@dataclass
class MAEConfig:
    """Defaults: the config 5 model (AFF-small on 1024 x 1024 single-channel
    images, patch stride 4, 0.5 token mask, 48-token neighbourhoods)."""
    img_size: int = 1024
    patch_size: int = 4
    in_chans: int = 1
    mask_ratio: float = 0.5
    embed_dims: tuple = (96, 192, 384, 512)
    depths: tuple = (2, 3, 9, 2)
    num_heads: tuple = (3, 6, 12, 16)
    nbhd_size: int = 48
    cluster_size: int = 8
    ds_rate: float = 0.4
    mlp_ratio: float = 2.0
    drop_path_rate: float = 0.1
    decoder_dim: int = 384
    decoder_heads: int = 6
    decoder_dropout: float = 0.1
    loss_weights: tuple = field(default=(0.05, 0.12, 1.0))  # res5, res4, res2 heads


# ------------------------------------------------------------- clustering --

@torch.no_grad()
def curve_clusters(pos: torch.Tensor, m: int, h: int, w: int):
    """Balanced clustering of tokens along a space-filling scan.

    The h x w canvas is cut into about n/m anchor cells visited row by row in
    alternating direction; a token's rank is its cell's visiting order plus,
    within the cell, its distance ratio to the previous and next anchors.
    Sorting by rank and cutting into runs of m gives the clusters
    (reference geometry.py:170-319, default scan, anchors on).

    Returns (pos in cluster order [B,n,2], cluster means [B,k,2],
    cluster_mask [B,k,m] long or None when n % m == 0, order [B,n] with
    order[b, i] = original index of the i-th token).
    """
    return clusters_in_order(pos, curve_key(pos, m, h, w).argsort(dim=1), m)


def clusters_in_order(pos: torch.Tensor, order: torch.Tensor, m: int):
    """The outputs of curve_clusters for a given token order [B,n]: runs of m
    tokens along it are the clusters, the last one partial when m does not
    divide n."""
    pos = pos.detach().float()
    B, n, _ = pos.shape
    dev = pos.device
    k = math.ceil(n / m)
    pos = pos.gather(1, order[..., None].expand(-1, -1, 2))
    if k * m == n:
        return pos, pos.view(B, k, m, 2).mean(2), None, order
    padded = torch.zeros((B, k * m, 2), device=dev)
    padded[:, :n] = pos
    cmask = torch.zeros((B, k * m), device=dev, dtype=torch.long)
    cmask[:, :n] = 1
    cmask = cmask.view(B, k, m)
    means = padded.view(B, k, m, 2).sum(2) / cmask.sum(2, keepdim=True)
    return pos, means, cmask, order


@torch.no_grad()
def curve_key(pos: torch.Tensor, m: int, h: int, w: int) -> torch.Tensor:
    """The scan rank of every token [B,n] fp32 (cell visiting order scaled
    above the largest within-cell distance ratio, plus the ratio): sorting
    it gives the cluster order.  Tokens with equal keys are left in the
    order the sort implementation picks, as in the reference."""
    pos = pos.detach().float()
    B, n, _ = pos.shape
    dev = pos.device
    k = math.ceil(n / m)
    cell = math.sqrt(h * w / k)
    ny, nx = int(round(h / cell)), int(round(w / cell))
    cy, cx = h / ny, w / nx
    gy, gx = torch.meshgrid(torch.arange(ny, device=dev), torch.arange(nx, device=dev), indexing="ij")
    visit = gy * nx + torch.where(gy % 2 == 1, nx - 1 - gx, gx)          # visiting rank of each cell
    cell_xy = torch.empty((ny * nx, 2), device=dev)
    cell_xy[visit.reshape(-1)] = torch.stack([gx, gy], -1).reshape(-1, 2).float()
    # cell sizes as fp32 scalars (no host-to-device copy, so nothing waits for the GPU)
    sx, sy = float(torch.tensor(cx, dtype=torch.float32)), float(torch.tensor(cy, dtype=torch.float32))
    anchors = torch.stack([cell_xy[:, 0] * sx + sx / 2 - 0.5, cell_xy[:, 1] * sy + sy / 2 - 0.5], -1)
    prev = torch.cat([2 * anchors[:1] - anchors[1:2], anchors[:-1]], 0)
    nxt = torch.cat([anchors[1:], 2 * anchors[-1:] - anchors[-2:-1]], 0)
    fx = (pos[..., 0] / sx).floor().long()
    fy = (pos[..., 1] / sy).floor().long()
    rank = visit.reshape(-1)[fx + fy * nx]                               # [B,n]
    d_prev = (pos - prev[rank]).pow(2).sum(-1)
    d_next = (pos - nxt[rank]).pow(2).sum(-1)
    ratio = d_prev / (d_next + 1e-5)
    return rank.float() * (ratio.max() + 1) + ratio


def neighbourhood(pos: torch.Tensor, means: torch.Tensor, cmask, nbhd: int, m: int):
    """member_idx [B,n,M] (int32, padding slots -> 0), mask [B,n,M] bool or
    None, pe_idx [B,n,M] int64 for tokens in cluster order (aff.py:426-465):
    the nearest-cluster search on the KNN kernel, then one kernel that expands
    the cluster ids into the three lists."""
    B, n, _ = pos.shape
    k = means.shape[1]
    nnc = min(int(round(nbhd / m)), k)
    assert m == 8, "the neighbour-list kernel expands clusters of 8 tokens"
    nearest = knn(pos, means, nnc).contiguous()                          # [B,n,nnc] int64
    M = nnc * m
    p = pos.float().contiguous()
    member = torch.empty((B, n, M), device=pos.device, dtype=torch.int32)
    pe_idx = torch.empty((B, n, M), device=pos.device, dtype=torch.int64)
    mask = torch.empty((B, n, M), device=pos.device, dtype=torch.bool) if cmask is not None else None
    nat.call("affb_nbhd_build", nat.ptr(p), nat.ptr(nearest), B, n, nnc, nat.ptr(member),
             nat.ptr(mask.view(torch.uint8)) if mask is not None else None, nat.ptr(pe_idx), nat.stream(pos.device))
    return member, mask, pe_idx


# ----------------------------------------------------------------- blocks --

class _LinearFunction(torch.autograd.Function):
    """y = x W^T + b in the autocast dtype; the backward computes the bias
    gradient as a matrix-vector product with a ones vector (a single cuBLAS
    GEMV over the gradient rows, fp32 accumulation) instead of a reduction
    kernel, and dW / dX with one GEMM each."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda", cast_inputs=torch.bfloat16)
    def forward(ctx, x, weight, bias):
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        return F.linear(x, weight, bias)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, g):
        x, weight = ctx.saved_tensors
        g2 = g.reshape(-1, g.shape[-1])
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = (g2 @ weight).view(x.shape)
        if ctx.needs_input_grad[1]:
            dw = g2.t() @ x.reshape(-1, x.shape[-1])
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = torch.mv(g2.t(), torch.ones(g2.shape[0], device=g.device, dtype=g.dtype))
        return dx, dw, db


def _linear(x, weight, bias):
    if x.is_cuda and torch.is_autocast_enabled("cuda"):
        return _LinearFunction.apply(x, weight, bias)
    return F.linear(x, weight, bias)


class Linear(nn.Linear):
    """nn.Linear whose CUDA autocast path runs through _LinearFunction."""

    def forward(self, x):
        return _linear(x, self.weight, self.bias)


class DropPath(nn.Module):
    def __init__(self, p: float):
        super().__init__()
        self.p = p

    def forward(self, x):
        f = self.factor(x.shape[0], x.device)
        return x if f is None else x * f.view((-1,) + (1,) * (x.dim() - 1)).to(x.dtype)

    def factor(self, B: int, device):
        """Per-sample factor [B] fp32 (0 or 1 / keep), None when inactive; the
        fused residual norms apply it inside their pass."""
        if not self.training or self.p == 0.0:
            return None
        keep = 1.0 - self.p
        return torch.empty((B,), device=device, dtype=torch.float32).bernoulli_(keep) / keep


class ClusterAttention(nn.Module):
    """Neighbourhood attention with relative-position bias and a per-head blank
    token (reference attention.py:20-207, local path)."""

    def __init__(self, dim: int, heads: int):
        super().__init__()
        self.heads = heads
        self.scale = (dim // heads) ** -0.5
        self.q = Linear(dim, dim)
        self.kv = Linear(dim, 2 * dim)
        self.blank_k = nn.Parameter(torch.randn(dim) * 0.2)
        self.blank_v = nn.Parameter(torch.randn(dim) * 0.2)
        self.pos_embed = Linear(5, heads)
        self.proj = Linear(dim, dim)

    def forward(self, feat, member_idx, mask, pe_idx, global_attn: bool = False):
        B, N, C = feat.shape
        H, d = self.heads, C // self.heads
        q = split_heads(self.q(feat), H)
        k, v = split_heads(self.kv(feat), H, 2)
        bias = rel_pos_bias(self.pos_embed.weight, self.pos_embed.bias, pe_idx, q.dtype)  # [B,H,N,M]
        if global_attn:
            # every token attends every token plus the blank token
            # (attention.py:157-180): pe_idx is [B,N,N]; the bias gets a zero
            # column for the blank key; PyTorch's fused attention (library code)
            bias = F.pad(bias, (0, 1))
            bk = self.blank_k.view(1, H, 1, d).expand(B, -1, -1, -1).to(q.dtype)
            bv = self.blank_v.view(1, H, 1, d).expand(B, -1, -1, -1).to(q.dtype)
            out = F.scaled_dot_product_attention(q, torch.cat([k, bk], 2), torch.cat([v, bv], 2), attn_mask=bias)
            return self.proj(merge_heads(out.contiguous()))
        out = FlashLocalAttentionFunction.apply(
            q, k, v, member_idx, bias, None if mask is None else mask[:, None],
            self.blank_k.view(H, d), self.blank_v.view(H, d), float(self.scale))
        return self.proj(merge_heads(out))


class ClusterBlock(nn.Module):
    def __init__(self, dim: int, heads: int, mlp_ratio: float, drop_path: float):
        super().__init__()
        self.norm1 = FusedLayerNorm(dim)
        self.attn = ClusterAttention(dim, heads)
        self.norm2 = FusedLayerNorm(dim)
        hidden = int(dim * mlp_ratio)
        self.fc1 = Linear(dim, hidden)
        self.fc2 = Linear(hidden, dim)
        self.drop_path = DropPath(drop_path)

    def forward(self, feat, member_idx, mask, pe_idx, global_attn: bool = False, pending=None):
        """Returns (feat, pending): the MLP branch's residual add is left
        pending, (delta, per-sample factor), so that it runs inside the next
        block's first norm; ``add_pending`` completes it.  Each residual add
        with its stochastic-depth factor and the following pre-norm are one
        fused pass (the norms feed only Linears, so their output is in the
        autocast dtype)."""
        B = feat.shape[0]
        if pending is None:
            h = self.norm1(feat, out32=False, out16=True)
        else:
            feat, h = self.norm1.residual(feat, *pending)
        a = self.attn(h, member_idx, mask, pe_idx, global_attn)
        feat, h = self.norm2.residual(feat, a, self.drop_path.factor(B, feat.device))
        return feat, (self.fc2(F.gelu(self.fc1(h))), self.drop_path.factor(B, feat.device))


def add_pending(feat, pending):
    """feat + factor * delta for a residual add left pending by ClusterBlock."""
    if pending is None:
        return feat
    delta, f = pending
    if f is not None:
        delta = delta * f.view((-1,) + (1,) * (delta.dim() - 1)).to(delta.dtype)
    return feat + delta


class ClusterMerging(nn.Module):
    """Adaptive downsampling (reference aff.py:123-299, cluster merging without
    reserve tokens): keep the int(n * ds_rate) tokens of highest learned
    importance; merge each kept token's neighbourhood with weights
    weight_net(rel_table)[pe_idx] * importance(neighbour) (* padding mask)."""

    def __init__(self, dim: int, out_dim: int, ds_rate: float, inner: int = 4):
        super().__init__()
        self.ds_rate = ds_rate
        self.weight_net = nn.Sequential(nn.Linear(5, inner), FusedLayerNorm(inner), nn.GELU())
        self.norm = FusedLayerNorm(inner * dim)
        self.linear = Linear(inner * dim, out_dim)
        self.register_buffer("rel_table", relative_position_table(), persistent=False)

    def forward(self, pos, feat, member_idx, mask, importance, pe_idx):
        B, n, C = feat.shape
        M = member_idx.shape[-1]
        keep = int(n * self.ds_rate)
        idx = importance.detach().view(B, n).topk(keep, dim=1, sorted=False)[1]
        pos_down = pos.gather(1, idx[..., None].expand(-1, -1, 2))
        sel = idx[..., None].expand(-1, -1, M)
        member = member_idx.gather(1, sel)
        pe = pe_idx.gather(1, sel)
        lp = importance.gather(1, member.reshape(B, -1, 1).long()).reshape(B, keep, M, 1)
        if mask is not None:
            lp = lp * mask.gather(1, sel)[..., None]
        table = self.weight_net(self.rel_table.to(feat.dtype))           # [T, inner]
        # gather through the bias kernel ([B,inner,keep,M]); its backward is one
        # block-reduced scatter-add into the table instead of a sorted index_put
        weights = pos_bias_gather(table, pe).permute(0, 2, 3, 1) * lp     # [B,keep,M,inner]
        if feat.is_cuda and torch.is_autocast_enabled("cuda"):
            # under autocast the merge reads 16-bit features (the tensor-core
            # kernel) whatever the dtype of the residual stream
            feat = feat.to(torch.get_autocast_dtype("cuda"))
        merged = weighted_features(weights.to(feat.dtype), feat, member)  # [B,keep,inner,C]
        return pos_down, self.linear(self.norm(merged.reshape(B, keep, -1), out32=False, out16=True))


class Stage(nn.Module):
    """One encoder stage (reference BasicLayer, aff.py:311-538)."""

    def __init__(self, dim, out_dim, depth, heads, cfg: MAEConfig, drop_paths):
        super().__init__()
        self.cfg = cfg
        self.blocks = nn.ModuleList(ClusterBlock(dim, heads, cfg.mlp_ratio, dp) for dp in drop_paths)
        self.merge = None
        if out_dim is not None:
            self.prob_net = Linear(dim, 1)
            self.merge = ClusterMerging(dim, out_dim, cfg.ds_rate)

    def forward(self, pos, feat, h, w):
        B, n, C = feat.shape
        m = self.cfg.cluster_size
        pos, means, cmask, order = curve_clusters(pos, m, h, w)
        feat = feat.gather(1, order[..., None].expand(-1, -1, C))
        member, mask, pe_idx = neighbourhood(pos, means, cmask, self.cfg.nbhd_size, m)
        global_attn = self.cfg.nbhd_size >= n  # BasicLayer.forward, aff.py:421-424
        att_pe = pe_idx
        if global_attn:  # relative indices of every token pair (aff.py:458-459)
            rel = ((pos[:, None, :, :] + REL_POS_WIDTH) - pos[:, :, None, :]).clamp(0, TABLE_WIDTH - 1)
            att_pe = (rel[..., 1] * TABLE_WIDTH + rel[..., 0]).long()
        pending = None
        in_dtype = feat.dtype
        for blk in self.blocks:
            feat, pending = blk(feat, member, mask, att_pe, global_attn, pending)
        # the fused norms carry the stream in fp32; the stage hands on the dtype it received
        feat = add_pending(feat, pending).to(in_dtype)
        if self.merge is None:
            return pos, feat, pos, feat
        importance = self.prob_net(feat).sigmoid()
        pos_down, feat_down = self.merge(pos, feat, member, mask, importance, pe_idx)
        return pos, feat, pos_down, feat_down


class PatchEmbed(nn.Module):
    """Stride-2 3x3 convolutions down to patch resolution; the token mask is
    re-applied after every convolution so masked patches never leak into
    visible tokens (reference aff.py:558-665).  The convolutions run channels
    last, so the channel LayerNorms see contiguous [.., C] rows and run on the
    fused kernel without a transpose copy."""

    def __init__(self, patch_size: int, in_chans: int, dim: int):
        super().__init__()
        layers = int(math.log2(patch_size))
        assert 2 ** layers == patch_size
        self.patch_size = patch_size
        self.convs = nn.ModuleList()
        self.norms = nn.ModuleList()
        ch = in_chans
        for i in range(layers):
            out = dim if i == layers - 1 else dim // 2
            self.convs.append(nn.Conv2d(ch, out, 3, stride=2, padding=1))
            if i < layers - 1:
                self.norms.append(FusedLayerNorm(out))
            ch = out
        self.norm = FusedLayerNorm(dim)

    def forward(self, x, token_mask):
        """x [B,C,H,W]; token_mask [B, H/p, W/p] (1 visible, 0 masked)."""
        x = x.contiguous(memory_format=torch.channels_last)
        for i, conv in enumerate(self.convs):
            x = conv(x)
            x = apply_token_mask(x, token_mask)
            if i < len(self.norms):
                y = self.norms[i](x.permute(0, 2, 3, 1), out32=False, out16=True)
                x = F.gelu(y).permute(0, 3, 1, 2)
        B, C, h, w = x.shape
        feat = self.norm(x.permute(0, 2, 3, 1).reshape(B, h * w, C))
        ys, xs = torch.meshgrid(torch.arange(h, device=x.device), torch.arange(w, device=x.device), indexing="ij")
        pos = torch.stack([xs, ys], -1).reshape(1, -1, 2).expand(B, -1, -1).float()
        return pos, feat, h, w


class Encoder(nn.Module):
    def __init__(self, cfg: MAEConfig):
        super().__init__()
        self.patch_embed = PatchEmbed(cfg.patch_size, cfg.in_chans, cfg.embed_dims[0])
        dpr = torch.linspace(0, cfg.drop_path_rate, sum(cfg.depths)).tolist()
        self.stages = nn.ModuleList()
        for i, depth in enumerate(cfg.depths):
            out = cfg.embed_dims[i + 1] if i + 1 < len(cfg.depths) else None
            s0 = sum(cfg.depths[:i])
            self.stages.append(Stage(cfg.embed_dims[i], out, depth, cfg.num_heads[i], cfg, dpr[s0:s0 + depth]))
        self.norms = nn.ModuleList(FusedLayerNorm(d) for d in cfg.embed_dims)
        self._init()

    def _init(self):
        """Initialisation of the reference encoder (aff.py:713-730): q/kv
        trunc-normal(0.02); position-bias, projection, MLP-in, importance,
        merging and weight-net layers Xavier-uniform; MLP-out Kaiming-uniform;
        LayerNorms (1, 0)."""
        for mod in self.modules():
            if isinstance(mod, ClusterAttention):
                nn.init.trunc_normal_(mod.q.weight, std=0.02)
                nn.init.trunc_normal_(mod.kv.weight, std=0.02)
                nn.init.xavier_uniform_(mod.pos_embed.weight)
                nn.init.xavier_uniform_(mod.proj.weight)
            elif isinstance(mod, ClusterBlock):
                nn.init.xavier_uniform_(mod.fc1.weight)
                nn.init.kaiming_uniform_(mod.fc2.weight, a=math.sqrt(5))
            elif isinstance(mod, ClusterMerging):
                nn.init.xavier_uniform_(mod.weight_net[0].weight)
                nn.init.xavier_uniform_(mod.linear.weight)
            elif isinstance(mod, Stage) and mod.merge is not None:
                nn.init.xavier_uniform_(mod.prob_net.weight)
            elif isinstance(mod, nn.LayerNorm):
                nn.init.ones_(mod.weight)
                nn.init.zeros_(mod.bias)

    def forward(self, feat, pos, h, w):
        """Per stage: (normalised features [B,n_s,C_s], positions [B,n_s,2])."""
        outs = []
        for stage, norm in zip(self.stages, self.norms):
            pos_out, x_out, pos, feat = stage(pos, feat, h, w)
            outs.append((norm(x_out, out32=False, out16=True), pos_out))  # consumed by Linears only
        return outs


# ---------------------------------------------------------------- decoder --

def sine_embedding(pos: torch.Tensor, dim: int, dtype=torch.float32) -> torch.Tensor:
    """[B,n,2] -> [B,n,dim]: sin/cos of x then y, each over dim/2 frequencies,
    coordinates scaled by 2*pi / max (reference decoder.py:16-62, normalised).
    On the GPU one kernel writes it in ``dtype`` with the same fp32 arithmetic."""
    half = dim // 2
    i = torch.arange(half, device=pos.device, dtype=torch.float32)
    freq = 10000.0 ** (2 * torch.div(i, 2, rounding_mode="floor") / half)
    if pos.is_cuda:
        p = pos.detach().float().contiguous()
        if p.data_ptr() % 8:
            p = p.clone()
        maxes = p.reshape(-1, 2).amax(0).contiguous()
        out = torch.empty(p.shape[:-1] + (dim,), device=p.device, dtype=dtype)
        nat.call("affb_sine_embed", nat.ptr(p), p.numel() // 2, dim, nat.ptr(maxes), nat.ptr(freq), nat.ptr(out),
                 nat.dcode(out), nat.stream(p.device))
        return out
    x = pos[..., 0].float()
    y = pos[..., 1].float()
    x = x / (x.max() + 1e-6) * (2 * math.pi)
    y = y / (y.max() + 1e-6) * (2 * math.pi)

    def enc(t):
        t = t[..., None] / freq
        return torch.cat([t[..., 0::2].sin(), t[..., 1::2].cos()], -1)
    return torch.cat([enc(x), enc(y)], -1).to(dtype)

class _SplitColumns(torch.autograd.Function):
    """x[..., :k] and x[..., k:] as contiguous fp32 tensors (the deformable
    kernels' offset and weight inputs); the gradient is one concatenation in
    the dtype of x, instead of two zero-filled slice gradients summed."""

    @staticmethod
    def forward(ctx, x, k):
        ctx.dtype, ctx.k, ctx.rest = x.dtype, k, x.shape[-1] - k
        return x[..., :k].float().contiguous(), x[..., k:].float().contiguous()

    @staticmethod
    def backward(ctx, ga, gb):
        if ga is None:
            ga = gb.new_zeros(gb.shape[:-1] + (ctx.k,))
        if gb is None:
            gb = ga.new_zeros(ga.shape[:-1] + (ctx.rest,))
        return torch.cat([ga, gb], -1).to(ctx.dtype), None


class DeformableAttention(nn.Module):
    """Single-level deformable attention with 4 sampling points per head and
    Shepard (inverse-distance softmax) interpolation over the 4 nearest
    tokens (reference attention.py:210-593, fused KNN path)."""

    def __init__(self, dim: int, heads: int, points: int = 4):
        super().__init__()
        self.heads, self.points = heads, points
        self.sampling_offsets = Linear(dim, heads * points * 2)
        self.attention_weights = Linear(dim, heads * points)
        self.value_proj = Linear(dim, dim)
        self.output_proj = Linear(dim, dim)
        self.shepard_power = nn.Parameter(torch.tensor(1.0))
        nn.init.zeros_(self.sampling_offsets.weight)
        theta = torch.arange(heads, dtype=torch.float32) * (2.0 * math.pi / heads)
        grid = torch.stack([theta.cos(), theta.sin()], -1)
        grid = (grid / grid.abs().max(-1, keepdim=True)[0])[:, None].repeat(1, points, 1)
        grid = grid * torch.arange(1, points + 1, dtype=torch.float32)[None, :, None]
        with torch.no_grad():
            self.sampling_offsets.bias.copy_(grid.reshape(-1))
        nn.init.zeros_(self.attention_weights.weight)
        nn.init.zeros_(self.attention_weights.bias)
        for lin in (self.value_proj, self.output_proj):
            nn.init.xavier_uniform_(lin.weight)
            nn.init.zeros_(lin.bias)

    def forward(self, query, query_pos, kv=None, kv_pos=None):
        B, n, C = query.shape
        H, P = self.heads, self.points
        # sampling offsets and attention weights read the same input: one GEMM
        # over the two weight matrices stacked (one input gradient, not two summed)
        ow = _linear(query, torch.cat([self.sampling_offsets.weight, self.attention_weights.weight]),
                     torch.cat([self.sampling_offsets.bias, self.attention_weights.bias]))
        off, logits = _SplitColumns.apply(ow, H * P * 2)            # fp32, contiguous
        off = off.view(B, n, H, P, 2)
        aw = F.softmax(logits.view(B, n, H, P), dim=-1)
        if kv is None:  # self attention
            vals = self.value_proj(query).view(B, n, H, C // H)
            out = fused_knn_deformable_self_attention(query_pos, off, aw, vals, self.shepard_power)
        else:
            vals = self.value_proj(kv).view(B, kv.shape[1], H, C // H)
            out = fused_knn_deformable_cross_attention(query_pos, kv_pos, off, aw, vals, self.shepard_power)
        return self.output_proj(out.reshape(B, n, C))


class DecoderBlock(nn.Module):
    """Deformable self-attention over the masked queries, deformable
    cross-attention into one encoder level, ReLU FFN; post-norm residuals
    (reference decoder.py:66-143)."""

    def __init__(self, dim: int, heads: int, ffn: int, dropout: float):
        super().__init__()
        self.self_attn = DeformableAttention(dim, heads)
        self.cross_attn = DeformableAttention(dim, heads)
        self.norm1, self.norm2, self.norm3 = FusedLayerNorm(dim), FusedLayerNorm(dim), FusedLayerNorm(dim)
        self.linear1 = Linear(dim, ffn)
        self.linear2 = Linear(ffn, dim)
        self.p = dropout
        self.drop = nn.Dropout(dropout)

    def forward(self, q, q16, q_pos, src, src_pos, src_embed):
        """q: fp32 residual stream; q16: the same values in the autocast dtype
        (the Linears' input).  Each norm(q + dropout(delta)) is one fused pass
        returning both."""
        q, q16 = self._norm(self.norm1, q, self.self_attn(q16, q_pos))
        q, q16 = self._norm(self.norm2, q, self.cross_attn(q16, q_pos, src + src_embed, src_pos))
        h = self.linear1(q16)
        # ReLU + dropout in one pass; the gradient passes where the output is positive
        ff = self.linear2(relu_dropout(h, self.p, self.training) if h.is_cuda else self.drop(F.relu(h)))
        return self._norm(self.norm3, q, ff)

    def _norm(self, norm, q, delta):
        """(fp32 residual stream, Linear input): a bf16 copy under autocast,
        the fp32 values themselves outside it."""
        if q.is_cuda and torch.is_autocast_enabled("cuda"):
            return norm(q, delta, self.p, out32=True, out16=True)
        y = norm(q, delta, self.p, out32=True)
        return y, y


class PixelDecoder(nn.Module):
    """Masked-token queries refined level by level from the coarsest encoder
    stage to the finest (reference CrossAttentionPixelDecoder,
    decoder.py:146-371, one block per level)."""

    def __init__(self, cfg: MAEConfig):
        super().__init__()
        D = cfg.decoder_dim
        self.dim = D
        self.input_proj = nn.ModuleList(nn.Sequential(Linear(c, D), FusedLayerNorm(D))
                                        for c in reversed(cfg.embed_dims))
        for proj in self.input_proj:
            nn.init.xavier_uniform_(proj[0].weight)
            nn.init.zeros_(proj[0].bias)
        self.blocks = nn.ModuleList(DecoderBlock(D, cfg.decoder_heads, 2 * D, cfg.decoder_dropout)
                                    for _ in cfg.embed_dims)

    def forward(self, stages, queries, q_pos):
        q = queries + sine_embedding(q_pos, self.dim, queries.dtype)
        # the Linears' input in the autocast dtype once, not a cast inside each of them
        amp = q.is_cuda and torch.is_autocast_enabled("cuda")
        q16 = q.to(torch.get_autocast_dtype("cuda")) if amp else q
        outs = []
        for proj, blk, (feat, pos) in zip(self.input_proj, self.blocks, reversed(stages)):
            # the projected level only feeds value projections: normalised straight into bf16
            src = proj[1](proj[0](feat), out32=False, out16=True)
            q, q16 = blk(q, q16, q_pos, src, pos, sine_embedding(pos, self.dim, src.dtype))
            outs.append(q)
        return outs  # coarsest level first


# ------------------------------------------------------------------- model --

class PredictionHead(nn.Module):
    """LayerNorm + Linear to the patch pixels (reference aff_mae.py:80-92)."""

    def __init__(self, dim: int, out: int):
        super().__init__()
        self.norm = FusedLayerNorm(dim)
        self.linear = Linear(dim, out)

    def forward(self, x):
        return self.linear(self.norm(x, out32=False, out16=True))


class AFFMaskedAutoEncoder(nn.Module):
    """forward(images [B,C,H,W]) -> (loss, [loss_res5, loss_res4, loss_res2])."""

    def __init__(self, cfg: MAEConfig = MAEConfig()):
        super().__init__()
        self.cfg = cfg
        self.encoder = Encoder(cfg)
        self.decoder = PixelDecoder(cfg)
        D = cfg.decoder_dim
        out = cfg.patch_size ** 2 * cfg.in_chans
        self.masked_token = nn.Parameter(torch.randn(1, 1, D) * 0.02)
        self.head_res5 = PredictionHead(D, out)
        self.head_res4 = PredictionHead(D, out)
        self.head_res2 = PredictionHead(D, out)

    def patchify(self, imgs):
        p, c = self.cfg.patch_size, self.cfg.in_chans
        B, _, H, W = imgs.shape
        x = imgs.reshape(B, c, H // p, p, W // p, p)
        return torch.einsum("nchpwq->nhwpqc", x).reshape(B, (H // p) * (W // p), p * p * c)

    def random_masking(self, B: int, L: int, device, generator=None, noise=None):
        """Uniform random split into kept and masked patch ids.  The masked ids
        (the decoder's queries) are returned in raster order: a query's
        prediction is compared with the target gathered by the same id, so
        their order is free, and spatially ordered queries let the decoder's
        deformable kernels hit cache for neighbouring queries' samples."""
        keep = int(L * (1 - self.cfg.mask_ratio))
        if noise is None:
            noise = torch.rand((B, L), device=device, generator=generator)
        ids = noise.argsort(dim=1)
        return ids[:, :keep], ids[:, keep:].sort(dim=1).values

    def forward(self, imgs, generator=None, noise=None):
        """``noise`` [B, L] (optional) replaces the random draw that picks the
        masked patches (the patches with the largest noise are masked)."""
        cfg = self.cfg
        B, _, H, W = imgs.shape
        p = cfg.patch_size
        patches = self.patchify(imgs)
        L = patches.shape[1]
        ids_keep, ids_masked = self.random_masking(B, L, imgs.device, generator, noise)
        token_mask = torch.ones((B, L), device=imgs.device)
        token_mask.scatter_(1, ids_masked, 0.0)
        token_mask = token_mask.view(B, H // p, W // p)
        pos, feat, h, w = self.encoder.patch_embed(apply_token_mask(imgs, token_mask), token_mask)
        C0 = feat.shape[-1]
        vis_feat = feat.gather(1, ids_keep[..., None].expand(-1, -1, C0))
        vis_pos = pos.gather(1, ids_keep[..., None].expand(-1, -1, 2))
        stages = self.encoder(vis_feat, vis_pos, h, w)
        m_pos = pos.gather(1, ids_masked[..., None].expand(-1, -1, 2))
        queries = self.masked_token.expand(B, m_pos.shape[1], -1)
        outs = self.decoder(stages, queries, m_pos)
        target = patches.gather(1, ids_masked[..., None].expand(-1, -1, patches.shape[-1]))
        preds = [self.head_res5(outs[0]), self.head_res4(outs[1]), self.head_res2(outs[-1])]
        losses = [F.mse_loss(pr.float(), target.float()) for pr in preds]
        loss = sum(wt * l for wt, l in zip(cfg.loss_weights, losses))
        return loss, losses
