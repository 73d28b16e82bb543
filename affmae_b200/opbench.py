"""Per-operator timings at the benchmark configurations' shapes.

``python -m affmae_b200.opbench <op> [--iters N]`` times one operator on the
GPU with CUDA events (inputs resident, L2 flushed by a 256 MiB write before
every call) and prints one JSON line with its algorithmic bytes and achieved
GB/s; the same command under ``ncu -k <kernel>`` gives the kernel profiles.

  knn        config 2: B=8, N=9216 jittered lattice, queries = points, K=48
  knn-brute  the same through the brute-force scan
  deform     config 4, one level (96x96 kv lattice): B=16, Nq=9216, H=8, C=32, bf16, fwd+bwd
  deform-mae config 5 decoder self-attention: B=16, 32768 masked-patch queries of a 256x256
             lattice in random order, kv = the queries, H=6, C=64, bf16, fwd+bwd
  deform-mae-raster  the same with the queries in raster order
  wfeat      config 5 stage-1 merging: weights [16,13107,48,4], feat [16,32768,96] bf16, fwd+bwd
  wfeat-fwd  the same, forward only
  wfeat-lists / wfeat-lists-fwd  the same with the merging step's own index lists (the stage-1
             neighbourhoods of the kept tokens: 6 runs of 8 consecutive rows) instead of random rows
  wgather    config 1: idx [2,1024,48], softmax weights, feat [2,4096,128] fp32, fwd+bwd
  layer-norm  config 5 stage 1: residual + dropout + LayerNorm, 524288 rows of 96, fwd+bwd
  layer-norm-dec  the same at the decoder width (524288 rows of 384)
  res-norm    config 5 stage 1 pre-norm residual (s = x + delta kept in fp32, y = LN(s) in bf16), fwd+bwd
  res-norm-s3 the same at stage 3 (16 x 5243 rows of 384)
  rel-bias    config 5 stage 1: in-kernel relative-position bias [16,3,32768,48], fwd+bwd
  head-layout config 5 stage 1: kv head split + output merge, [16,32768,3x32], fwd+bwd
  deform-nbidx  deformable attention with given 4-NN indices (non-fused path), fwd+bwd

Algorithmic bytes count every interface tensor once (inputs read, outputs
written), as the roofline of a gather-bound operator.
"""
from __future__ import annotations

import argparse
import json

import torch


def _time(fn, iters, flush):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        flush.fill_(1)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        total += a.elapsed_time(b)
    return total / iters


def _nbytes(*ts):
    return sum(t.numel() * t.element_size() for t in ts)


def op_knn(brute=False):
    from .kernels import knn as kmod
    from .workloads import knn_points
    if brute:
        kmod.GRID_MIN_POINTS = 1 << 40
    pos = knn_points(B=8, side=96, stride=4, device="cuda")
    K = 48
    out = kmod.knn(pos, pos, K)
    B, N, _ = pos.shape
    return (lambda: kmod.knn(pos, pos, K)), B * (N * 8 + N * 8 + N * K * 8), {
        "B": B, "N": N, "M": N, "K": K, "path": "brute" if brute else "grid", "out": list(out.shape)}


def op_deform():
    from .kernels.fused_deform_attn import FusedKNNDeformCrossAttnFunction
    from .workloads import deform_inputs
    d = deform_inputs(B=16, side=96, level_side=96, H=8, C=32, dtype=torch.bfloat16, device="cuda")
    leaves = {k: d[k].detach().clone().requires_grad_(k in ("offsets", "attn_weights", "values"))
              for k in ("query_pos", "kv_pos", "offsets", "attn_weights", "values")}

    def step():
        out = FusedKNNDeformCrossAttnFunction.apply(leaves["query_pos"], leaves["kv_pos"], leaves["offsets"],
                                                    leaves["attn_weights"], leaves["values"], d["power"], 2)
        out.backward(d["dout"])
    fwd = _nbytes(leaves["values"], leaves["offsets"], leaves["attn_weights"], leaves["query_pos"], leaves["kv_pos"],
                  d["dout"])
    bwd = fwd + _nbytes(d["dout"], leaves["values"], leaves["offsets"], leaves["attn_weights"], leaves["query_pos"])
    return step, fwd + bwd, {"B": 16, "Nq": 9216, "Nkv": 9216, "H": 8, "C": 32, "dtype": "bf16",
                             "pass": "fwd+bwd"}


def op_deform_mae(raster=False):
    from .kernels.fused_deform_attn import FusedKNNDeformCrossAttnFunction
    import math
    g = torch.Generator().manual_seed(0)
    B, side, H, C = 16, 256, 6, 64
    L = side * side
    Nq = L // 2
    ids = torch.rand((B, L), generator=g).argsort(1)[:, L - Nq:]
    if raster:
        ids = ids.sort(1).values
    ii = torch.arange(side).float()
    ys, xs = torch.meshgrid(ii, ii, indexing="ij")
    lat = torch.stack([xs, ys], -1).reshape(-1, 2)
    pos = lat[ids]  # masked patch positions in random order, as the decoder queries
    theta = torch.arange(H).float() * (2 * math.pi / H)
    d = torch.stack([theta.cos(), theta.sin()], -1)
    d = (d / d.abs().max(-1, keepdim=True)[0])[:, None] * torch.arange(1, 5).float()[None, :, None]
    off = d[None, None] + 0.5 * torch.randn((B, Nq, H, 4, 2), generator=g)
    aw = torch.softmax(torch.randn((B, Nq, H, 4), generator=g), -1)
    val = torch.randn((B, Nq, H, C), generator=g)
    dout = torch.randn((B, Nq, H, C), generator=g).to("cuda", torch.bfloat16)
    qp = pos.to("cuda")
    leaves = {"offsets": off.to("cuda").requires_grad_(True), "attn_weights": aw.to("cuda").requires_grad_(True),
              "values": val.to("cuda", torch.bfloat16).requires_grad_(True)}
    power = torch.tensor(1.0, device="cuda")

    def step():
        out = FusedKNNDeformCrossAttnFunction.apply(qp, qp, leaves["offsets"], leaves["attn_weights"],
                                                    leaves["values"], power, 2)
        out.backward(dout)
    fwd = _nbytes(leaves["values"], leaves["offsets"], leaves["attn_weights"], qp, qp, dout)
    bwd = fwd + _nbytes(dout, leaves["values"], leaves["offsets"], leaves["attn_weights"], qp)
    return step, fwd + bwd, {"B": B, "Nq": Nq, "Nkv": Nq, "H": H, "C": C, "dtype": "bf16", "pass": "fwd+bwd",
                             "queries": "masked patches of a 256x256 lattice, " + ("raster order" if raster else "random order")}


def op_wfeat(fwd_only=False, lists=False):
    from .kernels.weighted_features import weighted_features
    g = torch.Generator().manual_seed(0)
    B, No, M, IC, N, C = 16, 13107, 48, 4, 32768, 96
    w = torch.randn((B, No, M, IC), generator=g).to("cuda", torch.bfloat16).requires_grad_(True)
    f = torch.randn((B, N, C), generator=g).to("cuda", torch.bfloat16).requires_grad_(True)
    if lists:
        # the merging step's own index lists: the neighbourhoods of stage 1
        # (256 x 256 patch grid at a 0.5 mask, clusters of 8 along the
        # reference's anchor scan, 6 nearest clusters) of 13107 kept tokens
        from .workloads import clustered_tokens, neighbourhoods
        member, _ = neighbourhoods(clustered_tokens(B, 256, 0.5, 0, "cuda", "curve"), 8, M)
        keep = torch.rand((B, N), generator=g).argsort(1)[:, :No].sort(1).values.to("cuda")
        idx = member.gather(1, keep[..., None].expand(-1, -1, M)).long()
    else:
        idx = torch.randint(0, N, (B, No, M), generator=g).to("cuda")
    dout = torch.randn((B, No, IC, C), generator=g).to("cuda", torch.bfloat16)

    if fwd_only:
        def step():
            with torch.no_grad():
                weighted_features(w, f, idx)
        return step, _nbytes(w, f, idx, dout), {"B": B, "No": No, "M": M, "IC": IC, "N": N, "C": C,
                                                "dtype": "bf16", "pass": "fwd",
                                                "indices": "stage-1 lists" if lists else "random"}

    def step():
        weighted_features(w, f, idx).backward(dout)
    fwd = _nbytes(w, f, idx, dout)
    bwd = _nbytes(dout, w, f, idx) + _nbytes(w, f)
    return step, fwd + bwd, {"B": B, "No": No, "M": M, "IC": IC, "N": N, "C": C, "dtype": "bf16",
                             "pass": "fwd+bwd", "indices": "stage-1 lists" if lists else "random"}


def op_wgather():
    from .kernels.weighted_gather import weighted_gather
    g = torch.Generator().manual_seed(0)
    B, Mq, K, N, C = 2, 1024, 48, 4096, 128
    idx = torch.randint(0, N, (B, Mq, K), generator=g).to("cuda")
    w = torch.softmax(torch.randn((B, Mq, K), generator=g), -1).to("cuda").requires_grad_(True)
    f = torch.randn((B, N, C), generator=g).to("cuda").requires_grad_(True)
    dout = torch.randn((B, Mq, C), generator=g).to("cuda")

    def step():
        weighted_gather(idx, w, f).backward(dout)
    fwd = _nbytes(idx, w, f, dout)
    bwd = _nbytes(dout, idx, w, f) + _nbytes(w, f)
    return step, fwd + bwd, {"B": B, "M": Mq, "K": K, "N": N, "C": C, "dtype": "fp32", "pass": "fwd+bwd"}


def op_layer_norm(C=96):
    """Config 5 stage 1 (C=96) or decoder (C=384): LayerNorm(x + dropout(delta))
    over 16 x 32768 tokens, fp32 residual stream and bf16 delta, fp32 + bf16
    outputs, fwd+bwd."""
    from .kernels.layer_norm import fused_layer_norm
    g = torch.Generator().manual_seed(0)
    R = 16 * 32768
    x = torch.randn((R, C), generator=g).to("cuda").requires_grad_(True)
    d = torch.randn((R, C), generator=g).to("cuda", torch.bfloat16).requires_grad_(True)
    w = torch.ones(C, device="cuda", requires_grad=True)
    b = torch.zeros(C, device="cuda", requires_grad=True)
    g32 = torch.randn((R, C), generator=g).to("cuda")
    g16 = torch.randn((R, C), generator=g).to("cuda", torch.bfloat16)

    def step():
        y32, y16 = fused_layer_norm(x, w, b, 1e-5, delta=d, p=0.1, out32=True, out16=True)
        torch.autograd.backward((y32, y16), (g32, g16))
    # fwd: x, delta in; s (saved sum), y32, y16 out; bwd: g32, g16, s in; dx, ddelta out
    fwd = R * C * (4 + 2 + 4 + 4 + 2)
    bwd = R * C * (4 + 2 + 4 + 4 + 2)
    return step, fwd + bwd, {"rows": R, "C": C, "x": "fp32", "delta": "bf16", "p": 0.1, "pass": "fwd+bwd"}


def op_residual_norm(R=16 * 32768, C=96):
    """Pre-norm residual block of the encoder: (s, y) = (x + delta, LayerNorm(s))
    with s fp32 kept, y bf16; the backward takes ds and dy.  Config 5 stage 1
    (16 x 32768 tokens, C=96) or stage 3 (16 x 5243 tokens, C=384)."""
    from .kernels.layer_norm import ResidualNormFunction
    g = torch.Generator().manual_seed(0)
    x = torch.randn((R, C), generator=g).to("cuda").requires_grad_(True)
    d = torch.randn((R, C), generator=g).to("cuda", torch.bfloat16).requires_grad_(True)
    w = torch.ones(C, device="cuda", requires_grad=True)
    b = torch.zeros(C, device="cuda", requires_grad=True)
    gs = torch.randn((R, C), generator=g).to("cuda")
    gy = torch.randn((R, C), generator=g).to("cuda", torch.bfloat16)

    def step():
        s, y = ResidualNormFunction.apply(x, d, None, w, b, 1e-5)
        torch.autograd.backward((s, y), (gs, gy))
    # fwd: x, delta in; s, y16 out; bwd: ds, dy16, s in; dx, ddelta out
    fwd = R * C * (4 + 2 + 4 + 2)
    bwd = R * C * (4 + 2 + 4 + 4 + 2)
    return step, fwd + bwd, {"rows": R, "C": C, "x": "fp32", "delta": "bf16", "pass": "fwd+bwd"}


def op_rel_bias():
    """Config 5 stage 1 relative-position bias: pe_idx [16,32768,48], H=3, bf16 out, fwd+bwd."""
    from .kernels.pos_bias import rel_pos_bias
    g = torch.Generator().manual_seed(0)
    B, N, M, H = 16, 32768, 48, 3
    pe = (torch.randint(110, 145, (B, N, M), generator=g) * 255 + torch.randint(110, 145, (B, N, M), generator=g))
    pe = pe.to("cuda")
    w = (0.02 * torch.randn((H, 5), generator=g)).to("cuda").requires_grad_(True)
    bb = torch.zeros(H, device="cuda", requires_grad=True)
    dout = torch.randn((B, H, N, M), generator=g).to("cuda", torch.bfloat16)

    def step():
        rel_pos_bias(w, bb, pe, torch.bfloat16).backward(dout)
    fwd = B * N * M * 8 + B * H * N * M * 2
    bwd = B * N * M * 8 + B * H * N * M * 2
    return step, fwd + bwd, {"B": B, "N": N, "M": M, "H": H, "pass": "fwd+bwd"}


def op_head_layout():
    """ClusterAttention head split of a [16, 32768, 2 x 3 x 32] kv projection and the merge
    of the output, bf16, fwd+bwd."""
    from .kernels.head_layout import merge_heads, split_heads
    g = torch.Generator().manual_seed(0)
    B, N, H, d = 16, 32768, 3, 32
    x = torch.randn((B, N, 2 * H * d), generator=g).to("cuda", torch.bfloat16).requires_grad_(True)
    gk = torch.randn((B, H, N, d), generator=g).to("cuda", torch.bfloat16)

    def step():
        k, v = split_heads(x, H, 2)
        y = merge_heads(k)
        torch.autograd.backward([y, v], [gk.permute(0, 2, 1, 3).reshape(B, N, H * d), gk])
    el = B * N * H * d * 2
    return step, 2 * (2 * el * 2 + el * 2), {"B": B, "N": N, "H": H, "d": d, "pass": "split+merge fwd+bwd"}


def op_deform_nbidx():
    """The reference's non-fused deformable path (attention.py:339-358): 4-NN indices given,
    [B*H, Nq*4] samples over one 96^2 kv level, C=32 bf16 (config 4 level 0), fwd+bwd."""
    from .kernels.fused_deform_attn import FusedDeformAttnFunction
    g = torch.Generator().manual_seed(0)
    BH, S, Nkv, C = 16 * 8, 9216 * 4, 9216, 32
    ii = torch.arange(96).float()
    ys, xs = torch.meshgrid(ii, ii, indexing="ij")
    kv = torch.stack([xs, ys], -1).reshape(1, -1, 2).expand(BH, -1, -1).contiguous()
    sl = torch.rand((BH, S, 2), generator=g) * 96 - 0.5
    nb = (sl.round().clamp(0, 95)[..., 1:2] * 96 + sl.round().clamp(0, 95)[..., 0:1]).long()
    nb = torch.cat([nb, (nb + 1) % Nkv, (nb + 96) % Nkv, (nb + 97) % Nkv], -1)
    aw = torch.rand((BH, S), generator=g)
    val = torch.randn((BH, Nkv, C), generator=g)
    dout = torch.randn((BH, S, C), generator=g).to("cuda", torch.bfloat16)
    leaves = [t.to("cuda").requires_grad_(True) for t in (sl, kv)]
    awc = aw.to("cuda").requires_grad_(True)
    vc = val.to("cuda", torch.bfloat16).requires_grad_(True)
    nbc = nb.to("cuda").int()
    power = torch.tensor(1.0, device="cuda", requires_grad=True)

    def step():
        FusedDeformAttnFunction.apply(leaves[0], leaves[1], nbc, power, awc, vc, 2, None).backward(dout)
    fwd = _nbytes(sl, kv, nbc, aw) + _nbytes(vc, dout)
    bwd = _nbytes(dout, sl, kv, nbc, aw, vc) + _nbytes(sl, kv, aw, vc)
    return step, fwd + bwd, {"BH": BH, "samples": S, "Nkv": Nkv, "C": C, "pass": "fwd+bwd"}


OPS = {"knn": op_knn, "knn-brute": lambda: op_knn(brute=True), "deform": op_deform, "deform-mae": op_deform_mae,
       "deform-mae-raster": lambda: op_deform_mae(raster=True),
       "layer-norm-dec": lambda: op_layer_norm(C=384), "res-norm": op_residual_norm,
       "res-norm-s3": lambda: op_residual_norm(R=16 * 5243, C=384), "wfeat": op_wfeat,
       "wfeat-fwd": lambda: op_wfeat(fwd_only=True),
       "wfeat-lists": lambda: op_wfeat(lists=True), "wfeat-lists-fwd": lambda: op_wfeat(fwd_only=True, lists=True),
       "wgather": op_wgather, "layer-norm": op_layer_norm, "rel-bias": op_rel_bias,
       "head-layout": op_head_layout, "deform-nbidx": op_deform_nbidx, "tile-union": None}


def op_tile_union():
    """Config 3 lists (curve order): distinct key clusters per tile of T
    consecutive queries, i.e. the pairs a query-tiled kernel computes against
    the 48 listed per query, for the tile heights of mma.sync (16) and of
    tcgen05 (64 / 128 rows).  Host only."""
    from .workloads import clustered_tokens, neighbourhoods, tile_union
    member, _ = neighbourhoods(clustered_tokens(4, 96, 0.5, 0, "cpu"), 8, 48)
    for t in (8, 16, 32, 64, 128):
        u = tile_union(member, t)
        print(json.dumps({"op": "tile-union", "tile_queries": t, "clusters": round(u, 2), "keys": round(8 * u, 1),
                          "computed_per_listed": round(8 * u / 48, 2)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=sorted(OPS))
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    if a.op == "tile-union":
        op_tile_union()
        return
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    fn, nbytes, cfg = OPS[a.op]()
    ms = _time(fn, a.iters, flush)
    print(json.dumps({"op": a.op, "ms": ms, "algorithmic_bytes": nbytes, "GB_per_s": nbytes / ms / 1e6,
                      "config": cfg}), flush=True)


if __name__ == "__main__":
    main()
