"""Generate module-level golden vectors from the reference's own layer modules.

Runs the reference's unchanged ``ClusterAttention``,
``DeformableCrossAttention`` and ``DeformableSelfAttention``
(src/layers/attention.py:20-207, :210-404, :407-593) and ``ClusterMerging``
(src/layers/aff.py:120-299), BasicLayer (aff.py:330-510) and MSDecoderBlock
(src/layers/decoder.py:73-143) on the CPU with their
Triton kernels under ``TRITON_INTERPRET=1``, with seeded random parameters
and inputs, and stores parameters, inputs, outputs and every gradient in
``tests/golden/module_*.npz``.  ``tests/test_module_parity.py`` loads the same
parameters into this package's modules (affmae_b200.mae) and compares on the
GPU.  The reference's ``src/layers/kernels/util.py`` queries a GPU driver at
import and is replaced by a stub; the reference packages' ``__init__`` files
are skipped.

Usage:  python tests/golden/make_module_golden.py --reference /path/to/affmae
        (or AFFMAE_REFERENCE=/path/to/affmae python tests/golden/make_module_golden.py)
"""
from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def load_attention(root: str):
    def pkg(name, path):
        m = types.ModuleType(name)
        m.__path__ = [path]
        sys.modules[name] = m
    pkg("src", f"{root}/src")
    pkg("src.layers", f"{root}/src/layers")
    pkg("src.layers.kernels", f"{root}/src/layers/kernels")
    pkg("src.utils", f"{root}/src/utils")
    util = types.ModuleType("src.layers.kernels.util")
    util.NUM_STAGES_OPTIONS = [1, 2]
    util.is_hip = lambda: False
    util.is_cuda = lambda: True
    util.supports_host_descriptor = lambda: False
    sys.modules["src.layers.kernels.util"] = util
    # third-party imports of aff.py / geometry.py / decoder.py that the modules used here do
    # not call: pykeops (absent here) and timm's DropPath / trunc_normal_
    sys.modules.setdefault("pykeops", types.ModuleType("pykeops"))
    pk = types.ModuleType("pykeops.torch")
    pk.LazyTensor = None
    sys.modules.setdefault("pykeops.torch", pk)
    if "timm" not in sys.modules:
        layers = types.ModuleType("timm.models.layers")
        layers.DropPath = lambda p=0.0: torch.nn.Identity()
        layers.trunc_normal_ = torch.nn.init.trunc_normal_
        for name, mod in [("timm", types.ModuleType("timm")), ("timm.models", types.ModuleType("timm.models")),
                          ("timm.models.layers", layers)]:
            sys.modules[name] = mod
    if "fvcore" not in sys.modules:  # imported by decoder.py, unused by its blocks
        for name in ("fvcore", "fvcore.nn", "fvcore.nn.weight_init"):
            sys.modules[name] = types.ModuleType(name)
        sys.modules["fvcore.nn"].weight_init = sys.modules["fvcore.nn.weight_init"]
    import src.layers.attention as attention  # noqa: E402
    return attention


def randomise(module: torch.nn.Module, g: torch.Generator, std: float = 0.2):
    """Every parameter drawn N(0, std) (the zero initialisations of the offset
    and weight projections would leave their gradients untested)."""
    with torch.no_grad():
        for p in module.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * std)


def save(name, module, **arrays):
    out = {f"param.{k}": v.detach().numpy() for k, v in module.named_parameters()}
    out.update({f"grad.{k}": v.grad.detach().numpy() for k, v in module.named_parameters() if v.grad is not None})
    out.update({k: (v.detach().numpy() if torch.is_tensor(v) else np.asarray(v)) for k, v in arrays.items()})
    np.savez_compressed(HERE / f"module_{name}.npz", **out)
    print(f"  wrote module_{name}.npz", flush=True)


def gen_cluster_attention(A):
    """64 tokens on an 8x8 grid in row order, clusters of 8 consecutive tokens,
    each token attending the 6 clusters with the nearest means (48 keys),
    relative-position indices as in BasicLayer.forward (aff.py:426-465)."""
    g = torch.Generator().manual_seed(11)
    m = A.ClusterAttention(64, 2)
    randomise(m, g)
    N, M = 64, 48
    ys, xs = torch.meshgrid(torch.arange(8.0), torch.arange(8.0), indexing="ij")
    pos = torch.stack([xs, ys], -1).reshape(1, N, 2)
    means = pos.view(1, 8, 8, 2).mean(2)
    d = ((pos[:, :, None] - means[:, None]) ** 2).sum(-1)
    near = torch.sort(d, dim=-1, stable=True)[1][..., :6]
    member = (near[..., None] * 8 + torch.arange(8)).reshape(1, N, M)
    nb = pos[0][member[0]][None]
    rel = (nb - (pos[:, :, None] - 127)).clamp(0, 254).long()
    pe_idx = rel[..., 1] * 255 + rel[..., 0]
    feat = torch.randn((1, N, 64), generator=g).requires_grad_(True)
    dout = torch.randn((1, N, 64), generator=g)
    out = m(feat, member, None, pe_idx, False)
    out.backward(dout)
    save("cluster_attention", m, feat=feat, member=member, pe_idx=pe_idx, dout=dout, out=out,
         d_feat=feat.grad, dim=64, heads=2)


def gen_deformable(A, cls, name):
    g = torch.Generator().manual_seed(12 if cls is A.DeformableCrossAttention else 13)
    m = cls(64, 2, 4)
    randomise(m, g)
    with torch.no_grad():
        m.shepard_power.fill_(1.3)
    Nq, Nkv = 24, 40
    query = torch.randn((1, Nq, 64), generator=g).requires_grad_(True)
    qpos = torch.rand((1, Nq, 2), generator=g) * 8
    dout = torch.randn((1, Nq, 64), generator=g)
    if cls is A.DeformableCrossAttention:
        kv = torch.randn((1, Nkv, 64), generator=g).requires_grad_(True)
        kpos = torch.rand((1, Nkv, 2), generator=g) * 8
        out = m(query, qpos, kv, kpos)
        out.backward(dout)
        save(name, m, query=query, query_pos=qpos, kv=kv, kv_pos=kpos, dout=dout, out=out, d_query=query.grad,
             d_kv=kv.grad, dim=64, heads=2)
    else:
        out = m(query, qpos)
        out.backward(dout)
        save(name, m, query=query, query_pos=qpos, dout=dout, out=out, d_query=query.grad, dim=64, heads=2)


def gen_cluster_merging(A, root):
    """ClusterMerging (aff.py:120-299) with the model's settings (cluster
    merging, no reserve tokens, ds_rate 0.4).  Its weighted_features wrapper
    asserts CUDA tensors (weighted_features.py:411), so the reference's own
    launchers one layer down (weighted_features_triton and its backward) are
    bound into an autograd Function for this CPU run."""
    import importlib
    aff = importlib.import_module("src.layers.aff")
    wf = importlib.import_module("src.layers.kernels.weighted_features")

    class WF(torch.autograd.Function):
        @staticmethod
        def forward(ctx, w, f, idx):
            ctx.save_for_backward(w, f, idx)
            return wf.weighted_features_triton(w, f, idx.to(torch.int32))

        @staticmethod
        def backward(ctx, dout):
            w, f, idx = ctx.saved_tensors
            dw, df = wf.weighted_features_triton_backward(dout.contiguous(), w, f, idx.to(torch.int32))
            return dw, df, None

    aff.weighted_features = WF.apply
    g = torch.Generator().manual_seed(14)
    m = aff.ClusterMerging(64, 96, ds_rate=0.4, reserve_on=False)
    randomise(m, g)
    with torch.no_grad():
        m.weight_net[1].weight.add_(1.0)
        m.norm.weight.add_(1.0)
    n, M = 80, 48
    ys, xs = torch.meshgrid(torch.arange(8.0), torch.arange(10.0), indexing="ij")
    pos = (torch.stack([xs, ys], -1).reshape(1, n, 2) * 2)
    means = pos.view(1, n // 8, 8, 2).mean(2)
    d = ((pos[:, :, None] - means[:, None]) ** 2).sum(-1)
    near = torch.sort(d, dim=-1, stable=True)[1][..., :6]
    member = (near[..., None] * 8 + torch.arange(8)).reshape(1, n, M)
    nb = pos[0][member[0]][None]
    rel = (nb - (pos[:, :, None] - 127)).clamp(0, 254).long()
    pe_idx = rel[..., 1] * 255 + rel[..., 0]
    feat = torch.randn((1, n, 64), generator=g).requires_grad_(True)
    prob = torch.sigmoid(torch.randn((1, n, 1), generator=g)).requires_grad_(True)
    pos_down, feat_down = m(pos, feat, member, None, prob, 2, pe_idx, 0)
    dout = torch.randn(feat_down.shape, generator=g)
    feat_down.backward(dout)
    save("cluster_merging", m, pos=pos, feat=feat, member=member, pe_idx=pe_idx, prob=prob, pos_down=pos_down,
         feat_down=feat_down, dout=dout, d_feat=feat.grad, d_prob=prob.grad, dim=64, out_dim=96, ds_rate=0.4)


def gen_stage(A, root):
    """One encoder stage, BasicLayer (aff.py:330-510): space-filling clustering,
    nearest-cluster neighbourhoods, two ClusterTransformerBlocks and
    ClusterMerging, on 102 tokens in a 16x16 canvas (a partial last cluster).
    The stage's KNN wrapper asserts CUDA tensors (knn.py:1384); it is bound to
    the oracle's exact KNN (the reference kernel's (distance, index) order,
    pinned by the KNN golden vectors) for this CPU run."""
    import importlib
    sys.path.insert(0, str(HERE.parent.parent))
    import oracle
    aff = importlib.import_module("src.layers.aff")
    aff.triton_knn = lambda q, r, k, **kw: oracle.knn(q, r, k)
    g = torch.Generator().manual_seed(15)
    m = aff.BasicLayer(64, 96, cluster_size=8, nbhd_size=48, depth=2, num_heads=2, mlp_ratio=2.0, ds_rate=0.4,
                       downsample=aff.ClusterMerging)
    randomise(m, g)
    with torch.no_grad():
        for mod in m.modules():
            if isinstance(mod, torch.nn.LayerNorm):
                mod.weight.add_(1.0)
    n = 102
    # positions off the grid: the clustering sorts a key in which symmetric
    # grid positions can tie, and the order of ties is left to the sort
    # implementation (it differs between devices in the reference as well)
    pos = torch.rand((1, n, 2), generator=g) * 16
    feat = torch.randn((1, n, 64), generator=g).requires_grad_(True)
    pos_o, feat_o, pos_down, feat_down = m(pos, feat, 16, 16, False, 2)
    d_o = torch.randn(feat_o.shape, generator=g)
    d_down = torch.randn(feat_down.shape, generator=g)
    torch.autograd.backward([feat_o, feat_down], [d_o, d_down])
    save("stage", m, pos=pos, feat=feat, pos_out=pos_o, feat_out=feat_o, pos_down=pos_down, feat_down=feat_down,
         d_out=d_o, d_down=d_down, d_feat=feat.grad, dim=64, out_dim=96, heads=2, depth=2, hw=16)


def gen_decoder_block(root):
    """One decoder block, MSDecoderBlock (decoder.py:73-143): deformable
    self-attention, deformable cross-attention into encoder features with
    their position embedding, ReLU FFN, post-norm residuals; no dropout."""
    import importlib
    dec = importlib.import_module("src.layers.decoder")
    g = torch.Generator().manual_seed(16)
    m = dec.MSDecoderBlock(d_model=64, n_heads=2, n_points=4, d_ffn=128, dropout=0.0)
    randomise(m, g)
    with torch.no_grad():
        for mod in m.modules():
            if isinstance(mod, torch.nn.LayerNorm):
                mod.weight.add_(1.0)
        for att in (m.self_attn, m.cross_attn):
            att.shepard_power.fill_(1.2)
    Nq, Ns = 24, 40
    query = torch.randn((1, Nq, 64), generator=g).requires_grad_(True)
    qpos = torch.rand((1, Nq, 2), generator=g) * 8
    src = torch.randn((1, Ns, 64), generator=g).requires_grad_(True)
    spos = torch.rand((1, Ns, 2), generator=g) * 8
    embed = torch.randn((1, Ns, 64), generator=g) * 0.5
    out = m(query, qpos, src, spos, embed)
    dout = torch.randn(out.shape, generator=g)
    out.backward(dout)
    save("decoder_block", m, query=query, query_pos=qpos, src=src, src_pos=spos, src_embed=embed, out=out,
         dout=dout, d_query=query.grad, d_src=src.grad, dim=64, heads=2, ffn=128)


def gen_global(A):
    """The global path of a stage with no more tokens than the neighbourhood
    size (aff.py:421-424, attention.py:157-180): ClusterAttention over all
    token pairs plus the blank token, and BasicLayer (one block, no merging)
    on 40 tokens in a 16x16 canvas."""
    import importlib
    aff = importlib.import_module("src.layers.aff")
    g = torch.Generator().manual_seed(17)
    m = A.ClusterAttention(64, 2)
    randomise(m, g)
    N = 40
    pos = torch.rand((1, N, 2), generator=g) * 16
    rel = ((pos[:, None, :, :] + 127) - pos[:, :, None, :]).clamp(0, 254)
    pe_idx = (rel[..., 1] * 255 + rel[..., 0]).long()
    feat = torch.randn((1, N, 64), generator=g).requires_grad_(True)
    dout = torch.randn((1, N, 64), generator=g)
    out = m(feat, torch.zeros((1, N, N), dtype=torch.long), None, pe_idx, True)  # the list is not read
    out.backward(dout)
    save("cluster_attention_global", m, feat=feat, pe_idx=pe_idx, dout=dout, out=out, d_feat=feat.grad, dim=64,
         heads=2)
    st = aff.BasicLayer(64, None, cluster_size=8, nbhd_size=48, depth=1, num_heads=2, mlp_ratio=2.0)
    randomise(st, g)
    with torch.no_grad():
        for mod in st.modules():
            if isinstance(mod, torch.nn.LayerNorm):
                mod.weight.add_(1.0)
    feat = torch.randn((1, N, 64), generator=g).requires_grad_(True)
    pos_o, feat_o, _, _ = st(pos, feat, 16, 16, False, 2)
    d_o = torch.randn(feat_o.shape, generator=g)
    feat_o.backward(d_o)
    save("stage_global", st, pos=pos, feat=feat, pos_out=pos_o, feat_out=feat_o, d_out=d_o, d_feat=feat.grad,
         dim=64, heads=2, depth=1, hw=16)


MODEL_CFG = dict(img_size=100, patch_size=4, mask_ratio=0.488, embed_dims=(32, 32, 64, 64),
                 depths=(2, 1, 1, 1), num_heads=(1, 1, 2, 2), decoder_dim=64, decoder_heads=2)


def bind_cpu_wrappers(aff):
    """Bind the two CUDA-asserting wrappers the encoder calls for a CPU run:
    ``weighted_features`` (weighted_features.py:411) to the reference's own
    launchers one layer down, ``knn`` (knn.py:1384) to the oracle's exact KNN
    (the reference kernel's (distance, index) order, pinned by the KNN golden
    vectors)."""
    import importlib
    sys.path.insert(0, str(HERE.parent.parent))
    import oracle
    wf = importlib.import_module("src.layers.kernels.weighted_features")

    class WF(torch.autograd.Function):
        @staticmethod
        def forward(ctx, w, f, idx):
            ctx.save_for_backward(w, f, idx)
            return wf.weighted_features_triton(w, f, idx.to(torch.int32))

        @staticmethod
        def backward(ctx, dout):
            w, f, idx = ctx.saved_tensors
            dw, df = wf.weighted_features_triton_backward(dout.contiguous(), w, f, idx.to(torch.int32))
            return dw, df, None

    aff.weighted_features = WF.apply
    aff.triton_knn = lambda q, r, k, **kw: oracle.knn(q, r, k)


def gen_model(root, seeds=range(40, 60)):
    """The whole masked autoencoder, AFFMaskedAutoEncoder (aff_mae.py:26-205)
    with cluster merging, at a reduced size: one 100 x 100 image, patch 4, a
    25 x 25 token canvas with 320 visible tokens -> 128 -> 51 -> 20 (stages 1-3
    attend locally, the last one partially filled clusters, stage 4 globally)
    and 305 masked-patch queries; decoder width 64; the reference's own
    initialisation; eval mode (no dropout); fp32; loss and every parameter
    gradient.  The sizes keep the reference's decoder, whose deformable kernels
    scan every key per sample, to minutes under the interpreter.

    The token mask is an input: the reference draws it from Perlin noise (an
    absent package), so its masking call is given the split of a stored noise
    tensor, with the masked ids in raster order (the order this package's
    decoder uses; the loss does not depend on it).

    Two decision boundaries are pinned so that the comparison does not sit
    on one.  (1) The clustering sorts a key in which grid positions tie (the
    perpendicular bisector of two anchors, mirror images across an anchor
    row) and the order of tied tokens is left to the sort implementation: the
    order the reference chose at every stage is stored (``stage{i}.pos``, the
    positions in cluster order) for the comparison to follow within tied
    runs.  (2) A seed is kept only if each merging's importance top-k has a
    gap above 2e-3 between the last kept and the first dropped score (the
    reference rounds attention outputs through fp16, which moves the scores
    by about 1e-4); that is checked on the encoder alone before the full
    run."""
    import importlib
    for name in ("perlin_noise", "cv2", "matplotlib", "matplotlib.pyplot"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["perlin_noise"].perlin_noise = None
    sys.modules["matplotlib"].pyplot = sys.modules["matplotlib.pyplot"]
    m = types.ModuleType("src.models")
    m.__path__ = [f"{root}/src/models"]
    sys.modules["src.models"] = m
    aff = importlib.import_module("src.layers.aff")
    mae_ref = importlib.import_module("src.models.aff_mae")
    bind_cpu_wrappers(aff)
    rec = {"pos": [], "gaps": []}
    cluster = aff.space_filling_cluster

    def recorded_cluster(pos, *a, **kw):
        out = cluster(pos, *a, **kw)
        rec["pos"].append(out[0].detach().clone())
        return out

    aff.space_filling_cluster = recorded_cluster
    merge_fwd = aff.ClusterMerging.forward

    def checked_merge(self, pos, feat, member_idx, cluster_mask, learned_prob, *a, **kw):
        lp = learned_prob.detach().view(feat.shape[0], -1).sort(dim=1, descending=True).values
        keep = int(feat.shape[1] * self.ds_rate)
        rec["gaps"].append((lp[:, keep - 1] - lp[:, keep]).min().item())
        return merge_fwd(self, pos, feat, member_idx, cluster_mask, learned_prob, *a, **kw)

    aff.ClusterMerging.forward = checked_merge
    c = MODEL_CFG
    L = (c["img_size"] // c["patch_size"]) ** 2
    keep = int(L * (1 - c["mask_ratio"]))
    for seed in seeds:
        torch.manual_seed(seed)
        g = torch.Generator().manual_seed(seed)
        model = mae_ref.AFFMaskedAutoEncoder(
            patch_size=c["patch_size"], img_size=c["img_size"], in_channels=1, mask_ratio=c["mask_ratio"],
            encoder_embed_dim=list(c["embed_dims"]), encoder_depth=list(c["depths"]),
            encoder_num_heads=list(c["num_heads"]), encoder_nbhd_size=[48] * 4, cluster_size=8,
            ds_rate=[0.4] * 4, decoder_embed_dim=c["decoder_dim"], decoder_num_heads=c["decoder_heads"],
            mlp_ratio=2, merging_method="cluster").eval()
        imgs = torch.randn((1, 1, c["img_size"], c["img_size"]), generator=g)
        noise = torch.rand((1, L), generator=g)

        def masking(x, img_size, patch, ratio, noise=noise):
            ids = noise.argsort(dim=1)
            return ids[:, :keep], ids[:, keep:].sort(dim=1).values, ids.argsort(dim=1)

        mae_ref.perlin_masking = masking
        rec["pos"], rec["gaps"] = [], []
        with torch.no_grad():
            model.forward_encoder(imgs)
        print(f"  seed {seed}: stage sizes {[p.shape[1] for p in rec['pos']]}, "
              f"top-k gaps {['%.1e' % x for x in rec['gaps']]}", flush=True)
        if min(rec["gaps"]) > 2e-3:
            break
    else:
        raise RuntimeError("no seed with top-k margins")
    rec["pos"], rec["gaps"] = [], []
    loss, losses = model(imgs)
    loss.backward()
    out = {f"param.{k}": v.detach().numpy() for k, v in model.named_parameters()}
    out.update({f"grad.{k}": v.grad.detach().numpy() for k, v in model.named_parameters() if v.grad is not None})
    out.update({f"stage{i}.pos": p.numpy() for i, p in enumerate(rec["pos"])})
    out.update(images=imgs.numpy(), noise=noise.numpy(), loss=loss.detach().numpy(),
               losses=torch.stack(losses).detach().numpy(), seed=seed, topk_gap=min(rec["gaps"]))
    out.update({f"cfg.{k}": np.asarray(v) for k, v in c.items()})
    np.savez_compressed(HERE / "module_model.npz", **out)
    print("  wrote module_model.npz", flush=True)

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AFFMAE_REFERENCE"),
                    help="checkout of najafian-lab/affmae (or set AFFMAE_REFERENCE)")
    ap.add_argument("--only", choices=["modules", "model"], help="generate one of the two groups")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give the reference checkout with --reference or AFFMAE_REFERENCE")
    torch.set_num_threads(1)
    A = load_attention(a.reference)
    if a.only != "modules":
        gen_model(a.reference)
    if a.only == "model":
        return
    gen_cluster_attention(A)
    gen_deformable(A, A.DeformableCrossAttention, "deform_cross")
    gen_deformable(A, A.DeformableSelfAttention, "deform_self")
    gen_cluster_merging(A, a.reference)
    gen_stage(A, a.reference)
    gen_decoder_block(a.reference)
    gen_global(A)


if __name__ == "__main__":
    main()
