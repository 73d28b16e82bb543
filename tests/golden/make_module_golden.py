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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AFFMAE_REFERENCE"),
                    help="checkout of najafian-lab/affmae (or set AFFMAE_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give the reference checkout with --reference or AFFMAE_REFERENCE")
    torch.set_num_threads(1)
    A = load_attention(a.reference)
    gen_cluster_attention(A)
    gen_deformable(A, A.DeformableCrossAttention, "deform_cross")
    gen_deformable(A, A.DeformableSelfAttention, "deform_self")
    gen_cluster_merging(A, a.reference)
    gen_stage(A, a.reference)
    gen_decoder_block(a.reference)
    gen_global(A)


if __name__ == "__main__":
    main()
