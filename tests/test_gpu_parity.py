"""Parity of the CUDA operators (through the C ABI) with the CPU oracle and the
reference's golden vectors.

Tolerances (relative error = max|a-b| / max|b| per tensor):
  KNN indices: bit-exact;  fp32 forward: 1e-5;  atomics-based backward: 1e-4;
  bf16/fp16 inputs: 2e-2 against the oracle evaluated on the rounded inputs.
The reference stores the local-attention output through fp16
(local_attn.py:340), so its golden O is compared at 2e-3.
"""
import pytest
import torch

import oracle
from conftest import golden, rel_err

pytestmark = pytest.mark.gpu

TOL_F32, TOL_BWD, TOL_LP = 1e-5, 1e-4, 2e-2


def dev(t, device, dtype=None):
    t = t.to(device)
    return t.to(dtype) if dtype is not None else t


# ----------------------------------------------------------------------- KNN
@pytest.mark.parametrize("tag", ["d2_k4", "d2_k8_grid", "d3_k6", "d2_k3_grid"])
def test_knn_golden(cuda, tag):
    from affmae_b200.kernels.knn import knn
    g = golden(f"knn_{tag}")
    idx = knn(dev(g["query"], cuda), dev(g["ref"], cuda), int(g["k"]))
    assert idx.dtype == torch.int64
    assert torch.equal(idx.cpu(), g["idx"])


@pytest.fixture(params=["brute", "grid"])
def knn_path(request):
    """Runs a KNN test through the brute-force scan and through the 2-D grid search."""
    import affmae_b200.kernels.knn as kmod
    old = kmod.GRID_MIN_POINTS, kmod.GRID_MIN_PAIRS
    if request.param == "grid":
        kmod.GRID_MIN_POINTS, kmod.GRID_MIN_PAIRS = 1, 0
    else:
        kmod.GRID_MIN_POINTS = 1 << 40
    yield request.param
    kmod.GRID_MIN_POINTS, kmod.GRID_MIN_PAIRS = old


@pytest.mark.parametrize("K", [1, 6, 16, 33, 48, 100, 256])
@pytest.mark.parametrize("D", [2, 3, 4])
def test_knn_random_exact(cuda, K, D, knn_path):
    from affmae_b200.kernels.knn import knn
    gen = torch.Generator().manual_seed(K * 10 + D)
    q = torch.rand((2, 301, D), generator=gen) * 50
    r = torch.rand((2, 2600, D), generator=gen) * 50
    idx = knn(q.to(cuda), r.to(cuda), K)
    assert torch.equal(idx.cpu(), oracle.knn(q, r, K))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_knn_ties_and_low_precision(cuda, dtype, knn_path):
    from affmae_b200.kernels.knn import knn
    gen = torch.Generator().manual_seed(7)
    q = torch.randint(0, 20, (3, 200, 2), generator=gen).to(dtype)
    r = torch.randint(0, 20, (3, 500, 2), generator=gen).to(dtype)
    idx = knn(q.to(cuda), r.to(cuda), 48)
    assert torch.equal(idx.cpu(), oracle.knn(q.float(), r.float(), 48))


def test_knn_baseline_config_sweep(cuda):
    """Config 2 shapes: 96x96 stride-4 lattice jittered, B=8, N=2304 (self and 0.25N queries)."""
    from affmae_b200.kernels.knn import knn
    gen = torch.Generator().manual_seed(0)
    ys, xs = torch.meshgrid(torch.arange(48.), torch.arange(48.), indexing="ij")
    grid = torch.stack([xs, ys], -1).reshape(1, -1, 2) * 2
    pos = (grid + torch.rand((8, grid.shape[1], 2), generator=gen) - 0.5).float()
    for K in (16, 48):
        idx = knn(pos.to(cuda), pos.to(cuda), K)
        assert torch.equal(idx.cpu(), oracle.knn(pos, pos, K))
        qd = pos[:, : pos.shape[1] // 4]
        idx = knn(qd.to(cuda), pos.to(cuda), K)
        assert torch.equal(idx.cpu(), oracle.knn(qd, pos, K))


def test_knn_errors(cuda):
    from affmae_b200.kernels.knn import knn
    q = torch.rand((1, 4, 2), device=cuda)
    with pytest.raises(AssertionError):
        knn(q, q, 5)


# ------------------------------------------------------- neighbourhood attention
def _attn_inputs(B, H, N, D, M, dtype, mask=True, blank=True, bias=True, seed=0, cuda=None):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn((B, H, N, D), generator=gen) / D ** 0.5
    k = torch.randn((B, H, N, D), generator=gen) / D ** 0.5
    v = torch.randn((B, H, N, D), generator=gen) / D ** 0.5
    mi = torch.randint(0, N, (B, N, M), generator=gen, dtype=torch.int32)
    b = torch.randn((B, H, N, M), generator=gen) * 0.5 if bias else None
    m = (torch.rand((B, 1, N, M), generator=gen) > 0.2) if mask else None
    bk = torch.randn((H, D), generator=gen) * 0.2 if blank else None
    bv = torch.randn((H, D), generator=gen) * 0.2 if blank else None
    do = torch.randn((B, H, N, D), generator=gen)
    cast = lambda t: None if t is None else t.to(dtype)
    return dict(q=cast(q), k=cast(k), v=cast(v), mi=mi, bias=cast(b), mask=m, blank_k=cast(bk),
                blank_v=cast(bv), do=cast(do))


def _to(d, device):
    return {k: (None if v is None else v.to(device)) for k, v in d.items()}


@pytest.mark.parametrize("tag", ["full", "plain", "m24"])
def test_local_attn_golden(cuda, tag):
    from affmae_b200.kernels.local_attn import launch_flash_nbhood_attn_fwd, launch_flash_nbhood_attn_bwd
    g = golden(f"local_attn_{tag}")
    G = _to(g, cuda)
    kw = dict(bias=G.get("bias"), mask=G.get("mask"), blank_k=G.get("blank_k"), blank_v=G.get("blank_v"))
    scale = float(g["scale"])
    o, lse = launch_flash_nbhood_attn_fwd(G["q"], G["k"], G["v"], G["mi"], scale, **kw)
    assert rel_err(lse.cpu(), g["lse"]) < TOL_F32
    assert rel_err(o.cpu(), g["o"]) < 2e-3
    okw = dict(bias=g.get("bias"), mask=g.get("mask"), blank_k=g.get("blank_k"), blank_v=g.get("blank_v"))
    o_ref, _ = oracle.nbhd_attn_fwd(g["q"], g["k"], g["v"], g["mi"], scale, **okw)
    assert rel_err(o.cpu(), o_ref) < TOL_F32
    # backward from the reference's stored O (fp16-rounded) reproduces its grads
    dq, dk, dv, dbias, dbk, dbv = launch_flash_nbhood_attn_bwd(G["q"], G["k"], G["v"], G["mi"], scale,
                                                               G["o"], G["lse"], G["do"], **kw)
    for name, a in [("dq", dq), ("dk", dk), ("dv", dv), ("dbias", dbias), ("dbk", dbk), ("dbv", dbv)]:
        if name in g:
            assert rel_err(a.cpu(), g[name]) < TOL_BWD, name


@pytest.mark.parametrize("dtype,tol", [(torch.float32, TOL_F32), (torch.bfloat16, TOL_LP),
                                       (torch.float16, TOL_LP)])
@pytest.mark.parametrize("opts", [dict(), dict(mask=False), dict(blank=False, bias=False),
                                  dict(mask=False, blank=False, bias=False)])
@pytest.mark.parametrize("shape", [(2, 4, 200, 32, 48), (1, 3, 77, 64, 16), (1, 2, 40, 8, 8),
                                   (1, 2, 33, 128, 24)])
def test_local_attn_random(cuda, dtype, tol, opts, shape):
    from affmae_b200.kernels.local_attn import launch_flash_nbhood_attn_fwd, launch_flash_nbhood_attn_bwd
    B, H, N, D, M = shape
    inp = _attn_inputs(B, H, N, D, M, dtype, seed=sum(shape), **opts)
    G = _to(inp, cuda)
    kw = lambda d: dict(bias=d["bias"], mask=d["mask"], blank_k=d["blank_k"], blank_v=d["blank_v"])
    scale = D ** -0.5
    o, lse = launch_flash_nbhood_attn_fwd(G["q"], G["k"], G["v"], G["mi"], scale, **kw(G))
    assert o.dtype == dtype
    o_ref, lse_ref = oracle.nbhd_attn_fwd(inp["q"], inp["k"], inp["v"], inp["mi"], scale, **kw(inp))
    assert rel_err(o.cpu(), o_ref) < tol
    assert rel_err(lse.cpu(), lse_ref) < max(tol, TOL_F32)
    grads = launch_flash_nbhood_attn_bwd(G["q"], G["k"], G["v"], G["mi"], scale, o, lse, G["do"], **kw(G))
    ref = oracle.nbhd_attn_bwd(inp["q"], inp["k"], inp["v"], inp["mi"], scale, o.cpu(), lse.cpu(),
                               inp["do"], **kw(inp))
    btol = TOL_BWD if dtype == torch.float32 else TOL_LP
    for name, a, b in zip(["dq", "dk", "dv", "dbias", "dbk", "dbv"], grads, ref):
        assert (a is None) == (b is None), name
        if a is not None:
            assert a.dtype == dtype
            assert rel_err(a.cpu(), b) < btol, name


def test_local_attn_autograd_function(cuda):
    from affmae_b200.kernels.local_attn import FlashLocalAttentionFunction
    inp = _attn_inputs(2, 4, 64, 32, 48, torch.float32, seed=3)
    G = _to(inp, cuda)
    leaves = {n: G[n].clone().requires_grad_() for n in ("q", "k", "v", "bias", "blank_k", "blank_v")}
    out = FlashLocalAttentionFunction.apply(leaves["q"], leaves["k"], leaves["v"], G["mi"].long(),
                                            leaves["bias"], G["mask"], leaves["blank_k"],
                                            leaves["blank_v"], 32 ** -0.5)
    out.backward(G["do"])
    ref_leaves = {n: inp[n].double().requires_grad_() for n in leaves}
    ref = oracle.nbhd_attn_formula(ref_leaves["q"], ref_leaves["k"], ref_leaves["v"], inp["mi"], 32 ** -0.5,
                                   bias=ref_leaves["bias"], mask=inp["mask"], blank_k=ref_leaves["blank_k"],
                                   blank_v=ref_leaves["blank_v"])
    ref.backward(inp["do"].double())
    assert rel_err(out.detach().cpu(), ref.detach()) < TOL_F32
    for n in leaves:
        assert rel_err(leaves[n].grad.cpu(), ref_leaves[n].grad) < TOL_BWD, n


# --------------------------------------------------------- weighted features
def test_weighted_features_golden(cuda):
    from affmae_b200.kernels.weighted_features import weighted_features_fwd, weighted_features_bwd
    g = golden("weighted_features")
    G = _to(g, cuda)
    assert rel_err(weighted_features_fwd(G["w"], G["feat"], G["idx"]).cpu(), g["out"]) < TOL_F32
    dw, df = weighted_features_bwd(G["dout"], G["w"], G["feat"], G["idx"])
    assert rel_err(dw.cpu(), g["dw"]) < TOL_F32
    assert rel_err(df.cpu(), g["dfeat"]) < TOL_BWD


def test_weighted_gather_golden(cuda):
    from affmae_b200.kernels.weighted_gather import WeightedGatherFunction
    g = golden("weighted_gather")
    G = _to(g, cuda)
    w = G["w"].clone().requires_grad_()
    f = G["feat"].clone().requires_grad_()
    out = WeightedGatherFunction.apply(G["idx"], w, f)
    assert rel_err(out.detach().cpu(), g["out"]) < TOL_F32
    out.backward(G["dout"])
    assert rel_err(w.grad.cpu(), g["dw"]) < TOL_F32
    assert rel_err(f.grad.cpu(), g["dfeat"]) < TOL_BWD


@pytest.mark.parametrize("dtype,tol", [(torch.float32, TOL_F32), (torch.bfloat16, TOL_LP), (torch.float16, TOL_LP)])
@pytest.mark.parametrize("shape", [(2, 300, 48, 4, 700, 96), (2, 100, 48, 1, 4096, 128), (1, 50, 7, 3, 60, 13),
                                   (1, 20, 40, 9, 30, 24), (1, 33, 17, 8, 50, 16), (1, 40, 5, 2, 64, 80),
                                   (1, 10, 48, 4, 100, 384), (1, 7, 1, 3, 9, 32)])
def test_weighted_features_random(cuda, dtype, tol, shape):
    from affmae_b200.kernels.weighted_features import weighted_features_fwd, weighted_features_bwd
    B, No, M, IC, N, C = shape
    gen = torch.Generator().manual_seed(sum(shape))
    w = torch.randn((B, No, M, IC), generator=gen).to(dtype)
    f = torch.randn((B, N, C), generator=gen).to(dtype)
    idx = torch.randint(0, N, (B, No, M), generator=gen, dtype=torch.int32)
    do = torch.randn((B, No, IC, C), generator=gen).to(dtype)
    out = weighted_features_fwd(w.to(cuda), f.to(cuda), idx.to(cuda))
    assert rel_err(out.cpu(), oracle.weighted_features_fwd(w, f, idx)) < tol
    dw, df = weighted_features_bwd(do.to(cuda), w.to(cuda), f.to(cuda), idx.to(cuda))
    rdw, rdf = oracle.weighted_features_bwd(do, w, f, idx)
    assert rel_err(dw.cpu(), rdw) < tol
    assert rel_err(df.cpu(), rdf) < (TOL_BWD if dtype == torch.float32 else tol)


def test_baseline_config1_chain(cuda):
    """Config 1: KNN(K=48) -> 4-head neighbourhood attention -> weighted gather to M=1024 (fp32)."""
    from affmae_b200.kernels.knn import knn
    from affmae_b200.kernels.local_attn import launch_flash_nbhood_attn_fwd
    from affmae_b200.kernels.weighted_gather import weighted_gather
    gen = torch.Generator().manual_seed(0)
    B, N, C, K, H = 2, 4096, 128, 48, 4
    pos = torch.rand((B, N, 2), generator=gen) * 64
    x = torch.randn((B, N, C), generator=gen)
    w = torch.softmax(torch.randn((B, 1024, K), generator=gen), -1)
    idx = knn(pos.to(cuda), pos.to(cuda), K)
    ridx = oracle.knn(pos, pos, K)
    assert torch.equal(idx.cpu(), ridx)
    xh = x.view(B, N, H, C // H).permute(0, 2, 1, 3).contiguous()
    o, _ = launch_flash_nbhood_attn_fwd(xh.to(cuda), xh.to(cuda), xh.to(cuda), idx, (C // H) ** -0.5)
    ro, _ = oracle.nbhd_attn_fwd(xh, xh, xh, ridx, (C // H) ** -0.5)
    assert rel_err(o.cpu(), ro) < TOL_F32
    y = o.permute(0, 2, 1, 3).reshape(B, N, C)
    out = weighted_gather(idx[:, :1024], w.to(cuda), y)
    rout = oracle.weighted_features_fwd(w[..., None], ro.permute(0, 2, 1, 3).reshape(B, N, C), ridx[:, :1024])[:, :, 0]
    assert rel_err(out.cpu(), rout) < TOL_F32


# ------------------------------------------------------ deformable attention
@pytest.mark.parametrize("tag", ["cross", "cross_grid"])
def test_deform_cross_golden(cuda, tag):
    from affmae_b200.kernels.fused_deform_attn import (fused_knn_deform_cross_attn_forward_save,
                                                       fused_knn_deform_cross_attn_backward)
    g = golden(f"deform_{tag}")
    G = _to(g, cuda)
    out, ki, kd = fused_knn_deform_cross_attn_forward_save(G["qpos"], G["kvpos"], G["off"], G["aw"], G["val"],
                                                           G["power"])
    assert torch.equal(ki.cpu(), g["knn_idx"])
    assert torch.equal(kd.cpu(), g["knn_d2"])
    assert rel_err(out.cpu(), g["out"]) < TOL_F32
    grads = fused_knn_deform_cross_attn_backward(G["dout"], G["qpos"], G["kvpos"], G["off"], G["aw"], G["val"],
                                                 G["power"], ki, kd)
    for name, a in zip(["d_qpos", "d_kvpos", "d_off", "d_aw", "d_val", "d_power"], grads):
        assert rel_err(a.cpu(), g[name]) < TOL_BWD, name


def test_deform_self_golden(cuda):
    from affmae_b200.kernels.fused_deform_attn import FusedKNNDeformSelfAttnFunction
    g = golden("deform_self")
    G = _to(g, cuda)
    leaves = [G[n].clone().requires_grad_() for n in ("pos", "off", "aw", "val", "power")]
    out = FusedKNNDeformSelfAttnFunction.apply(*leaves, 2)
    assert rel_err(out.detach().cpu(), g["out"]) < TOL_F32
    out.backward(G["dout"])
    for name, t in zip(["d_pos", "d_off", "d_aw", "d_val", "d_power"], leaves):
        assert rel_err(t.grad.cpu(), g[name].reshape(t.shape)) < TOL_BWD, name


def _deform_inputs(B, Nq, kv_side, H, C, dtype, seed, integer=False):
    gen = torch.Generator().manual_seed(seed)
    ys, xs = torch.meshgrid(torch.arange(float(kv_side)), torch.arange(float(kv_side)), indexing="ij")
    kv = torch.stack([xs, ys], -1).reshape(1, -1, 2).expand(B, -1, -1).clone()
    if not integer:
        kv = kv + (torch.rand(kv.shape, generator=gen) - 0.5) * 0.8
    qp = torch.rand((B, Nq, 2), generator=gen) * kv_side
    off = torch.randn((B, Nq, H, 4, 2), generator=gen) * 2
    if integer:
        qp = qp.floor()
        off = off.round()
    aw = torch.softmax(torch.randn((B, Nq, H, 4), generator=gen), -1)
    val = torch.randn((B, kv.shape[1], H, C), generator=gen).to(dtype)
    do = torch.randn((B, Nq, H, C), generator=gen).to(dtype)
    return qp, kv, off, aw, val, torch.tensor(1.7), do


@pytest.mark.parametrize("dtype,tol", [(torch.float32, TOL_F32), (torch.bfloat16, TOL_LP)])
@pytest.mark.parametrize("integer", [False, True])
@pytest.mark.parametrize("H,C", [(8, 32), (6, 64), (3, 16)])
def test_deform_cross_random(cuda, dtype, tol, integer, H, C):
    from affmae_b200.kernels.fused_deform_attn import (fused_knn_deform_cross_attn_forward_save,
                                                       fused_knn_deform_cross_attn_backward)
    qp, kv, off, aw, val, power, do = _deform_inputs(2, 300, 40, H, C, dtype, seed=H * C, integer=integer)
    args = [t.to(cuda) for t in (qp, kv, off, aw, val, power)]
    out, ki, kd = fused_knn_deform_cross_attn_forward_save(*args)
    rout, ridx, rd2 = oracle.deform_knn_fwd(qp, kv, off, aw, val, power)
    assert torch.equal(ki.cpu().long(), ridx)
    assert torch.equal(kd.cpu(), rd2)
    assert rel_err(out.cpu(), rout) < tol
    grads = fused_knn_deform_cross_attn_backward(do.to(cuda), *args, ki, kd)
    rgrads = oracle.deform_knn_bwd(do, qp, kv, off, aw, val, power, ridx, rd2)
    btol = TOL_BWD if dtype == torch.float32 else tol
    for name, a, b in zip(["d_qpos", "d_kvpos", "d_off", "d_aw", "d_val", "d_power"], grads, rgrads):
        assert rel_err(a.cpu(), b) < btol, name


def test_deform_far_samples_and_duplicates(cuda):
    """Samples far outside the kv bounding box and duplicated kv positions."""
    from affmae_b200.kernels.fused_deform_attn import fused_knn_deform_cross_attn_forward_save
    qp, kv, off, aw, val, power, _ = _deform_inputs(1, 64, 10, 2, 8, torch.float32, seed=5)
    off = off * 40
    kv[:, 50:60] = kv[:, 10:20]
    out, ki, kd = fused_knn_deform_cross_attn_forward_save(*[t.to(cuda) for t in (qp, kv, off, aw, val, power)])
    rout, ridx, rd2 = oracle.deform_knn_fwd(qp, kv, off, aw, val, power)
    assert torch.equal(ki.cpu().long(), ridx)
    assert rel_err(out.cpu(), rout) < TOL_F32


def test_deform_nbidx_golden(cuda):
    from affmae_b200.kernels.fused_deform_attn import FusedDeformAttnFunction
    g = golden("deform_nbidx")
    G = _to(g, cuda)
    leaves = {n: G[n].clone().requires_grad_() for n in ("sl", "kvpos", "power", "aw", "val")}
    out = FusedDeformAttnFunction.apply(leaves["sl"], leaves["kvpos"], G["nb"], leaves["power"], leaves["aw"],
                                        leaves["val"], 2, None)
    assert rel_err(out.detach().cpu(), g["out"]) < TOL_F32
    out.backward(G["dout"])
    for name, key in [("d_sl", "sl"), ("d_kvpos", "kvpos"), ("d_power", "power"), ("d_aw", "aw"), ("d_val", "val")]:
        assert rel_err(leaves[key].grad.cpu(), g[name]) < TOL_BWD, name


def test_mssample_golden(cuda):
    from affmae_b200.kernels.mssample import MSSampleFunction
    g = golden("mssample")
    G = _to(g, cuda)
    sl = G["sl"].clone().requires_grad_()
    kv = G["kvpos"].clone().requires_grad_()
    p = G["power"].clone().requires_grad_()
    w = MSSampleFunction.apply(sl, kv, G["nb"], p, 2)
    assert rel_err(w.detach().cpu(), g["w"]) < TOL_F32
    w.backward(G["dw"])
    assert rel_err(sl.grad.cpu(), g["d_sl"]) < TOL_BWD
    assert rel_err(kv.grad.cpu(), g["d_kvpos"]) < TOL_BWD
    assert rel_err(p.grad.cpu(), g["d_power"]) < TOL_BWD


def test_msdetrpc_golden(cuda):
    from affmae_b200.kernels.msdetrpc import MSDETRPCFunction
    g = golden("msdetrpc")
    G = _to(g, cuda)
    leaves = {n: G[n].clone().requires_grad_() for n in ("w", "attn", "val")}
    out = MSDETRPCFunction.apply(G["idx"], leaves["w"], leaves["attn"], leaves["val"])
    assert rel_err(out.detach().cpu(), g["out"]) < TOL_F32
    out.backward(G["dout"])
    for name, key in [("d_w", "w"), ("d_attn", "attn"), ("d_val", "val")]:
        assert rel_err(leaves[key].grad.cpu(), g[name]) < TOL_BWD, name


def test_pos_bias_gather(cuda):
    from affmae_b200.kernels.pos_bias import pos_bias_gather
    gen = torch.Generator().manual_seed(11)
    T, H, B, N, M = 255 * 255, 4, 2, 300, 48
    table = torch.randn((T, H), generator=gen)
    pe = torch.randint(0, T, (B, N, M), generator=gen)
    t = table.to(cuda).requires_grad_()
    out = pos_bias_gather(t, pe.to(cuda))
    assert torch.equal(out.detach().cpu(), oracle.pos_bias_fwd(table, pe).float())
    g = torch.randn((B, H, N, M), generator=gen)
    out.backward(g.to(cuda))
    assert rel_err(t.grad.cpu(), oracle.pos_bias_bwd(g, pe, T)) < TOL_BWD


@pytest.mark.parametrize("H", [4, 8, 12])
def test_pos_bias_gather_small_offsets(cuda, H):
    """Table gradient when the indices are the small relative offsets of
    neighbour lists (the shared-memory window around the table centre, and
    offsets just outside it), for head counts inside (4, 8) and beyond (12) the
    window kernel's limit."""
    from affmae_b200.kernels.pos_bias import pos_bias_gather
    gen = torch.Generator().manual_seed(12 + H)
    T, B, N, M = 255 * 255, 3, 257, 48
    d = torch.randint(-20, 21, (B, N, M, 2), generator=gen)
    pe = (d[..., 1] + 127) * 255 + d[..., 0] + 127
    table = torch.randn((T, H), generator=gen)
    t = table.to(cuda).requires_grad_()
    out = pos_bias_gather(t, pe.to(cuda))
    g = torch.randn((B, H, N, M), generator=gen)
    out.backward(g.to(cuda))
    assert rel_err(t.grad.cpu(), oracle.pos_bias_bwd(g, pe, T)) < TOL_BWD


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mask_heads", [0, 1, 4])
def test_local_attn_clustered_tensor_core_path(cuda, dtype, mask_heads):
    """Cluster-structured neighbourhoods (the model's and config 3's) take the
    tensor-core path; random neighbourhoods above take the CUDA-core fallback."""
    from affmae_b200.workloads import nbhd_attention_inputs
    from affmae_b200.kernels.local_attn import launch_flash_nbhood_attn_fwd, launch_flash_nbhood_attn_bwd
    inp = nbhd_attention_inputs(B=2, side=48, H=4, dtype=dtype, seed=mask_heads, device=cuda)
    B, H, N, D = inp["q"].shape
    M = inp["member_idx"].shape[-1]
    mask = None
    if mask_heads:
        gen = torch.Generator().manual_seed(9)
        mask = (torch.rand((B, mask_heads, N, M), generator=gen) > 0.15).to(cuda)
        mask[0, 0, 5] = False  # a fully masked row (blank token keeps it finite)
    kw = dict(bias=inp["bias"], mask=mask, blank_k=inp["blank_k"], blank_v=inp["blank_v"])
    o, lse = launch_flash_nbhood_attn_fwd(inp["q"], inp["k"], inp["v"], inp["member_idx"], inp["scale"], **kw)
    cpu = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in kw.items()}
    ro, rlse = oracle.nbhd_attn_fwd(inp["q"].cpu(), inp["k"].cpu(), inp["v"].cpu(), inp["member_idx"].cpu(),
                                    inp["scale"], **cpu)
    assert rel_err(o.cpu(), ro) < TOL_LP
    assert rel_err(lse.cpu(), rlse) < 1e-3
    grads = launch_flash_nbhood_attn_bwd(inp["q"], inp["k"], inp["v"], inp["member_idx"], inp["scale"], o, lse,
                                         inp["dout"], **kw)
    ref = oracle.nbhd_attn_bwd(inp["q"].cpu(), inp["k"].cpu(), inp["v"].cpu(), inp["member_idx"].cpu(),
                               inp["scale"], o.cpu(), lse.cpu(), inp["dout"].cpu(), **cpu)
    for name, a, b in zip(["dq", "dk", "dv", "dbias", "dbk", "dbv"], grads, ref):
        assert rel_err(a.cpu(), b) < TOL_LP, name


def test_local_attn_duplicate_neighbours_tensor_core(cuda):
    """Repeated indices inside one neighbour list (allowed by the API) on the tensor-core path."""
    from affmae_b200.kernels.local_attn import launch_flash_nbhood_attn_fwd, launch_flash_nbhood_attn_bwd
    inp = _attn_inputs(1, 2, 48, 32, 16, torch.bfloat16, seed=5)
    inp["mi"] = torch.randint(0, 10, inp["mi"].shape, dtype=torch.int32)  # few keys => many duplicates
    G = _to(inp, cuda)
    kw = lambda d: dict(bias=d["bias"], mask=d["mask"], blank_k=d["blank_k"], blank_v=d["blank_v"])
    o, lse = launch_flash_nbhood_attn_fwd(G["q"], G["k"], G["v"], G["mi"], 32 ** -0.5, **kw(G))
    ro, _ = oracle.nbhd_attn_fwd(inp["q"], inp["k"], inp["v"], inp["mi"], 32 ** -0.5, **kw(inp))
    assert rel_err(o.cpu(), ro) < TOL_LP
    grads = launch_flash_nbhood_attn_bwd(G["q"], G["k"], G["v"], G["mi"], 32 ** -0.5, o, lse, G["do"], **kw(G))
    ref = oracle.nbhd_attn_bwd(inp["q"], inp["k"], inp["v"], inp["mi"], 32 ** -0.5, o.cpu(), lse.cpu(), inp["do"],
                               **kw(inp))
    for name, a, b in zip(["dq", "dk", "dv", "dbias", "dbk", "dbv"], grads, ref):
        assert rel_err(a.cpu(), b) < TOL_LP, name


def test_local_attn_mixed_block_and_general_tiles(cuda):
    """Cluster-block tiles and general tiles in one call (block kernel + union kernel)."""
    from affmae_b200.workloads import nbhd_attention_inputs
    from affmae_b200.kernels.local_attn import launch_flash_nbhood_attn_fwd, launch_flash_nbhood_attn_bwd
    inp = nbhd_attention_inputs(B=2, side=40, H=4, dtype=torch.bfloat16, seed=3, device=cuda)
    mi = inp["member_idx"].clone()
    mi[0, 17, 5] = (mi[0, 17, 5] + 3) % mi.shape[1]          # breaks the run: general tile
    mi[1, 100:116] = torch.flip(mi[1, 100:116], dims=[-1])    # reversed runs: general tiles
    N = mi.shape[1]
    mi[1, N - 3:] = torch.randint(0, N, (3, mi.shape[2]), dtype=torch.int32, device=cuda)
    kw = dict(bias=inp["bias"], blank_k=inp["blank_k"], blank_v=inp["blank_v"])
    o, lse = launch_flash_nbhood_attn_fwd(inp["q"], inp["k"], inp["v"], mi, inp["scale"], **kw)
    cpu = {k: v.cpu() for k, v in kw.items()}
    ro, _ = oracle.nbhd_attn_fwd(inp["q"].cpu(), inp["k"].cpu(), inp["v"].cpu(), mi.cpu(), inp["scale"], **cpu)
    assert rel_err(o.cpu(), ro) < TOL_LP
    grads = launch_flash_nbhood_attn_bwd(inp["q"], inp["k"], inp["v"], mi, inp["scale"], o, lse, inp["dout"], **kw)
    ref = oracle.nbhd_attn_bwd(inp["q"].cpu(), inp["k"].cpu(), inp["v"].cpu(), mi.cpu(), inp["scale"], o.cpu(),
                               lse.cpu(), inp["dout"].cpu(), **cpu)
    for name, a, b in zip(["dq", "dk", "dv", "dbias", "dbk", "dbv"], grads, ref):
        assert rel_err(a.cpu(), b) < TOL_LP, name


@pytest.mark.gpu
def test_local_attn_key_major_long_and_empty_lists(cuda):
    """Key clusters listed by more queries than fit the shared-memory sort (unsorted
    path), clusters listed by nobody and a partial last cluster (N % 8 != 0): dK and
    dV of the key-major pass."""
    from affmae_b200.kernels.local_attn import launch_flash_nbhood_attn_fwd, launch_flash_nbhood_attn_bwd
    B, H, N, D, M = 1, 4, 1029, 32, 64
    inp = _attn_inputs(B, H, N, D, M, torch.bfloat16, seed=11)
    gen = torch.Generator().manual_seed(12)
    runs = torch.stack([torch.randperm(10, generator=gen)[:8] for _ in range(N)])  # clusters 0..9
    inp["mi"] = (runs[:, :, None] * 8 + torch.arange(8)).reshape(1, N, M).to(torch.int32)
    G = _to(inp, cuda)
    kw = lambda d: dict(bias=d["bias"], mask=d["mask"], blank_k=d["blank_k"], blank_v=d["blank_v"])
    o, lse = launch_flash_nbhood_attn_fwd(G["q"], G["k"], G["v"], G["mi"], 32 ** -0.5, **kw(G))
    grads = launch_flash_nbhood_attn_bwd(G["q"], G["k"], G["v"], G["mi"], 32 ** -0.5, o, lse, G["do"], **kw(G))
    ref = oracle.nbhd_attn_bwd(inp["q"], inp["k"], inp["v"], inp["mi"], 32 ** -0.5, o.cpu(), lse.cpu(), inp["do"],
                               **kw(inp))
    for name, a, b in zip(["dq", "dk", "dv", "dbias", "dbk", "dbv"], grads, ref):
        assert rel_err(a.cpu(), b) < TOL_LP, name
    assert torch.count_nonzero(grads[1][:, :, 80:]) == 0 and torch.count_nonzero(grads[2][:, :, 80:]) == 0


@pytest.mark.gpu
def test_local_attn_backward_deterministic(cuda):
    """Sorted inverse lists and no atomics on dQ/dK/dV: two calls agree bit for bit."""
    from affmae_b200.workloads import nbhd_attention_inputs
    from affmae_b200.kernels.local_attn import launch_flash_nbhood_attn_fwd, launch_flash_nbhood_attn_bwd
    inp = nbhd_attention_inputs(B=2, side=48, H=4, dtype=torch.bfloat16, seed=4, device=cuda)
    kw = dict(bias=inp["bias"], blank_k=inp["blank_k"], blank_v=inp["blank_v"])
    o, lse = launch_flash_nbhood_attn_fwd(inp["q"], inp["k"], inp["v"], inp["member_idx"], inp["scale"], **kw)
    g1 = launch_flash_nbhood_attn_bwd(inp["q"], inp["k"], inp["v"], inp["member_idx"], inp["scale"], o, lse,
                                      inp["dout"], **kw)
    g2 = launch_flash_nbhood_attn_bwd(inp["q"], inp["k"], inp["v"], inp["member_idx"], inp["scale"], o, lse,
                                      inp["dout"], **kw)
    for name, a, b in zip(["dq", "dk", "dv", "dbias"], g1[:4], g2[:4]):
        assert torch.equal(a, b), name


@pytest.mark.gpu
def test_nbhd_bwd_workspace_checked(cuda):
    """The C entry point rejects a workspace below affb_nbhd_attn_bwd_workspace_bytes."""
    from affmae_b200 import _native as nat
    B, H, N, D, M = 1, 2, 64, 32, 16
    need = int(nat.lib().affb_nbhd_attn_bwd_workspace_bytes(nat.BF16, B, H, N, D, M))
    assert need > 0
    t = torch.zeros((B, H, N, D), device=cuda, dtype=torch.bfloat16)
    lse = torch.zeros((B, H, N), device=cuda)
    mi = torch.zeros((B, N, M), device=cuda, dtype=torch.int32)
    ws = torch.empty((need,), device=cuda, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="workspace"):
        nat.call("affb_nbhd_attn_bwd", t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(),
                 lse.data_ptr(), mi.data_ptr(), None, None, 1, None, None, nat.BF16, B, H, N, D, M, 1.0,
                 t.data_ptr(), t.data_ptr(), t.data_ptr(), None, None, None, ws.data_ptr(), need - 1,
                 nat.stream(t.device))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_local_attn_partial_last_cluster(cuda, dtype):
    """The model's lists when N % 8 != 0: the last cluster is partial and its
    padding slots point at token 0 with mask 0 (cluster-run fast path), plus the
    same lists with one padding slot left unmasked (general path)."""
    from affmae_b200.kernels.local_attn import launch_flash_nbhood_attn_fwd, launch_flash_nbhood_attn_bwd
    from affmae_b200.mae import curve_clusters, neighbourhood
    g = golden("clusters_ragged")
    pos, means, cmask, _ = curve_clusters(g["pos"].to(cuda), 8, 64, 64)
    member, mask, _ = neighbourhood(pos, means, cmask, 48, 8)
    B, N, M = member.shape
    inp = _attn_inputs(B, 2, N, 32, M, dtype, mask=False, seed=21)
    inp["mi"] = member.cpu().to(torch.int32)
    for variant in ("masked", "unmasked_slot"):
        m = mask.clone()
        if variant == "unmasked_slot":
            pad = (~m).nonzero()
            m[tuple(pad[0])] = True
        inp["mask"] = m.cpu()[:, None]
        G = _to(inp, cuda)
        kw = lambda d: dict(bias=d["bias"], mask=d["mask"], blank_k=d["blank_k"], blank_v=d["blank_v"])
        o, lse = launch_flash_nbhood_attn_fwd(G["q"], G["k"], G["v"], G["mi"], 32 ** -0.5, **kw(G))
        ro, rlse = oracle.nbhd_attn_fwd(inp["q"], inp["k"], inp["v"], inp["mi"], 32 ** -0.5, **kw(inp))
        assert rel_err(o.cpu(), ro) < TOL_LP, variant
        assert rel_err(lse.cpu(), rlse) < 1e-3, variant
        grads = launch_flash_nbhood_attn_bwd(G["q"], G["k"], G["v"], G["mi"], 32 ** -0.5, o, lse, G["do"], **kw(G))
        ref = oracle.nbhd_attn_bwd(inp["q"], inp["k"], inp["v"], inp["mi"], 32 ** -0.5, o.cpu(), lse.cpu(),
                                   inp["do"], **kw(inp))
        for name, a, b in zip(["dq", "dk", "dv", "dbias", "dbk", "dbv"], grads, ref):
            assert rel_err(a.cpu(), b) < TOL_LP, (variant, name)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rel_pos_bias_matches_table_gather(cuda, dtype):
    """In-kernel relative-position bias == Linear(5 -> H) over the reference's
    table followed by the gather; weight/bias gradients == autograd of that."""
    from affmae_b200.kernels.pos_bias import rel_pos_bias
    from affmae_b200.workloads import relative_position_table
    g = torch.Generator().manual_seed(3)
    H, B, N, M = 6, 2, 97, 48
    w = (torch.randn((H, 5), generator=g) * 0.3).to(cuda).requires_grad_(True)
    b = (torch.randn((H,), generator=g) * 0.1).to(cuda).requires_grad_(True)
    # offsets within +-20 tokens plus a few at the clamp limits and zero
    pe = (torch.randint(107, 148, (B, N, M), generator=g) * 255 + torch.randint(107, 148, (B, N, M), generator=g))
    pe[0, 0, :3] = torch.tensor([0, 65024, 127 * 255 + 127])
    pe = pe.to(cuda)
    out = rel_pos_bias(w, b, pe, dtype)
    table = relative_position_table().to(cuda)
    ref = (table @ w.T + b)[pe].permute(0, 3, 1, 2)
    assert rel_err(out.float().cpu(), ref.detach().cpu()) < (1e-6 if dtype == torch.float32 else 8e-3)
    go = torch.randn(ref.shape, generator=g).to(cuda)
    gw, gb = torch.autograd.grad(out, (w, b), go.to(dtype))
    rw, rb = torch.autograd.grad(ref, (w, b), go.to(dtype).float())
    assert rel_err(gw.cpu(), rw.cpu()) < 1e-4 and rel_err(gb.cpu(), rb.cpu()) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("xdtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("C", [48, 96, 192, 320, 384, 1536])
def test_fused_layer_norm_matches_torch(cuda, xdtype, C):
    """LayerNorm(x) with fp32 and bf16 outputs, values and all gradients, against
    torch.nn.functional.layer_norm in fp32."""
    from affmae_b200.kernels.layer_norm import fused_layer_norm
    g = torch.Generator().manual_seed(C)
    x = (torch.randn((3, 77, C), generator=g) * 2 + 0.5).to(cuda, xdtype).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(C, generator=g)).to(cuda).requires_grad_(True)
    b = (0.1 * torch.randn(C, generator=g)).to(cuda).requires_grad_(True)
    y32, y16 = fused_layer_norm(x, w, b, 1e-5, out32=True, out16=True)
    xr = x.detach().float().requires_grad_(True)
    ref = torch.nn.functional.layer_norm(xr, (C,), w, b, 1e-5)
    assert rel_err(y32.cpu(), ref.detach().cpu()) < 1e-5
    assert rel_err(y16.float().cpu(), ref.detach().cpu()) < 8e-3
    g32 = torch.randn(ref.shape, generator=g).to(cuda)
    g16 = torch.randn(ref.shape, generator=g).to(cuda, torch.bfloat16)
    dx, dw, db = torch.autograd.grad((y32, y16), (x, w, b), (g32, g16))
    rx, rw, rb = torch.autograd.grad(ref, (xr, w, b), g32 + g16.float())
    tol = 1e-4 if xdtype == torch.float32 else 8e-3
    assert rel_err(dx.float().cpu(), rx.cpu()) < tol
    assert rel_err(dw.cpu(), rw.cpu()) < 1e-4 and rel_err(db.cpu(), rb.cpu()) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("p", [0.0, 0.1])
def test_fused_residual_dropout_layer_norm(cuda, p):
    """LayerNorm(x + dropout(delta)) with a bf16 delta: without dropout equal to
    the torch sequence; with dropout the mask seen by the backward (zeros of
    d_delta) is the one the forward applied, and about p of the elements drop."""
    from affmae_b200.kernels.layer_norm import fused_layer_norm
    g = torch.Generator().manual_seed(5)
    C = 384
    x = torch.randn((4, 300, C), generator=g).to(cuda).requires_grad_(True)
    d = torch.randn((4, 300, C), generator=g).to(cuda, torch.bfloat16).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(C, generator=g)).to(cuda).requires_grad_(True)
    b = (0.1 * torch.randn(C, generator=g)).to(cuda).requires_grad_(True)
    y32 = fused_layer_norm(x, w, b, 1e-5, delta=d, p=p, out32=True)
    gy = torch.randn(y32.shape, generator=g).to(cuda)
    dx, dd = torch.autograd.grad(y32, (x, d), gy)
    keep = (dd != 0).float() if p > 0 else torch.ones_like(x)
    if p > 0:
        frac = 1 - keep.mean().item()
        assert abs(frac - p) < 0.01, frac
    xr = x.detach().clone().requires_grad_(True)
    dr = d.detach().float().clone().requires_grad_(True)
    ref = torch.nn.functional.layer_norm(xr + dr * keep / (1 - p), (C,), w, b, 1e-5)
    assert rel_err(y32.cpu(), ref.detach().cpu()) < 1e-5
    rx, rd = torch.autograd.grad(ref, (xr, dr), gy)
    assert rel_err(dx.cpu(), rx.cpu()) < 1e-4
    assert rel_err(dd.float().cpu(), rd.cpu()) < 8e-3


@pytest.mark.gpu
@pytest.mark.parametrize("scaled", [False, True])
@pytest.mark.parametrize("with_ds", [False, True])
def test_residual_layer_norm_pre_norm_form(cuda, scaled, with_ds):
    """(s, y) = (x + f_b * delta, LayerNorm(s)) with a per-sample factor f_b
    (stochastic depth; 0 for one sample) against the torch sequence in fp32;
    the backward with and without a gradient of s from its other uses."""
    from affmae_b200.kernels.layer_norm import ResidualNormFunction
    g = torch.Generator().manual_seed(7)
    B, N, C = 3, 211, 384
    x = torch.randn((B, N, C), generator=g).to(cuda).requires_grad_(True)
    d = torch.randn((B, N, C), generator=g).to(cuda, torch.bfloat16).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(C, generator=g)).to(cuda).requires_grad_(True)
    b = (0.1 * torch.randn(C, generator=g)).to(cuda).requires_grad_(True)
    f = torch.tensor([1 / 0.9, 0.0, 1 / 0.9], device=cuda) if scaled else None
    s, y = ResidualNormFunction.apply(x, d, f, w, b, 1e-5)
    xr = x.detach().clone().requires_grad_(True)
    dr = d.detach().float().clone().requires_grad_(True)
    sr = xr + dr * (f.view(B, 1, 1) if scaled else 1.0)
    yr = torch.nn.functional.layer_norm(sr, (C,), w, b, 1e-5)
    assert rel_err(s.detach().cpu(), sr.detach().cpu()) < 1e-6
    assert rel_err(y.float().detach().cpu(), yr.detach().cpu()) < 8e-3
    gy = torch.randn(y.shape, generator=g).to(cuda, torch.bfloat16)
    gs = torch.randn(s.shape, generator=g).to(cuda) if with_ds else None
    outs, grads = ((s, y), (gs, gy)) if with_ds else ((y,), (gy,))
    dx, dd, dw, db = torch.autograd.grad(outs, (x, d, w, b), grads)
    routs, rgrads = ((sr, yr), (gs, gy.float())) if with_ds else ((yr,), (gy.float(),))
    rx, rd, rw, rb = torch.autograd.grad(routs, (xr, dr, w, b), rgrads)
    assert rel_err(dx.cpu(), rx.cpu()) < 1e-4
    assert rel_err(dd.float().cpu(), rd.cpu()) < 8e-3
    if scaled:
        assert bool((dd[1] == 0).all())
    assert rel_err(dw.cpu(), rw.cpu()) < 1e-4 and rel_err(db.cpu(), rb.cpu()) < 1e-4


@pytest.mark.gpu
def test_knn2d_grid_far_queries_and_duplicates(cuda):
    """Grid search: duplicated reference points (ties broken by index), queries
    far outside the points' bounding box and exactly on cell edges; equal to
    the oracle and to the brute-force entry point."""
    from affmae_b200 import _native as nat
    from affmae_b200.kernels.knn import knn
    gen = torch.Generator().manual_seed(17)
    r = torch.randint(0, 40, (2, 1500, 2), generator=gen).float()
    r[:, 700:900] = r[:, :200]                                   # exact duplicates
    q = torch.cat([torch.rand((2, 100, 2), generator=gen) * 40,
                   torch.tensor([[-500.0, 3.0], [1e4, 1e4], [20.0, -300.0], [39.0, 39.0]]).expand(2, 4, 2),
                   r[:, :50] + 0.5], dim=1)
    import affmae_b200.kernels.knn as kmod
    old = kmod.GRID_MIN_PAIRS
    kmod.GRID_MIN_PAIRS = 0  # force the grid path at this size
    for K in (1, 7, 48, 130):
        idx = knn(q.to(cuda), r.to(cuda), K)
        assert torch.equal(idx.cpu(), oracle.knn(q, r, K)), K
        brute = torch.empty_like(idx)
        qc, rc = q.to(cuda).contiguous(), r.to(cuda).contiguous()
        nat.call("affb_knn", nat.ptr(qc), nat.ptr(rc), nat.F32, 2, q.shape[1], r.shape[1], 2, K, nat.ptr(brute),
                 nat.stream(qc.device))
        assert torch.equal(idx, brute), K
    kmod.GRID_MIN_PAIRS = old


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("parts", [1, 2])
def test_head_split_merge(cuda, dtype, parts):
    """Head splits / merges of ClusterAttention are exact permute copies, and
    so are their gradients."""
    from affmae_b200.kernels.head_layout import merge_heads, split_heads
    B, N, H, d = 2, 37, 3, 32
    gen = torch.Generator().manual_seed(parts)
    x = torch.randn((B, N, H * parts * d), generator=gen).to(cuda, dtype).requires_grad_(True)
    outs = split_heads(x, H, parts)
    outs = (outs,) if parts == 1 else outs
    ref = x.detach().view(B, N, H, parts, d).permute(3, 0, 2, 1, 4)
    for p in range(parts):
        assert outs[p].is_contiguous() and torch.equal(outs[p], ref[p])
    gs = [torch.randn((B, H, N, d), generator=gen).to(cuda, dtype) for _ in range(parts)]
    torch.autograd.backward(list(outs), gs)
    assert torch.equal(x.grad, torch.stack(gs, 0).permute(1, 3, 2, 0, 4).reshape(B, N, H * parts * d))
    o = torch.randn((B, H, N, d), generator=gen).to(cuda, dtype).requires_grad_(True)
    y = merge_heads(o)
    assert torch.equal(y, o.detach().permute(0, 2, 1, 3).reshape(B, N, H * d))
    gy = torch.randn(y.shape, generator=gen).to(cuda, dtype)
    y.backward(gy)
    assert torch.equal(o.grad, gy.view(B, N, H, d).permute(0, 2, 1, 3))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_deform_backward_recomputes_distances(cuda, dtype):
    """The autograd path saves only the neighbour indices: the backward given
    knn_d2 = None recomputes the squared distances and returns the same
    gradients as the backward given the saved distances."""
    from affmae_b200.kernels.fused_deform_attn import (fused_knn_deform_cross_attn_forward_save,
                                                       fused_knn_deform_cross_attn_backward)
    qp, kv, off, aw, val, power, do = _deform_inputs(2, 300, 40, 8, 32, dtype, seed=9)
    args = [t.to(cuda) for t in (qp, kv, off, aw, val, power)]
    _, ki, kd = fused_knn_deform_cross_attn_forward_save(*args)
    _, ki2, none = fused_knn_deform_cross_attn_forward_save(*args, save_dist=False)
    assert none is None and torch.equal(ki, ki2)
    g1 = fused_knn_deform_cross_attn_backward(do.to(cuda), *args, ki, kd)
    g2 = fused_knn_deform_cross_attn_backward(do.to(cuda), *args, ki, None)
    # per-sample gradients are written once: bit-exact; the scatter-added ones
    # (atomics, order not fixed) within fp32 summation-order error
    for name, a, b in zip(["d_qpos", "d_kvpos", "d_off", "d_aw", "d_val", "d_power"], g1, g2):
        if name in ("d_off", "d_aw"):
            assert torch.equal(a, b), name
        else:
            assert rel_err(a.float().cpu(), b.float().cpu()) < (1e-5 if dtype == torch.float32 else 1e-2), name


def test_reference_public_helpers(cuda):
    """The reference modules' remaining public helpers exist with their
    signatures and agree with the main entry points."""
    from affmae_b200.kernels import fused_deform_attn as fd, knn as kn, weighted_features as wf
    gen = torch.Generator().manual_seed(3)
    q = (torch.rand((2, 100, 2), generator=gen) * 20).to(cuda)
    r = (torch.rand((2, 400, 2), generator=gen) * 20).to(cuda)
    assert torch.equal(kn.knn_pytorch_large(q, r, 12), kn.knn(q, r, 12))
    assert torch.equal(kn.knn_large_k_fallback(q, r, 40), oracle.knn(q.cpu(), r.cpu(), 40).to(cuda))
    w = torch.randn((2, 30, 48, 4), generator=gen).to(cuda)
    f = torch.randn((2, 100, 32), generator=gen).to(cuda)
    idx = torch.randint(0, 100, (2, 30, 48), generator=gen).to(cuda)
    assert torch.equal(wf.weighted_features_triton(w, f, idx), wf.weighted_features_fwd(w, f, idx))
    dw, df = wf.weighted_features_triton_backward(torch.ones((2, 30, 4, 32), device=cuda), w, f, idx)
    assert dw.shape == w.shape and df.shape == f.shape
    qp, kv, off, aw, val, power, _ = _deform_inputs(1, 64, 12, 2, 16, torch.float32, seed=2)
    args = [t.to(cuda) for t in (qp, kv, off, aw, val, power)]
    out, _, d2 = fd.fused_knn_deform_cross_attn_forward_save(*args)
    assert torch.equal(fd.fused_knn_deform_cross_attn_forward(*args), out)
    sw = fd.compute_softmax_weights(d2, args[-1])
    assert torch.allclose(sw.sum(-1), torch.ones_like(sw.sum(-1)))
    fd.set_use_heuristics(False)
    fd.set_use_heuristics(True)


@pytest.mark.parametrize("variant", ["clusters", "ragged_masked", "general"])
def test_local_attn_tile_plan_reuse(cuda, variant):
    """The backward given the forward's tile plan (its tiles' cluster unions)
    returns exactly the gradients of the backward that rebuilds them."""
    from affmae_b200.kernels.local_attn import launch_flash_nbhood_attn_fwd, launch_flash_nbhood_attn_bwd
    from affmae_b200.mae import curve_clusters, neighbourhood
    from affmae_b200.workloads import nbhd_attention_inputs
    if variant == "clusters":
        inp = nbhd_attention_inputs(B=2, side=48, H=4, dtype=torch.bfloat16, seed=6, device=cuda)
        q, k, v, mi, do = inp["q"], inp["k"], inp["v"], inp["member_idx"], inp["dout"]
        kw = dict(bias=inp["bias"], blank_k=inp["blank_k"], blank_v=inp["blank_v"])
        scale = inp["scale"]
    else:
        g = golden("clusters_ragged")
        pos, means, cmask, _ = curve_clusters(g["pos"].to(cuda), 8, 64, 64)
        member, mask, _ = neighbourhood(pos, means, cmask, 48, 8)
        B, N, M = member.shape
        d = _attn_inputs(B, 2, N, 32, M, torch.float16, mask=False, seed=22)
        m = mask.clone()
        if variant == "general":
            m[tuple((~m).nonzero()[0])] = True
        G = _to(d, cuda)
        q, k, v, mi, do = G["q"], G["k"], G["v"], member.to(torch.int32), G["do"]
        kw = dict(bias=G["bias"], mask=m[:, None], blank_k=G["blank_k"], blank_v=G["blank_v"])
        scale = 32 ** -0.5
    o, lse, plan = launch_flash_nbhood_attn_fwd(q, k, v, mi, scale, return_plan=True, **kw)
    o2, lse2 = launch_flash_nbhood_attn_fwd(q, k, v, mi, scale, **kw)
    assert plan is not None and torch.equal(o, o2) and torch.equal(lse, lse2)
    g1 = launch_flash_nbhood_attn_bwd(q, k, v, mi, scale, o, lse, do, plan=plan, **kw)
    g2 = launch_flash_nbhood_attn_bwd(q, k, v, mi, scale, o, lse, do, **kw)
    for name, a, b in zip(["dq", "dk", "dv", "dbias"], g1[:4], g2[:4]):
        if variant == "general" and name in ("dk", "dv"):  # scatter-added: order of the adds is free
            assert rel_err(a.float().cpu(), b.float().cpu()) < 1e-2, name
        else:
            assert torch.equal(a, b), name
