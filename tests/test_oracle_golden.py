"""The CPU oracle against golden vectors produced by the reference's own kernels.

The golden vectors come from the reference Triton kernels run under the
Triton interpreter (tests/golden/make_golden.py).  The reference rounds the
local-attention output through fp16 (local_attn.py:340), so that output and
everything downstream of it (lse is unaffected; dq/dk/dv/dbias depend on O via
Delta) are compared at 2e-3; everything else at 1e-5.
"""
import pytest
import torch

import oracle
from conftest import golden, rel_err


@pytest.mark.parametrize("tag", ["d2_k4", "d2_k8_grid", "d3_k6", "d2_k3_grid"])
def test_knn_oracle_matches_reference(tag):
    g = golden(f"knn_{tag}")
    idx = oracle.knn(g["query"], g["ref"], int(g["k"]))
    assert torch.equal(idx, g["idx"])


@pytest.mark.parametrize("tag", ["full", "plain", "m24"])
def test_local_attn_oracle_matches_reference(tag):
    g = golden(f"local_attn_{tag}")
    kw = dict(bias=g.get("bias"), mask=g.get("mask"), blank_k=g.get("blank_k"), blank_v=g.get("blank_v"))
    scale = float(g["scale"])
    o, lse = oracle.nbhd_attn_fwd(g["q"], g["k"], g["v"], g["mi"], scale, **kw)
    assert rel_err(lse, g["lse"]) < 1e-5
    assert rel_err(o, g["o"]) < 2e-3          # reference O is fp16-rounded
    # backward from the reference's own stored O and lse
    dq, dk, dv, dbias, dbk, dbv = oracle.nbhd_attn_bwd(g["q"], g["k"], g["v"], g["mi"], scale,
                                                       g["o"], g["lse"], g["do"], **kw)
    for name, a in [("dq", dq), ("dk", dk), ("dv", dv)]:
        assert rel_err(a, g[name]) < 1e-4, name
    if "dbias" in g:
        assert rel_err(dbias, g["dbias"]) < 1e-4
    if "dbk" in g:
        assert rel_err(dbk, g["dbk"]) < 1e-4
        assert rel_err(dbv, g["dbv"]) < 1e-4


def test_local_attn_oracle_matches_reference_formula():
    """Kernel-semantics oracle == the reference's PyTorch formula (local_attn.py:979-1006)
    whenever every row has at least one attended neighbour."""
    g = golden("local_attn_full")
    q, k, v = (g[n].double().requires_grad_() for n in ("q", "k", "v"))
    bias = g["bias"].double().requires_grad_()
    bk, bv = g["blank_k"].double(), g["blank_v"].double()
    mask = g["mask"].clone()
    mask[0, 0, 3, 0] = 1
    scale = float(g["scale"])
    ref = oracle.nbhd_attn_formula(q, k, v, g["mi"], scale, bias=bias, mask=mask, blank_k=bk, blank_v=bv)
    o, lse = oracle.nbhd_attn_fwd(q.detach(), k.detach(), v.detach(), g["mi"], scale, bias=bias.detach(),
                                  mask=mask, blank_k=bk, blank_v=bv)
    assert rel_err(o, ref.detach()) < 1e-12
    do = g["do"].double()
    gq, gk, gv, gb = torch.autograd.grad(ref, (q, k, v, bias), do)
    dq, dk, dv, db, _, _ = oracle.nbhd_attn_bwd(q.detach(), k.detach(), v.detach(), g["mi"], scale, o, lse,
                                                do, bias=bias.detach(), mask=mask, blank_k=bk, blank_v=bv)
    for a, b in [(dq, gq), (dk, gk), (dv, gv), (db, gb)]:
        assert rel_err(a, b) < 1e-10


def test_weighted_features_oracle_matches_reference():
    g = golden("weighted_features")
    assert rel_err(oracle.weighted_features_fwd(g["w"], g["feat"], g["idx"]), g["out"]) < 1e-5
    dw, df = oracle.weighted_features_bwd(g["dout"], g["w"], g["feat"], g["idx"])
    assert rel_err(dw, g["dw"]) < 1e-5
    assert rel_err(df, g["dfeat"]) < 1e-5


def test_weighted_gather_oracle_matches_reference():
    g = golden("weighted_gather")
    out = oracle.weighted_features_fwd(g["w"][..., None], g["feat"], g["idx"])[:, :, 0]
    assert rel_err(out, g["out"]) < 1e-5
    dw, df = oracle.weighted_features_bwd(g["dout"][:, :, None], g["w"][..., None], g["feat"], g["idx"])
    assert rel_err(dw[..., 0], g["dw"]) < 1e-5
    assert rel_err(df, g["dfeat"]) < 1e-5


@pytest.mark.parametrize("tag", ["cross", "cross_grid"])
def test_deform_cross_oracle_matches_reference(tag):
    g = golden(f"deform_{tag}")
    out, idx, d2 = oracle.deform_knn_fwd(g["qpos"], g["kvpos"], g["off"], g["aw"], g["val"], g["power"])
    assert torch.equal(idx, g["knn_idx"].long())
    assert torch.equal(d2, g["knn_d2"])
    assert rel_err(out, g["out"]) < 1e-5
    grads = oracle.deform_knn_bwd(g["dout"], g["qpos"], g["kvpos"], g["off"], g["aw"], g["val"],
                                  g["power"], idx, d2)
    for name, a in zip(["d_qpos", "d_kvpos", "d_off", "d_aw", "d_val", "d_power"], grads):
        assert rel_err(a, g[name]) < 1e-4, name


def test_deform_self_oracle_matches_reference():
    g = golden("deform_self")
    out, idx, d2 = oracle.deform_knn_fwd(g["pos"], g["pos"], g["off"], g["aw"], g["val"], g["power"])
    assert torch.equal(idx, g["knn_idx"].long())
    assert rel_err(out, g["out"]) < 1e-5
    d_pos, _, d_off, d_aw, d_val, d_pow = oracle.deform_knn_bwd(
        g["dout"], g["pos"], g["pos"], g["off"], g["aw"], g["val"], g["power"], idx, d2, self_attn=True)
    for name, a in [("d_pos", d_pos), ("d_off", d_off), ("d_aw", d_aw), ("d_val", d_val), ("d_power", d_pow)]:
        assert rel_err(a, g[name]) < 1e-4, name


def test_deform_nbidx_oracle_matches_reference():
    g = golden("deform_nbidx")
    out = oracle.deform_nbidx_fwd(g["sl"], g["kvpos"], g["nb"], g["power"], g["aw"], g["val"])
    assert rel_err(out, g["out"]) < 1e-5
    grads = oracle.deform_nbidx_bwd(g["dout"], g["sl"], g["kvpos"], g["nb"], g["power"], g["aw"], g["val"])
    for name, a in zip(["d_sl", "d_kvpos", "d_power", "d_aw", "d_val"], grads):
        assert rel_err(a, g[name]) < 1e-4, name


def test_mssample_oracle_matches_reference():
    g = golden("mssample")
    w = oracle.mssample_fwd(g["sl"], g["kvpos"], g["nb"], g["power"])
    assert rel_err(w, g["w"]) < 1e-5
    grads = oracle.mssample_bwd(g["dw"], g["sl"], g["kvpos"], g["nb"], g["power"], g["w"])
    for name, a in zip(["d_sl", "d_kvpos", "d_power"], grads):
        assert rel_err(a, g[name]) < 1e-4, name


def test_msdetrpc_oracle_matches_reference():
    g = golden("msdetrpc")
    assert rel_err(oracle.msdetrpc_fwd(g["idx"], g["w"], g["attn"], g["val"]), g["out"]) < 1e-5
    grads = oracle.msdetrpc_bwd(g["dout"], g["idx"], g["w"], g["attn"], g["val"])
    for name, a in zip(["d_w", "d_attn", "d_val"], grads):
        assert rel_err(a, g[name]) < 1e-5, name
