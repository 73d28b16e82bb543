"""Generate the golden vectors in tests/golden/*.npz from the reference itself.

Runs the reference's own Triton kernels (najafian-lab/affmae,
src/layers/kernels/*.py) on the CPU under ``TRITON_INTERPRET=1`` on small
seeded inputs and stores inputs and outputs.  Two shims are needed because
the reference package touches a GPU driver at import time:
  * ``src/layers/kernels/util.py`` queries ``triton.runtime.driver`` at import
    (util.py:6-23); it is replaced by a stub module with the same names;
  * ``src/layers/kernels/__init__.py`` is skipped by loading each kernel file
    as a module of a bare package.
Launchers that assert ``is_cuda`` are bypassed by calling the next layer down
(the launcher functions the asserting wrapper calls).

Usage:  python tests/golden/make_golden.py --reference /path/to/affmae
        (or AFFMAE_REFERENCE=/path/to/affmae python tests/golden/make_golden.py)
This needs the reference checkout and is only run when fixtures change; the
tests read the committed .npz files.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import time
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def load_reference(root: str):
    kdir = os.path.join(root, "src", "layers", "kernels")
    pkg = types.ModuleType("refk")
    pkg.__path__ = [kdir]
    sys.modules["refk"] = pkg
    util = types.ModuleType("refk.util")
    util.NUM_STAGES_OPTIONS = [1, 2]
    util.is_hip = lambda: False
    util.is_cuda = lambda: True
    util.supports_host_descriptor = lambda: False
    sys.modules["refk.util"] = util
    mods = {}
    for name in ["knn", "local_attn", "weighted_features", "weighted_gather",
                 "fused_deform_attn", "msdetrpc", "mssample"]:
        spec = importlib.util.spec_from_file_location("refk." + name, os.path.join(kdir, name + ".py"))
        m = importlib.util.module_from_spec(spec)
        sys.modules["refk." + name] = m
        spec.loader.exec_module(m)
        mods[name] = m
    return mods


def npz(name, **arrays):
    out = {k: (v.detach().cpu().numpy() if torch.is_tensor(v) else np.asarray(v)) for k, v in arrays.items()}
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"  wrote {name}.npz ({', '.join(out)})", flush=True)


def gen_knn(R):
    m = R["knn"]
    g = torch.Generator().manual_seed(1)
    for tag, D, K, integer in [("d2_k4", 2, 4, False), ("d2_k8_grid", 2, 8, True),
                               ("d3_k6", 3, 6, False), ("d2_k3_grid", 2, 3, True)]:
        B, M, N = 2, 37, 53
        if integer:  # integer lattice points: many exact distance ties
            q = torch.randint(0, 6, (B, M, D), generator=g).float()
            r = torch.randint(0, 6, (B, N, D), generator=g).float()
        else:
            q = torch.rand((B, M, D), generator=g) * 10
            r = torch.rand((B, N, D), generator=g) * 10
        kk = 4 if K <= 4 else 8
        out = torch.zeros((B, M, kk), dtype=torch.int32)
        kern = getattr(m, f"_knn_kernel_simple_k{kk}_d{D}_noautotune")
        kern[(triton_cdiv(M, 64), B)](q, r, out, B, M, N, *q.stride(), *r.stride(), *out.stride(),
                                      BLOCK_M=64, BLOCK_N=32)
        npz(f"knn_{tag}", query=q, ref=r, k=K, idx=out[:, :, :K].long())


def triton_cdiv(a, b):
    return (a + b - 1) // b


def gen_local_attn(R):
    m = R["local_attn"]
    g = torch.Generator().manual_seed(2)
    for tag, masked, blank, bias, N, M in [("full", True, True, True, 24, 16),
                                           ("plain", False, False, False, 20, 8),
                                           ("m24", True, True, True, 19, 24)]:
        B, H, D = 2, 2, 16
        q = torch.randn((B, H, N, D), generator=g)
        k = torch.randn((B, H, N, D), generator=g)
        v = torch.randn((B, H, N, D), generator=g)
        mi = torch.randint(0, N, (B, N, M), generator=g, dtype=torch.int32)
        bias_t = torch.randn((B, H, N, M), generator=g) * 0.5 if bias else None
        mask_t = (torch.rand((B, 1, N, M), generator=g) > 0.25).to(torch.int32) if masked else None
        if masked:
            mask_t[0, 0, 3, :] = 0  # a fully masked row
        bk = torch.randn((H, D), generator=g) if blank else None
        bv = torch.randn((H, D), generator=g) if blank else None
        do = torch.randn((B, H, N, D), generator=g)
        scale = D ** -0.5
        o, lse = m.launch_flash_nbhood_attn_fwd(q, k, v, mi, scale, bias=bias_t, mask=mask_t,
                                                blank_k=bk, blank_v=bv)
        dq, dk, dv, dbias, dbk, dbv = m.launch_flash_nbhood_attn_bwd(
            q, k, v, mi, scale, o, lse, do, bias=bias_t, mask=mask_t, blank_k=bk, blank_v=bv)
        arrs = dict(q=q, k=k, v=v, mi=mi, do=do, scale=scale, o=o, lse=lse, dq=dq, dk=dk, dv=dv)
        if bias:
            arrs.update(bias=bias_t, dbias=dbias)
        if masked:
            arrs.update(mask=mask_t)
        if blank:
            arrs.update(blank_k=bk, blank_v=bv, dbk=dbk, dbv=dbv)
        npz(f"local_attn_{tag}", **arrs)


def gen_weighted(R):
    wf = R["weighted_features"]
    wg = R["weighted_gather"]
    g = torch.Generator().manual_seed(3)
    B, No, M, IC, N, C = 2, 10, 8, 4, 30, 20
    w = torch.randn((B, No, M, IC), generator=g)
    f = torch.randn((B, N, C), generator=g)
    idx = torch.randint(0, N, (B, No, M), generator=g, dtype=torch.int32)
    do = torch.randn((B, No, IC, C), generator=g)
    out = wf.weighted_features_triton(w, f, idx)
    dw, df = wf.weighted_features_triton_backward(do, w, f, idx)
    npz("weighted_features", w=w, feat=f, idx=idx, dout=do, out=out, dw=dw, dfeat=df)
    B, N, K, No, C = 2, 20, 6, 25, 32
    w = torch.softmax(torch.randn((B, N, K), generator=g), -1)
    f = torch.randn((B, No, C), generator=g)
    idx = torch.randint(0, No, (B, N, K), generator=g, dtype=torch.int32)
    do = torch.randn((B, N, C), generator=g)
    out = wg.launch_weighted_gather_fwd_kernel(idx, w, f)
    dw, df = wg.launch_weighted_gather_bwd_kernel(do, idx, w, f)
    npz("weighted_gather", w=w, feat=f, idx=idx, dout=do, out=out, dw=dw, dfeat=df)


def gen_deform(R):
    fd = R["fused_deform_attn"]
    g = torch.Generator().manual_seed(4)
    B, Nq, Nkv, H, C = 1, 9, 30, 2, 8
    power = torch.tensor(1.3)
    for tag, grid in [("cross", False), ("cross_grid", True)]:
        if grid:  # integer lattice kv, integer offsets: exact ties everywhere
            xs = torch.arange(6).float()
            kv = torch.stack(torch.meshgrid(xs, xs, indexing="ij"), -1).reshape(1, 36, 2)
            Nk = 36
            qp = torch.randint(0, 6, (B, Nq, 2), generator=g).float()
            off = torch.randint(-2, 3, (B, Nq, H, 4, 2), generator=g).float()
        else:
            Nk = Nkv
            kv = torch.rand((B, Nk, 2), generator=g) * 8
            qp = torch.rand((B, Nq, 2), generator=g) * 8
            off = torch.randn((B, Nq, H, 4, 2), generator=g)
        aw = torch.softmax(torch.randn((B, Nq, H, 4), generator=g), -1)
        val = torch.randn((B, Nk, H, C), generator=g)
        do = torch.randn((B, Nq, H, C), generator=g)
        out, ki, kd = fd.fused_knn_deform_cross_attn_forward_save(qp, kv, off, aw, val, power)
        grads = fd.fused_knn_deform_cross_attn_backward(do, qp, kv, off, aw, val, power, ki, kd)
        names = ["d_qpos", "d_kvpos", "d_off", "d_aw", "d_val", "d_power"]
        npz(f"deform_{tag}", qpos=qp, kvpos=kv, off=off, aw=aw, val=val, power=power, dout=do,
            out=out, knn_idx=ki, knn_d2=kd, **dict(zip(names, grads)))
    N = 14
    pos = torch.rand((B, N, 2), generator=g) * 5
    off = torch.randn((B, N, H, 4, 2), generator=g) * 0.7
    aw = torch.softmax(torch.randn((B, N, H, 4), generator=g), -1)
    val = torch.randn((B, N, H, C), generator=g)
    do = torch.randn((B, N, H, C), generator=g)
    out, ki, kd = fd.fused_knn_deform_self_attn_forward_save(pos, off, aw, val, power)
    grads = fd.fused_knn_deform_self_attn_backward(do, pos, off, aw, val, power, ki, kd)
    npz("deform_self", pos=pos, off=off, aw=aw, val=val, power=power, dout=do, out=out,
        knn_idx=ki, knn_d2=kd, **dict(zip(["d_pos", "d_off", "d_aw", "d_val", "d_power"], grads)))
    # deformable attention with given neighbours
    Bn, Nn, Nkv, K, Cn = 2, 11, 20, 4, 12
    sl = torch.rand((Bn, Nn, 2), generator=g) * 4
    kvp = torch.rand((Bn, Nkv, 2), generator=g) * 4
    nb = torch.randint(0, Nkv, (Bn, Nn, K), generator=g, dtype=torch.int32)
    awn = torch.rand((Bn, Nn), generator=g)
    valn = torch.randn((Bn, Nkv, Cn), generator=g)
    don = torch.randn((Bn, Nn, Cn), generator=g)
    out = fd.fused_deform_attn_forward(sl, kvp, nb, power, awn, valn, use_heuristics=True)
    grads = fd.fused_deform_attn_backward(don, sl, kvp, nb, power, awn, valn, use_heuristics=True)
    npz("deform_nbidx", sl=sl, kvpos=kvp, nb=nb, power=power, aw=awn, val=valn, dout=don,
        out=out, **dict(zip(["d_sl", "d_kvpos", "d_power", "d_aw", "d_val"], grads)))


def gen_ms(R):
    ms = R["mssample"]
    md = R["msdetrpc"]
    # one configuration each, so the autotuner launches without benchmarking
    for kern in (ms._mssample_fwd_kernel, ms._mssample_bwd_kernel):
        kern.configs = kern.configs[:1]
    g = torch.Generator().manual_seed(5)
    B, N, Nkv, K = 2, 13, 21, 4
    sl = torch.rand((B, N, 2), generator=g) * 4
    kvp = torch.rand((B, Nkv, 2), generator=g) * 4
    nb = torch.randint(0, Nkv, (B, N, K), generator=g, dtype=torch.int32)
    power = torch.tensor(2.0)
    w = ms.mssample_forward(sl, kvp, nb, power)
    dw = torch.randn(w.shape, generator=g)
    grads = ms.mssample_backward(dw, sl, kvp, nb, power, w)
    npz("mssample", sl=sl, kvpos=kvp, nb=nb, power=power, w=w, dw=dw,
        **dict(zip(["d_sl", "d_kvpos", "d_power"], grads)))
    B, N, M, K, Nv, C = 2, 17, 3, 4, 23, 40
    idx = torch.randint(0, Nv, (B, N, M, K), generator=g, dtype=torch.int32)
    w = torch.rand((B, N, M, K), generator=g)
    attn = torch.rand((B, N, M), generator=g)
    val = torch.randn((B, Nv, C), generator=g)
    do = torch.randn((B, N, C), generator=g)
    out = md.launch_msdetrpc_forward(idx, w, attn, val)
    d_nw, d_att, d_val = md.launch_msdetrpc_backward(do, idx, w, attn, val)
    npz("msdetrpc", idx=idx, w=w, attn=attn, val=val, dout=do, out=out, d_w=d_nw, d_attn=d_att,
        d_val=d_val)


def gen_clusters(R):
    """The model's token clustering, src/utils/geometry.py:170-319, loaded with
    a stub for the pykeops import at the top of that file (unused by it)."""
    root = R["_root"]
    sys.modules.setdefault("pykeops", types.ModuleType("pykeops"))
    pk = types.ModuleType("pykeops.torch")
    pk.LazyTensor = None
    sys.modules.setdefault("pykeops.torch", pk)
    # geometry.py also imports two kernel wrappers that space_filling_cluster does not use
    for name, attr in [("src", None), ("src.layers", None), ("src.layers.kernels", None),
                       ("src.layers.kernels.weighted_gather", "weighted_gather"),
                       ("src.layers.kernels.knn", "knn")]:
        mod = sys.modules.setdefault(name, types.ModuleType(name))
        if attr:
            setattr(mod, attr, None)
    spec = importlib.util.spec_from_file_location("refgeom", os.path.join(root, "src", "utils", "geometry.py"))
    geo = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(geo)
    g = torch.Generator().manual_seed(7)
    cases = {}
    # on-grid 32x32; half of a 64x64 grid in random order; 1021 tokens of it (padded last cluster)
    ys, xs = torch.meshgrid(torch.arange(32), torch.arange(32), indexing="ij")
    cases["grid"] = (torch.stack([xs, ys], -1).reshape(1, -1, 2).float().repeat(2, 1, 1), 32)
    ys, xs = torch.meshgrid(torch.arange(64), torch.arange(64), indexing="ij")
    full = torch.stack([xs, ys], -1).reshape(-1, 2).float()
    half = torch.stack([full[torch.randperm(4096, generator=g)[:2048]] for _ in range(2)])
    cases["half"] = (half, 64)
    cases["ragged"] = (half[:, :1021].contiguous(), 64)
    for tag, (pos, hw) in cases.items():
        p2, means, member, cmask, order = geo.space_filling_cluster(pos, 8, hw, hw, no_reorder=False)
        npz(f"clusters_{tag}", pos=pos, hw=hw, pos_out=p2, means=means, member=member, order=order.squeeze(2),
            cmask=cmask if cmask is not None else np.zeros(0))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AFFMAE_REFERENCE"),
                    help="checkout of najafian-lab/affmae (or set AFFMAE_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give the reference checkout with --reference or AFFMAE_REFERENCE")
    R = load_reference(a.reference)
    R["_root"] = a.reference
    torch.set_num_threads(1)
    for fn in [gen_knn, gen_local_attn, gen_weighted, gen_deform, gen_ms, gen_clusters][int(os.environ.get("GOLDEN_FROM", "0")):]:
        t = time.time()
        print(fn.__name__, flush=True)
        fn(R)
        print(f"  {time.time() - t:.1f}s", flush=True)


if __name__ == "__main__":
    main()
