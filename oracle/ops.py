"""Vectorised CPU restatement of the reference operators (test infrastructure).

Floating-point math runs in float64 on torch CPU tensors unless a step must
reproduce the reference's fp32 rounding (KNN distances, sample positions), in
which case it is done in float32 with every product and sum rounded
separately, as the reference Triton kernels do under the interpreter.
"""
from __future__ import annotations

import numpy as np
import torch

F64 = torch.float64


def _t(x, dtype=None):
    t = torch.as_tensor(x)
    t = t.detach().cpu()
    return t.to(dtype) if dtype is not None else t


# ---------------------------------------------------------------------------
# KNN — src/layers/kernels/knn.py:258-338 (K<=8 streaming top-K: strict '<'
# insertion in ascending index order => ties keep the lower index), with the
# same rule extended to every K (the reference's K>8 path, knn.py:1312, uses
# cdist+topk whose tie order is unspecified).
# ---------------------------------------------------------------------------
def _sqdist_f32(q, r):
    """q [..., M, D], r [..., N, D] float32 -> [..., M, N] float32, left-to-right."""
    d = None
    for k in range(q.shape[-1]):
        diff = q[..., :, None, k] - r[..., None, :, k]
        sq = diff * diff
        d = sq if d is None else d + sq
    return d


def _topk_stable(d, k):
    """Indices of the k smallest entries of each row, ties by lower index."""
    # (d, index) packed into one unique uint64 key: non-negative fp32 values
    # order like their bit patterns, so the key order is the (d, index) order;
    # a partition then a sort of the k smallest keys is exact and avoids a full sort.
    n = d.shape[-1]
    if k >= n or d.dtype != np.float32 or (d < 0).any() or np.isnan(d).any():
        return np.argsort(d, axis=-1, kind="stable")[..., :k]
    key = (d.view(np.uint32).astype(np.uint64) << np.uint64(32)) | np.arange(n, dtype=np.uint64)
    part = np.partition(key, k - 1, axis=-1)[..., :k]
    part.sort(axis=-1)
    return (part & np.uint64(0xFFFFFFFF)).astype(np.int64)


def knn(query, ref, k, chunk=512):
    """int64 [B, M, k] (reference knn.py:1615 contract, exact tie rule)."""
    q = np.ascontiguousarray(_t(query, torch.float32).numpy())
    r = np.ascontiguousarray(_t(ref, torch.float32).numpy())
    B, M, _ = q.shape
    out = np.empty((B, M, k), dtype=np.int64)
    for b in range(B):
        for m0 in range(0, M, chunk):
            d = _sqdist_f32(q[b, m0:m0 + chunk], r[b])
            out[b, m0:m0 + chunk] = _topk_stable(d, k)
    return torch.from_numpy(out)


# ---------------------------------------------------------------------------
# Neighbourhood attention — local_attn.py:80-340 (fwd), :350-553 (bwd).
# ---------------------------------------------------------------------------
def _padded_neighbours(M):
    # smallest_valid_power_2 block width, local_attn.py:46-57
    bn = 32 if M >= 32 else 16 if M >= 16 else 8 if M >= 8 else 4 if M >= 4 else 1
    return -(-M // bn) * bn


def _gather_rows(x, mi):
    """x [B,H,N,D], mi [B,N,M] -> [B,H,N,M,D]."""
    B = x.shape[0]
    bidx = torch.arange(B)[:, None, None]
    g = x.permute(0, 2, 1, 3)[bidx, mi]  # [B,N,M,H,D]
    return g.permute(0, 3, 1, 2, 4)


def _valid(mask, B, H, N, M):
    if mask is None:
        return torch.ones((B, H, N, M), dtype=torch.bool)
    m = _t(mask)
    if m.dim() == 3:
        m = m[:, None]
    return (m > 0).expand(B, H, N, M)


def _nbhd_logits(q, k, mi, bias, mask, scale):
    B, H, N, D = q.shape
    M = mi.shape[-1]
    kg = _gather_rows(k, mi)
    valid = _valid(mask, B, H, N, M)
    s = scale * (q[:, :, :, None, :] * kg).sum(-1)
    if bias is not None:
        s = s + _t(bias, F64)
    s = torch.where(valid, s, torch.full_like(s, -1e11))
    return s, valid, kg


def nbhd_attn_fwd(q, k, v, mi, scale, bias=None, mask=None, blank_k=None, blank_v=None):
    """Kernel semantics of _nbhood_attn_fwd: returns (o [B,H,N,D], lse [B,H,N]) in float64."""
    q, k, v = _t(q, F64), _t(k, F64), _t(v, F64)
    mi = _t(mi, torch.int64)
    B, H, N, D = q.shape
    M = mi.shape[-1]
    s, valid, _ = _nbhd_logits(q, k, mi, bias, mask, scale)
    vg = _gather_rows(v, mi) * valid[..., None]
    cols = [s]
    vals = [vg]
    pad = _padded_neighbours(M) - M
    if pad:
        cols.append(torch.full((B, H, N, pad), -1e11, dtype=F64))
        vals.append(torch.zeros((B, H, N, pad, D), dtype=F64))
    if blank_k is not None:
        bk, bv = _t(blank_k, F64), _t(blank_v, F64)
        cols.append((scale * (q * bk[None, :, None, :]).sum(-1))[..., None])
        vals.append(bv[None, :, None, None, :].expand(B, H, N, 1, D))
    logits = torch.cat(cols, -1)
    vall = torch.cat(vals, -2)
    m = logits.max(-1, keepdim=True).values
    p = torch.exp(logits - m)
    l = p.sum(-1, keepdim=True)
    lse = m + torch.log(l + 1e-12)
    o = (torch.exp(logits - lse)[..., None] * vall).sum(-2)
    return o, lse[..., 0]


def nbhd_attn_bwd(q, k, v, mi, scale, o, lse, do, bias=None, mask=None, blank_k=None, blank_v=None):
    """Kernel semantics of _nbhood_attn_bwd_internal (local_attn.py:387-553).

    Returns (dq, dk, dv, dbias | None, dblank_k | None, dblank_v | None) in float64.
    """
    q, k, v = _t(q, F64), _t(k, F64), _t(v, F64)
    o, lse, do = _t(o, F64), _t(lse, F64), _t(do, F64)
    mi = _t(mi, torch.int64)
    B, H, N, D = q.shape
    M = mi.shape[-1]
    s, valid, kg = _nbhd_logits(q, k, mi, bias, mask, scale)
    kg = kg * valid[..., None]
    vg = _gather_rows(v, mi) * valid[..., None]
    delta = (o * do).sum(-1)
    p = torch.exp(s - lse[..., None])
    dp = (do[:, :, :, None, :] * vg).sum(-1)
    ds = p * (dp - delta[..., None])
    ds_v = torch.where(valid, ds, torch.zeros_like(ds))
    dq = (ds_v[..., None] * kg).sum(-2)
    dk = torch.zeros_like(k)
    dv = torch.zeros_like(v)
    # scatter: dk[b,h,mi[b,n,m]] += scale*ds*q ; dv[...] += p*do
    contrib_k = scale * ds_v[..., None] * q[:, :, :, None, :]
    contrib_v = (p * valid)[..., None] * do[:, :, :, None, :]
    flat = (torch.arange(B)[:, None, None, None] * (H * N) + torch.arange(H)[None, :, None, None] * N
            + mi[:, None, :, :]).reshape(-1)
    dk.view(-1, D).index_add_(0, flat, contrib_k.reshape(-1, D))
    dv.view(-1, D).index_add_(0, flat, contrib_v.reshape(-1, D))
    dbias = ds_v if bias is not None else None
    dbk = dbv = None
    if blank_k is not None:
        bk, bv = _t(blank_k, F64), _t(blank_v, F64)
        sb = scale * (q * bk[None, :, None, :]).sum(-1)
        pb = torch.exp(sb - lse)
        dpb = (do * bv[None, :, None, :]).sum(-1)
        dsb = pb * (dpb - delta)
        dq = dq + dsb[..., None] * bk[None, :, None, :]
        dbk = scale * (dsb[..., None] * q).sum((0, 2))
        dbv = (pb[..., None] * do).sum((0, 2))
    return scale * dq, dk, dv, dbias, dbk, dbv


def nbhd_blank_grads(q, scale, lse, o, do, blank_k, blank_v):
    """(dblank_k [H,D], dblank_v [H,D]) in float64 from the per-row blank terms
    of nbhd_attn_bwd (local_attn.py:530-550); needs no neighbour gather, so it
    runs on whole large batches."""
    q, o, do, lse = _t(q, F64), _t(o, F64), _t(do, F64), _t(lse, F64)
    bk, bv = _t(blank_k, F64), _t(blank_v, F64)
    delta = (o * do).sum(-1)
    sb = scale * (q * bk[None, :, None, :]).sum(-1)
    pb = torch.exp(sb - lse)
    dsb = pb * ((do * bv[None, :, None, :]).sum(-1) - delta)
    return scale * (dsb[..., None] * q).sum((0, 2)), (pb[..., None] * do).sum((0, 2))


def nbhd_attn_formula(q, k, v, mi, scale, bias=None, mask=None, blank_k=None, blank_v=None):
    """The reference's own PyTorch formula (local_attn.py:979-1006: gathered
    scores + bias, masked_fill(-inf), softmax with the blank logit appended),
    differentiable; inputs are used as given (use float64 leaves for grads)."""
    B, H, N, D = q.shape
    M = mi.shape[-1]
    mi = mi.to(torch.int64)
    kg = _gather_rows(k, mi)
    vg = _gather_rows(v, mi)
    scores = (q[:, :, :, None, :] * kg).sum(-1) * scale
    if bias is not None:
        scores = scores + bias
    if mask is not None:
        m = mask if mask.dim() == 4 else mask[:, None]
        scores = scores.masked_fill(m.expand(B, H, N, M) == 0, float("-inf"))
    cols = [scores]
    if blank_k is not None:
        cols.append((q * blank_k.view(1, H, 1, D)).sum(-1, keepdim=True) * scale)
    attn = torch.softmax(torch.cat(cols, -1), -1)
    out = (attn[..., :M, None] * vg).sum(-2)
    if blank_k is not None:
        out = out + attn[..., M:] * blank_v.view(1, H, 1, D)
    return out


# ---------------------------------------------------------------------------
# Weighted features / gather — weighted_features.py:440-457 (formula),
# kernels :30-345; weighted_gather.py:410-411.
# ---------------------------------------------------------------------------
def _gather_feat(feat, idx):
    B, No, M = idx.shape
    C = feat.shape[-1]
    g = feat.gather(1, idx.reshape(B, No * M)[..., None].expand(-1, -1, C))
    return g.reshape(B, No, M, C)


def weighted_features_fwd(w, feat, idx):
    """w [B,No,M,IC], feat [B,N,C], idx [B,No,M] -> [B,No,IC,C] (float64)."""
    w, feat, idx = _t(w, F64), _t(feat, F64), _t(idx, torch.int64)
    return torch.einsum("bnmi,bnmc->bnic", w, _gather_feat(feat, idx))


def weighted_features_bwd(dout, w, feat, idx):
    """Returns (dw [B,No,M,IC], dfeat [B,N,C]) in float64."""
    dout, w, feat = _t(dout, F64), _t(w, F64), _t(feat, F64)
    idx = _t(idx, torch.int64)
    B, No, M = idx.shape
    C = feat.shape[-1]
    g = _gather_feat(feat, idx)
    dw = torch.einsum("bnmc,bnic->bnmi", g, dout)
    contrib = torch.einsum("bnmi,bnic->bnmc", w, dout)
    dfeat = torch.zeros_like(feat)
    flat = (torch.arange(B)[:, None, None] * feat.shape[1] + idx).reshape(-1)
    dfeat.view(-1, C).index_add_(0, flat, contrib.reshape(-1, C))
    return dw, dfeat


# ---------------------------------------------------------------------------
# Fused KNN deformable attention — fused_deform_attn.py:1342-1509 (fwd, cross;
# self = cross with kv_pos = pos), :1982-2381 (bwd).
# ---------------------------------------------------------------------------
def _samples(qpos, offsets):
    qp = _t(qpos, torch.float32)
    off = _t(offsets, torch.float32)
    return qp[:, :, None, None, :] + off  # float32 add, [B,Nq,H,4,2]


def _knn4(samp, kv, chunk=4096):
    """Exact top-4 over kv for every sample, (d2, index) order. Returns idx int64, d2 float32."""
    B = samp.shape[0]
    s = samp.reshape(B, -1, 2).numpy()
    r = _t(kv, torch.float32).numpy()
    idx = np.empty(s.shape[:2] + (4,), dtype=np.int64)
    d2 = np.empty(s.shape[:2] + (4,), dtype=np.float32)
    for b in range(B):
        for i0 in range(0, s.shape[1], chunk):
            d = _sqdist_f32(s[b, i0:i0 + chunk], r[b])
            top = _topk_stable(d, 4)
            idx[b, i0:i0 + chunk] = top
            d2[b, i0:i0 + chunk] = np.take_along_axis(d, top, -1)
    shp = samp.shape[:-1] + (4,)
    return torch.from_numpy(idx).reshape(shp), torch.from_numpy(d2).reshape(shp)


def _shepard(d2, power):
    P = max(float(power), 1e-6)
    dist = torch.sqrt(d2.to(F64)) + 1e-6
    lg = -P * dist
    e = torch.exp(lg - lg.max(-1, keepdim=True).values)
    return e / (e.sum(-1, keepdim=True) + 1e-8), dist, P


def _gather_val(values, idx):
    """values [B,Nkv,H,C], idx [B,Nq,H,4,4] -> [B,Nq,H,4,4,C]."""
    B, Nq, H = idx.shape[:3]
    bi = torch.arange(B)[:, None, None, None, None]
    hi = torch.arange(H)[None, None, :, None, None]
    return values[bi, idx, hi]


def deform_knn_fwd(query_pos, kv_pos, offsets, attn_w, values, power):
    """Returns (out [B,Nq,H,C] float64, knn_idx int64, knn_d2 float32)."""
    samp = _samples(query_pos, offsets)
    idx, d2 = _knn4(samp, kv_pos)
    w, _, _ = _shepard(d2, power)
    vg = _gather_val(_t(values, F64), idx)
    aw = _t(attn_w, F64)
    out = (aw[..., None] * (w[..., None] * vg).sum(-2)).sum(-2)
    return out, idx, d2


def deform_knn_bwd(dout, query_pos, kv_pos, offsets, attn_w, values, power, knn_idx, knn_d2,
                   self_attn=False):
    """Returns (d_qpos, d_kvpos, d_offsets, d_attn_w, d_values, d_power) in float64.
    For self-attention d_qpos already includes the neighbour part and d_kvpos is None."""
    samp = _samples(query_pos, offsets).to(F64)
    idx = _t(knn_idx, torch.int64)
    w, dist, P = _shepard(_t(knn_d2, torch.float32), power)
    vals = _t(values, F64)
    vg = _gather_val(vals, idx)
    g = _t(dout, F64)
    aw = _t(attn_w, F64)
    B, Nq, H = idx.shape[:3]
    Nkv = vals.shape[1]
    dot = (vg * g[:, :, :, None, None, :]).sum(-1)            # [B,Nq,H,4,4]
    d_aw = (w * dot).sum(-1)
    dp = aw[..., None] * dot
    wdp = (w * dp).sum(-1, keepdim=True)
    ds = w * (dp - wdp)
    d_power = (ds * (-dist)).sum()
    dd2 = (ds * (-P)) / (2.0 * dist)
    kv = _t(kv_pos, F64)
    bi = torch.arange(B)[:, None, None, None, None]
    kvn = kv[bi, idx]                                          # [B,Nq,H,4,4,2]
    diff = samp[..., None, :] - kvn
    d_off = 2.0 * (diff * dd2[..., None]).sum(-2)
    d_qpos = d_off.sum((2, 3))
    d_kv = torch.zeros((B, Nkv, 2), dtype=F64)
    flat = (torch.arange(B)[:, None, None, None, None] * Nkv + idx).reshape(-1)
    d_kv.view(-1, 2).index_add_(0, flat, (-2.0 * diff * dd2[..., None]).reshape(-1, 2))
    d_val = torch.zeros_like(vals)
    C = vals.shape[-1]
    cf = aw[..., None] * w                                     # [B,Nq,H,4,4]
    contrib = cf[..., None] * g[:, :, :, None, None, :]
    hidx = torch.arange(H)[None, None, :, None, None]
    flat_v = ((torch.arange(B)[:, None, None, None, None] * Nkv + idx) * H + hidx).reshape(-1)
    d_val.view(-1, C).index_add_(0, flat_v, contrib.reshape(-1, C))
    if self_attn:
        return d_qpos + d_kv, None, d_off, d_aw, d_val, d_power
    return d_qpos, d_kv, d_off, d_aw, d_val, d_power


# ---------------------------------------------------------------------------
# Deformable attention with given neighbours — fused_deform_attn.py:79-231
# (fwd) and :252-491 (bwd, note max(dist - 1e-6, 1e-8) in the denominator).
# MSSample — mssample.py:17-297 (sqrt(d2 + 1e-6)); MSDETRPC — msdetrpc.py:25-299.
# ---------------------------------------------------------------------------
def _nb_geometry(sl, kv, nb, eps_inside):
    sl = _t(sl, torch.float32)
    kv = _t(kv, torch.float32)
    nb = _t(nb, torch.int64)
    B = sl.shape[0]
    bi = torch.arange(B)[:, None, None]
    p = kv[bi, nb]                                  # [B,N,K,D] float32
    diff = sl[:, :, None, :] - p
    sq = diff * diff
    d2 = sq[..., 0]
    for d in range(1, sq.shape[-1]):
        d2 = d2 + sq[..., d]
    d2 = d2.to(F64)
    dist = torch.sqrt(d2 + 1e-6) if eps_inside else torch.sqrt(d2) + 1e-6
    return dist, diff.to(F64), nb


def _softmax_neg(dist, power):
    P = max(float(power), 1e-6)
    lg = -P * dist
    e = torch.exp(lg - lg.max(-1, keepdim=True).values)
    return e / (e.sum(-1, keepdim=True) + 1e-8), P


def deform_nbidx_fwd(sl, kv, nb, power, attn_w, values):
    dist, _, nb = _nb_geometry(sl, kv, nb, False)
    w, _ = _softmax_neg(dist, power)
    vals = _t(values, F64)
    bi = torch.arange(vals.shape[0])[:, None, None]
    vg = vals[bi, nb]                               # [B,N,K,C]
    return _t(attn_w, F64)[..., None] * (w[..., None] * vg).sum(-2)


def deform_nbidx_bwd(dout, sl, kv, nb, power, attn_w, values):
    """Returns (d_sl, d_kv, d_power, d_attn, d_values) in float64."""
    dist, diff, nb = _nb_geometry(sl, kv, nb, False)
    w, P = _softmax_neg(dist, power)
    vals = _t(values, F64)
    B, Nkv, C = vals.shape
    bi = torch.arange(B)[:, None, None]
    vg = vals[bi, nb]
    g = _t(dout, F64)
    a = _t(attn_w, F64)
    dot = (vg * g[:, :, None, :]).sum(-1)
    d_attn = (w * dot).sum(-1)
    dnw = a[..., None] * dot
    dl = w * (dnw - (dnw * w).sum(-1, keepdim=True))
    d_power = (dl * (-dist)).sum()
    dd = -P * dl
    den = torch.clamp(dist - 1e-6, min=1e-8)
    gdiff = dd[..., None] * diff / den[..., None]
    d_sl = gdiff.sum(-2)
    D = diff.shape[-1]
    d_kv = torch.zeros((B, Nkv, D), dtype=F64)
    flat = (torch.arange(B)[:, None, None] * Nkv + nb).reshape(-1)
    d_kv.view(-1, D).index_add_(0, flat, (-gdiff).reshape(-1, D))
    d_val = torch.zeros_like(vals)
    contrib = (a[..., None] * w)[..., None] * g[:, :, None, :]
    d_val.view(-1, C).index_add_(0, flat, contrib.reshape(-1, C))
    return d_sl, d_kv, d_power, d_attn, d_val


def mssample_fwd(sl, kv, nb, power):
    dist, _, _ = _nb_geometry(sl, kv, nb, True)
    w, _ = _softmax_neg(dist, power)
    return w[..., None]


def mssample_bwd(dw, sl, kv, nb, power, w):
    dist, diff, nb = _nb_geometry(sl, kv, nb, True)
    P = max(float(power), 1e-6)
    dw = _t(dw, F64).reshape(dist.shape)
    w = _t(w, F64).reshape(dist.shape)
    dl = w * (dw - (dw * w).sum(-1, keepdim=True))
    d_power = (dl * (-dist)).sum()
    gdiff = (dl * (-P))[..., None] * diff / (dist + 1e-8)[..., None]
    d_sl = gdiff.sum(-2)
    B = dist.shape[0]
    Nkv = _t(kv).shape[1]
    D = diff.shape[-1]
    d_kv = torch.zeros((B, Nkv, D), dtype=F64)
    flat = (torch.arange(B)[:, None, None] * Nkv + nb).reshape(-1)
    d_kv.view(-1, D).index_add_(0, flat, (-gdiff).reshape(-1, D))
    return d_sl, d_kv, d_power


def msdetrpc_fwd(idx, w, attn, val):
    idx = _t(idx, torch.int64)
    w, attn, val = _t(w, F64), _t(attn, F64), _t(val, F64)
    B = val.shape[0]
    bi = torch.arange(B)[:, None, None, None]
    vg = val[bi, idx]                                # [B,N,M,K,C]
    return (attn[..., None, None] * w[..., None] * vg).sum((2, 3))


def msdetrpc_bwd(dout, idx, w, attn, val):
    """Returns (d_w, d_attn, d_val) in float64."""
    idx = _t(idx, torch.int64)
    w, attn, val, g = _t(w, F64), _t(attn, F64), _t(val, F64), _t(dout, F64)
    B, Nv, C = val.shape
    bi = torch.arange(B)[:, None, None, None]
    vg = val[bi, idx]
    dot = (vg * g[:, :, None, None, :]).sum(-1)      # [B,N,M,K]
    d_w = attn[..., None] * dot
    d_attn = (w * dot).sum(-1)
    d_val = torch.zeros_like(val)
    contrib = (attn[..., None] * w)[..., None] * g[:, :, None, None, :]
    flat = (torch.arange(B)[:, None, None, None] * Nv + idx).reshape(-1)
    d_val.view(-1, C).index_add_(0, flat, contrib.reshape(-1, C))
    return d_w, d_attn, d_val


# ---------------------------------------------------------------------------
# Relative-position bias — attention.py:110-124 (index_select + permute).
# ---------------------------------------------------------------------------
def pos_bias_fwd(table, pe_idx):
    table = _t(table, F64)
    pe = _t(pe_idx, torch.int64)
    B, N, M = pe.shape
    H = table.shape[1]
    return table.index_select(0, pe.reshape(-1)).view(B, N, M, H).permute(0, 3, 1, 2).contiguous()


def pos_bias_bwd(dbias, pe_idx, T):
    g = _t(dbias, F64)
    pe = _t(pe_idx, torch.int64)
    H = g.shape[1]
    d = torch.zeros((T, H), dtype=F64)
    d.index_add_(0, pe.reshape(-1), g.permute(0, 2, 3, 1).reshape(-1, H))
    return d
