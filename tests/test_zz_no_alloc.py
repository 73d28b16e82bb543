"""The allocation-free deformable-attention entry point, called through the C ABI.

affb_deform_knn_fwd_noalloc exists for callers that may not allocate device
memory on the call path (their memory belongs to another allocator or pool,
and a cudaMalloc there would synchronise the device and escape its budget).
It builds its spatial grid in a fixed device array instead of a workspace.
This test checks, on two calls in a row, that it returns the same output,
neighbour indices and distances as affb_deform_knn_fwd given a workspace.
The file is collected last on purpose.
"""
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _inputs(device, seed):
    from affmae_b200.workloads import deform_inputs
    return deform_inputs(B=2, side=40, level_side=20, H=8, C=32, dtype=torch.bfloat16, seed=seed, device=device)


def _run(nat, d, noalloc):
    B, Nq, _ = d["query_pos"].shape
    Nkv = d["kv_pos"].shape[1]
    H, C = d["values"].shape[2], d["values"].shape[3]
    dev = d["values"].device
    out = torch.empty((B, Nq, H, C), dtype=d["values"].dtype, device=dev)
    idx = torch.empty((B, Nq, H, 4, 4), dtype=torch.int32, device=dev)
    d2 = torch.empty((B, Nq, H, 4, 4), dtype=torch.float32, device=dev)
    power = nat.scalar_dev(d["power"], dev)
    common = [nat.ptr(d["query_pos"]), nat.ptr(d["kv_pos"]), nat.ptr(d["offsets"]),
              nat.ptr(d["attn_weights"]), nat.ptr(d["values"]), nat.ptr(power), nat.dcode(d["values"]),
              B, Nq, Nkv, H, C, nat.ptr(out), nat.ptr(idx), nat.ptr(d2)]
    if noalloc:
        nat.call("affb_deform_knn_fwd_noalloc", *common, nat.stream(dev))
    else:
        ws = torch.empty(int(nat.lib().affb_deform_workspace_bytes(B, Nkv)), dtype=torch.uint8, device=dev)
        nat.call("affb_deform_knn_fwd", *common, nat.ptr(ws), nat.stream(dev))
    torch.cuda.synchronize()
    return out, idx, d2


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    from affmae_b200 import _native as nat
    for seed in (0, 1):  # two calls in a row, different inputs: no state carried over
        d = _inputs(cuda, seed)
        ref = _run(nat, d, noalloc=False)
        got = _run(nat, d, noalloc=True)
        assert torch.equal(got[1], ref[1])
        assert torch.equal(got[2], ref[2])
        assert rel_err(got[0].float(), ref[0].float()) < 1e-5


def test_noalloc_near_capacity(cuda):
    """A grid that just fits the fixed array (close to its whole size): the
    layout inside the array matches the workspace entry point bit for bit."""
    from affmae_b200 import _native as nat
    lib = nat.lib()
    cap = int(lib.affb_deform_noalloc_max_scratch_bytes())
    lo, hi = 1, cap
    while lo < hi:  # largest kv count of one image whose grid fits
        mid = (lo + hi + 1) // 2
        if int(lib.affb_deform_workspace_bytes(1, mid)) <= cap:
            lo = mid
        else:
            hi = mid - 1
    nkv = lo
    assert int(lib.affb_deform_workspace_bytes(1, nkv)) > 0.95 * cap
    g = torch.Generator().manual_seed(3)
    side = float(nkv) ** 0.5
    d = dict(query_pos=(torch.rand((1, 256, 2), generator=g) * side).to(cuda),
             kv_pos=(torch.rand((1, nkv, 2), generator=g) * side).to(cuda),
             offsets=torch.randn((1, 256, 1, 4, 2), generator=g).to(cuda),
             attn_weights=torch.softmax(torch.randn((1, 256, 1, 4), generator=g), -1).to(cuda),
             values=torch.randn((1, nkv, 1, 8), generator=g).to(cuda, torch.bfloat16),
             power=torch.tensor(1.0, device=cuda))
    for _ in range(2):
        ref = _run(nat, d, noalloc=False)
        got = _run(nat, d, noalloc=True)
        assert torch.equal(got[1], ref[1]) and torch.equal(got[2], ref[2])
        assert torch.equal(got[0], ref[0])


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    from affmae_b200 import _native as nat
    cap = int(nat.lib().affb_deform_noalloc_max_scratch_bytes())
    big_nkv = cap // 16 + 1  # more kv points than the grid scratch can hold
    with pytest.raises(RuntimeError, match="fixed"):
        nat.call("affb_deform_knn_fwd_noalloc", None, None, None, None, None, None, 2, 1, 1, big_nkv, 8, 32,
                 None, None, None, None)
