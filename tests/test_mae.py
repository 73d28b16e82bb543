"""AFF-small MAE pretraining path (config 5): token clustering against the
reference's own space_filling_cluster (golden fixtures), the data-parallel
training harness on CPU with gloo, and the model on the GPU kernels."""
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from conftest import golden


@pytest.mark.parametrize("tag", ["grid", "half", "ragged"])
def test_curve_clusters_golden(tag):
    from affmae_b200.mae import curve_clusters
    g = golden(f"clusters_{tag}")
    hw = int(g["hw"])
    pos, means, cmask, order = curve_clusters(g["pos"], 8, hw, hw)
    assert torch.equal(order, g["order"])
    assert torch.equal(pos, g["pos_out"])
    torch.testing.assert_close(means, g["means"], rtol=1e-6, atol=1e-5)
    if g["cmask"].numel():
        assert torch.equal(cmask, g["cmask"])
    else:
        assert cmask is None


def test_param_groups():
    from affmae_b200.pretrain import param_groups
    m = nn.Sequential(nn.Linear(4, 8), nn.LayerNorm(8), nn.Linear(8, 2))
    decay, no_decay = param_groups(m, 0.05)
    assert decay["weight_decay"] == 0.05 and no_decay["weight_decay"] == 0.0
    assert {id(p) for p in decay["params"]} == {id(m[0].weight), id(m[2].weight)}
    assert len(no_decay["params"]) == 4


class _Toy(nn.Module):
    def __init__(self):
        super().__init__()
        self.net = nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 16))

    def forward(self, x):
        loss = ((self.net(x) - x) ** 2).mean()
        return loss, [loss]


def _ddp_worker(rank, world, port, batch, out):
    import torch.distributed as dist
    from affmae_b200.pretrain import make_optimizer, train_step, wrap_ddp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    model = wrap_ddp(_Toy())
    opt = make_optimizer(model)
    half = batch.shape[0] // world
    for _ in range(3):
        train_step(model, opt, batch[rank * half:(rank + 1) * half])
    torch.save({k: v.clone() for k, v in model.module.state_dict().items()}, f"{out}.{rank}")
    dist.destroy_process_group()


def test_ddp_step_matches_single_process(tmp_path):
    """Two gloo ranks, each on half the batch, end with the parameters of one
    process stepping on the whole batch (gradients averaged across ranks)."""
    import torch.multiprocessing as mp
    from affmae_b200.pretrain import make_optimizer, train_step
    torch.manual_seed(1)
    batch = torch.randn(8, 16)
    out = str(tmp_path / "state")
    port = 29500 + (os.getpid() % 1000)
    mp.spawn(_ddp_worker, args=(2, port, batch, out), nprocs=2, join=True)
    torch.manual_seed(0)
    ref = _Toy()
    opt = make_optimizer(ref)
    for _ in range(3):
        train_step(ref, opt, batch)
    s0, s1 = torch.load(f"{out}.0"), torch.load(f"{out}.1")
    for k, v in ref.state_dict().items():
        assert torch.equal(s0[k], s1[k]), k
        torch.testing.assert_close(s0[k], v, rtol=2e-2, atol=2e-3)


@pytest.mark.gpu
def test_neighbourhood_on_gpu_matches_exact_knn(cuda):
    """member_idx / pe_idx of a stage built on the GPU (KNN kernel) equal the
    ones from an exact CPU nearest-cluster search."""
    from affmae_b200.mae import curve_clusters, neighbourhood
    from affmae_b200.workloads import REL_POS_WIDTH, TABLE_WIDTH
    g = golden("clusters_ragged")
    pos, means, cmask, _ = curve_clusters(g["pos"].to(cuda), 8, 64, 64)
    member, mask, pe = neighbourhood(pos, means, cmask, 48, 8)
    d = torch.cdist(pos.cpu().double(), means.cpu().double()) ** 2
    near = torch.sort(d, dim=-1, stable=True)[1][..., :6]
    raw = (near[..., None] * 8 + torch.arange(8)).reshape(*near.shape[:2], 48)
    n = pos.shape[1]
    assert member.dtype == torch.int32
    assert torch.equal(member.cpu().long(), torch.where(raw < n, raw, torch.zeros_like(raw)))
    assert torch.equal(mask.cpu(), raw < n)
    nb = pos.cpu()[torch.arange(2)[:, None, None], member.cpu()]
    rel = (nb - (pos.cpu()[:, :, None] - REL_POS_WIDTH)).clamp(0, TABLE_WIDTH - 1)
    assert torch.equal(pe.cpu(), (rel[..., 1] * TABLE_WIDTH + rel[..., 0]).long())


@pytest.mark.gpu
def test_mae_small_training_steps(cuda):
    """A reduced config 5 (128 px images) trains on the GPU kernels: finite
    losses, every parameter receives a gradient, the loss moves."""
    from affmae_b200.mae import MAEConfig
    from affmae_b200.pretrain import build, synthetic_images, train_step
    cfg = MAEConfig(img_size=128)
    model, opt = build(cfg, device=cuda)
    imgs = synthetic_images(2, 128, 0, device=cuda)
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        loss, parts = model(imgs)
    loss.backward()
    missing = [n for n, p in model.named_parameters() if p.grad is None]
    assert not missing, missing
    opt.zero_grad(set_to_none=True)
    losses = [float(train_step(model, opt, imgs)) for _ in range(4)]
    assert all(np.isfinite(losses)), losses
    assert len(set(losses)) > 1


def _mae_ddp_worker(rank, world, port, imgs, noise, out):
    import torch.distributed as dist
    from affmae_b200.mae import MAEConfig
    from affmae_b200.pretrain import build
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    cfg = MAEConfig(img_size=128, drop_path_rate=0.0, decoder_dropout=0.0)
    model, _ = build(cfg, device=dev, ddp=True, seed=0)
    half = imgs.shape[0] // world
    sl = slice(rank * half, (rank + 1) * half)
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        loss, _ = model(imgs[sl].to(dev), noise=noise[sl].to(dev))
    loss.backward()
    grads = {n: p.grad.detach().float().cpu() for n, p in model.module.named_parameters()}
    if rank == 0:
        torch.save(grads, out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_mae_ddp_two_gpus_matches_single_gpu(cuda, tmp_path):
    """Config 5's data-parallel step over NCCL on two GPUs: each rank takes half
    of the batch; the gradients DDP all-reduces equal those of one GPU on the
    whole batch (same weights, same masks, no dropout), within bf16 tolerance."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from affmae_b200.mae import MAEConfig
    from affmae_b200.pretrain import build, synthetic_images
    cfg = MAEConfig(img_size=128, drop_path_rate=0.0, decoder_dropout=0.0)
    imgs = synthetic_images(4, 128, seed=3, device="cpu")
    L = (128 // cfg.patch_size) ** 2
    noise = torch.rand((4, L), generator=torch.Generator().manual_seed(4))
    out = str(tmp_path / "ddp_grads.pt")
    port = 29700 + (os.getpid() % 1000)
    mp.spawn(_mae_ddp_worker, args=(2, port, imgs, noise, out), nprocs=2, join=True)
    model, _ = build(cfg, device=cuda, ddp=False, seed=0)
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        loss, _ = model(imgs.to(cuda), noise=noise.to(cuda))
    loss.backward()
    ddp = torch.load(out)
    num = den = 0.0
    for n, p in model.named_parameters():
        g = p.grad.detach().float().cpu()
        num += float((ddp[n] - g).pow(2).sum())
        den += float(g.pow(2).sum())
        assert torch.isfinite(ddp[n]).all(), n
    assert (num / den) ** 0.5 < 2e-2, (num / den) ** 0.5


@pytest.mark.gpu
@pytest.mark.parametrize("C,scale,dtype", [(1, 4, torch.float32), (48, 2, torch.bfloat16), (96, 1, torch.bfloat16),
                                           (12, 2, torch.float32)])
def test_token_mask_matches_upsampled_multiply(cuda, C, scale, dtype):
    """The patch stem's re-masking kernel equals x * repeat_interleave(mask)
    bit for bit, forward and gradient (reference aff.py:591-639)."""
    from affmae_b200.kernels.token_mask import apply_token_mask
    g = torch.Generator().manual_seed(C)
    B, th, tw = 2, 16, 16
    tm = (torch.rand((B, th, tw), generator=g) > 0.5).float().to(cuda)
    x = torch.randn((B, C, th * scale, tw * scale), generator=g).to(cuda, dtype)
    x = x.contiguous(memory_format=torch.channels_last).requires_grad_(True)
    up = tm.repeat_interleave(scale, 1).repeat_interleave(scale, 2)[:, None].to(dtype)
    out = apply_token_mask(x, tm)
    assert torch.equal(out, x.detach() * up)
    gy = torch.randn(out.shape, generator=g).to(cuda, dtype)
    (gx,) = torch.autograd.grad(out, x, gy)
    assert torch.equal(gx, gy * up)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1021, 1024])
def test_neighbour_list_kernel_matches_torch_sequence(cuda, n):
    """The neighbour-list kernel equals the reference's PyTorch sequence
    (aff.py:445-465: expand the nearest clusters, zero the padding, gather the
    positions, clamp the offsets, index the table) bit for bit, also for
    positions off the integer grid (the stage-4 tokens of a merged stage)."""
    from affmae_b200.mae import neighbourhood
    from affmae_b200.workloads import REL_POS_WIDTH, TABLE_WIDTH
    g = torch.Generator().manual_seed(n)
    pos = (torch.rand((2, n, 2), generator=g) * 180).to(cuda)
    k = (n + 7) // 8
    means = (torch.rand((2, k, 2), generator=g) * 180).to(cuda)
    cmask = torch.ones((2, k, 8), device=cuda) if n % 8 else None
    member, mask, pe = neighbourhood(pos, means, cmask, 48, 8)
    from affmae_b200.kernels.knn import knn
    nearest = knn(pos, means, 6)
    raw = (nearest[..., None] * 8 + torch.arange(8, device=cuda)).reshape(2, n, 48)
    ref_member = torch.where(raw < n, raw, torch.zeros_like(raw))
    nb = pos.gather(1, ref_member.reshape(2, -1, 1).expand(-1, -1, 2)).reshape(2, n, 48, 2)
    rel = (nb - (pos[:, :, None] - REL_POS_WIDTH)).clamp(0, TABLE_WIDTH - 1)
    ref_pe = (rel[..., 1] * TABLE_WIDTH + rel[..., 0]).long()
    assert torch.equal(member.long(), ref_member)
    assert torch.equal(pe, ref_pe)
    if n % 8:
        assert torch.equal(mask, raw < n)
    else:
        assert mask is None
