"""Benchmark: neighbourhood (cluster) attention forward + backward on B200.

Workload: bf16, B=32 images, N=4608 visible tokens (0.5
mask of a 96x96 grid), clusters of 8 queries attending the 48 members of their
6 nearest clusters, 4 heads x d=32, relative-position bias [B,H,N,M], blank
token.  One step = one forward + one backward call of the hot path.

  value : algorithmic bytes of fwd+bwd (interface bytes: inputs read once,
          outputs written once) / device time, inputs resident in HBM, L2
          flushed (256 MiB write) before every step outside the timed events.
  e2e   : the same bytes / time of the public autograd path
          (FlashLocalAttentionFunction.apply + backward) including the
          host->device copies of all inputs from pinned memory and the
          device->host copies of the output and all gradients, every step;
          consecutive steps overlap (inputs of the next step travel in while
          the current one computes and the previous one's results travel out).

Multi-GPU: the op has no exchange step, so N GPUs run N independent replicas
(weak scaling); value is summed over ranks using the max time over ranks.
Every run also times config 5 (AFF-small MAE pretraining, 16 images per GPU)
at the same N and reports it as the nested ``mae`` object: under DDP with an
NCCL gradient all-reduce overlapped with the backward when WORLD_SIZE > 1
(``--no-mae`` skips it; ``--workload mae`` runs it alone as the main line).

``--impl reference`` times the reference's pure-PyTorch formula of this op
(the gathered-softmax formula of local_attn.py:979-1006, autograd backward)
on the host cores on a bounded sample (one image per step).
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "nbr-attn fwd+bwd HBM GB/s"
# our kernels per timed step: the forward, and in the backward the list-counter
# clear, the list count + prologue, the list scan and fill, the query-side kernel
# (returns at once for cluster-run lists), the key-side kernel and the dQ kernel
LAUNCHES_PER_STEP = 8
CFG = dict(B=32, side=96, keep=0.5, H=4, d=32, nbhd=48)
# DRAM bytes (read + write) of one backward call per image, from one ncu capture of
# every backward kernel at B=16 (profiles/nbhd_attn_kernels_config3_b16.md: 286.2 MB);
# the traffic of each kernel grows with the batch, so it is scaled by B
BWD_DRAM_BYTES_PER_IMAGE = 286.21952e6 / 16


def workload_config(extra=None):
    c = {"workload": "neighbourhood attention fwd+bwd (config 3)", "global_batch": CFG["B"],
         "tokens": int(CFG["side"] ** 2 * CFG["keep"]), "heads": CFG["H"], "head_dim": CFG["d"],
         "neighbours": CFG["nbhd"], "bias": True, "blank": True, "mask": None,
         "cluster_order": {"curve": "reference anchor scan (geometry.py:170-319)",
                           "morton": "Z-order"}[CFG.get("order", "curve")],
         "l2": "flushed by a 256 MiB write before every timed step"}
    if extra:
        c.update(extra)
    return c


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------- helpers --
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend)
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda" if torch.cuda.is_available() else "cpu", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------ CPU baseline --
def cpu_reference_step(inp_cpu, threads):
    """The reference's PyTorch formula (local_attn.py:979-1006) on one image, fp32,
    forward + autograd backward.  Returns seconds."""
    import oracle
    torch.set_num_threads(threads)
    leaves = {n: inp_cpu[n].float().requires_grad_() for n in ("q", "k", "v", "bias", "blank_k", "blank_v")}
    t0 = time.perf_counter()
    out = oracle.nbhd_attn_formula(leaves["q"], leaves["k"], leaves["v"], inp_cpu["member_idx"],
                                   inp_cpu["scale"], bias=leaves["bias"], blank_k=leaves["blank_k"],
                                   blank_v=leaves["blank_v"])
    out.backward(inp_cpu["dout"].float())
    return time.perf_counter() - t0


def cpu_sample(inp, b=1):
    """First `b` images of the workload, on the host."""
    out = {}
    for k, v in inp.items():
        if torch.is_tensor(v) and v.dim() >= 3:
            out[k] = v[:b].detach().cpu()
        elif torch.is_tensor(v):
            out[k] = v.detach().cpu()
        else:
            out[k] = v
    return out


def bytes_for(B):
    from affmae_b200.workloads import nbhd_attention_bytes
    N = int(CFG["side"] ** 2 * CFG["keep"])
    f, b = nbhd_attention_bytes(B, CFG["H"], N, CFG["d"], CFG["nbhd"])
    return f, b


def run_reference(args, world, rank):
    if rank != 0:
        return
    from affmae_b200.workloads import nbhd_attention_inputs
    threads = os.cpu_count() or 1
    inp = nbhd_attention_inputs(B=1, dtype=torch.float32, device="cpu",
                                **{k: CFG[k] for k in ("side", "keep", "H", "d", "nbhd")})
    inp = cpu_sample(inp, 1)
    f, b = bytes_for(1)
    for _ in range(args.warmup):
        cpu_reference_step(inp, threads)
    ts = [cpu_reference_step(inp, threads) for _ in range(args.steps)]
    t = sum(ts) / len(ts)
    value = (f + b) / t / 1e9
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config({"sample": "1 of 32 images per step"}), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": "1 image (1/32 of the batch) per step, reference PyTorch formula, fp32"},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU arm --
def run_gpu(args, world, rank, local):
    from affmae_b200 import _native as nat
    from affmae_b200.workloads import nbhd_attention_inputs
    from affmae_b200.kernels.local_attn import (FlashLocalAttentionFunction, launch_flash_nbhood_attn_bwd,
                                                launch_flash_nbhood_attn_fwd)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    nat.lib()
    inp = nbhd_attention_inputs(B=CFG["B"], dtype=torch.bfloat16, seed=rank, device=dev, order=args.order,
                                **{k: CFG[k] for k in ("side", "keep", "H", "d", "nbhd")})
    q, k, v, mi, bias = inp["q"], inp["k"], inp["v"], inp["member_idx"], inp["bias"]
    bk, bv, do, scale = inp["blank_k"], inp["blank_v"], inp["dout"], inp["scale"]
    fwd_bytes, bwd_bytes = bytes_for(CFG["B"])
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        o, lse, plan = launch_flash_nbhood_attn_fwd(q, k, v, mi, scale, bias=bias, blank_k=bk, blank_v=bv,
                                                    return_plan=True)
        if ev is not None:
            ev[0].record(stream)
        g = launch_flash_nbhood_attn_bwd(q, k, v, mi, scale, o, lse, do, bias=bias, blank_k=bk, blank_v=bv,
                                         plan=plan)
        if ev is not None:
            ev[1].record(stream)
        return o, g

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- device-timed value: per-step events, L2 flushed before each step
    times, fwd_t, bwd_t = [], [], []
    barrier(world)
    torch.cuda.synchronize()
    clk = ClockSampler(local)
    clk.__enter__()
    if True:
        for _ in range(args.steps):
            flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            ef = torch.cuda.Event(enable_timing=True)
            eb0 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step((ef, e1))
            times.append((e0, ef, e1))
        torch.cuda.synchronize()
        # kernel-only bwd timing (the dominant kernel): events around the C call
        o, lse, plan = launch_flash_nbhood_attn_fwd(q, k, v, mi, scale, bias=bias, blank_k=bk, blank_v=bv,
                                                    return_plan=True)
        dq = torch.empty_like(q)
        dk = torch.empty_like(q)
        dv = torch.empty_like(q)
        dbias = torch.empty_like(bias)
        dbk = torch.zeros(bk.shape, device=dev, dtype=torch.float32)
        dbv = torch.zeros(bv.shape, device=dev, dtype=torch.float32)
        B, H, N, D = q.shape
        wsb = int(nat.lib().affb_nbhd_attn_bwd_workspace_bytes(nat.BF16, B, H, N, D, CFG["nbhd"]))
        ws = torch.empty((wsb,), device=dev, dtype=torch.uint8)
        kern_ms = []
        for _ in range(args.steps):
            flush.fill_(1)
            a = torch.cuda.Event(enable_timing=True)
            c = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            nat.call("affb_nbhd_attn_bwd_plan", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                     do.data_ptr(), lse.data_ptr(), mi.data_ptr(), bias.data_ptr(), None, 1, bk.data_ptr(),
                     bv.data_ptr(), nat.BF16, B, H, N, D, CFG["nbhd"], float(scale), dq.data_ptr(),
                     dk.data_ptr(), dv.data_ptr(), dbias.data_ptr(), dbk.data_ptr(), dbv.data_ptr(),
                     plan.data_ptr(), plan.numel(), ws.data_ptr(), wsb, stream.cuda_stream)
            c.record(stream)
            kern_ms.append((a, c))
        torch.cuda.synchronize()
    step_ms = [a.elapsed_time(c) for a, _, c in times]
    f_ms = [a.elapsed_time(f) for a, f, _ in times]
    b_ms = [f.elapsed_time(c) for _, f, c in times]
    total_s = sum(step_ms) / 1e3
    total_s = max_over_ranks(total_s, world)
    value = world * args.steps * (fwd_bytes + bwd_bytes) / total_s / 1e9
    kbwd = sum(a.elapsed_time(c) for a, c in kern_ms) / len(kern_ms)
    peak, peak_kind = measured_peaks()
    achieved = bwd_bytes / (kbwd / 1e3) / 1e9

    # ---- e2e through the public autograd API with host buffers
    # Every step copies its inputs from pinned host memory and reads its
    # output and all gradients back.  Steps are pipelined over three streams:
    # the inputs of step i+1 travel host->device while step i computes and
    # step i-1's results travel device->host (PCIe is full duplex); device
    # input buffers are double-buffered.
    def run_e2e():
        names = ("q", "k", "v", "member_idx", "bias", "blank_k", "blank_v", "dout")
        host = {n: inp[n].detach().cpu().pin_memory() for n in names}
        h2d = sum(t.numel() * t.element_size() for t in host.values())
        dev_in = [{n: torch.empty_like(t, device=dev) for n, t in host.items()} for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]
        res_ready = [torch.cuda.Event() for _ in range(2)]
        outs_host = None

        def e2e_step(i):
            nonlocal outs_host
            k = i % 2
            with torch.cuda.stream(s_in):
                s_in.wait_event(in_free[k])  # compute of step i-2 is done with these buffers
                for n in names:
                    dev_in[k][n].copy_(host[n], non_blocking=True)
                in_ready[k].record(s_in)
            stream.wait_event(in_ready[k])
            d = dev_in[k]
            leaves = {n: d[n].detach().requires_grad_() for n in ("q", "k", "v", "bias", "blank_k", "blank_v")}
            out = FlashLocalAttentionFunction.apply(leaves["q"], leaves["k"], leaves["v"], d["member_idx"],
                                                    leaves["bias"], None, leaves["blank_k"], leaves["blank_v"], scale)
            out.backward(d["dout"])
            in_free[k].record(stream)
            res = [out.detach()] + [leaves[n].grad for n in ("q", "k", "v", "bias", "blank_k", "blank_v")]
            res_ready[k].record(stream)
            if outs_host is None:  # pinned host buffers for the results, allocated once
                outs_host = [torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in res]
            with torch.cuda.stream(s_out):
                s_out.wait_event(res_ready[k])
                for hbuf, r in zip(outs_host, res):
                    hbuf.copy_(r, non_blocking=True)
                    r.record_stream(s_out)

        for i in range(max(1, args.warmup)):
            e2e_step(i)
        torch.cuda.synchronize()
        d2h = sum(t.numel() * t.element_size() for t in outs_host)
        barrier(world)
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        c = torch.cuda.Event(enable_timing=True)
        a.record(s_in)
        stream.wait_event(a)
        s_out.wait_event(a)
        for i in range(args.steps):
            e2e_step(i)
        done = torch.cuda.Event()
        done.record(s_out)
        stream.wait_event(done)
        c.record(stream)
        torch.cuda.synchronize()
        e2e_s = max_over_ranks(a.elapsed_time(c) / 1e3, world)
        e2e_value = world * args.steps * (fwd_bytes + bwd_bytes) / e2e_s / 1e9
        return e2e_value, e2e_s, h2d, d2h

    e2e_value = e2e_s = h2d = d2h = None
    if not args.no_e2e:
        e2e_value, e2e_s, h2d, d2h = run_e2e()
    clk.__exit__(None, None, None)
    clocks = clk.summary()

    # ---- CPU baseline (rank 0, N=1 only): reference formula on one image
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        sample = cpu_sample({k2: (v2.float() if torch.is_tensor(v2) and v2.is_floating_point() else v2)
                             for k2, v2 in inp.items()}, 1)
        cpu_reference_step(sample, threads)
        ts = [cpu_reference_step(sample, threads) for _ in range(3)]
        f1, b1 = bytes_for(1)
        cpu = {"value": (f1 + b1) / (sum(ts) / len(ts)) / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": "1 image (1/32 of the batch), reference PyTorch formula fwd+autograd bwd, fp32, 3 runs"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": total_s * 1e3 / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": workload_config({"parallelism": f"replicas x{world}" if world > 1 else "single GPU"}),
                "fwd_ms": statistics.median(f_ms), "bwd_ms": statistics.median(b_ms),
                "e2e": None if e2e_value is None else {
                    "value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_s * 1e3 / args.steps},
                "roofline": {"kernel": "affb_nbhd_attn_bwd_plan (list, prologue, key-side and dQ kernels)", "bound": "hbm", "achieved": achieved, "peak": peak,
                             "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                             "traffic": BWD_DRAM_BYTES_PER_IMAGE * CFG["B"],
                             "traffic_note": "ncu dram__bytes_read+write of the backward kernels at B=16, scaled by B",
                             "algorithmic_bytes": bwd_bytes, "kernel_ms": kbwd},
                "cpu_baseline": cpu, "clocks": clocks,
                "gpu_launches": args.steps * LAUNCHES_PER_STEP}
        return line
    return None


def run_mae(args, world, rank, local, steps=None, warmup=None):
    """Config 5: AFF-small MAE pretraining steps, data parallel over `world`
    GPUs (DDP, NCCL all-reduce overlapped with the backward pass).  Returns
    the JSON line on rank 0 (None elsewhere)."""
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    from affmae_b200 import _native as nat
    from affmae_b200.mae import MAEConfig
    from affmae_b200.pretrain import build, synthetic_images, train_step
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = MAEConfig()
    per_gpu = args.mae_batch
    model, opt = build(cfg, device=dev, ddp=world > 1, seed=0)
    imgs = synthetic_images(per_gpu, cfg.img_size, seed=1000 + rank, device=dev)
    gen = torch.Generator(device=dev).manual_seed(rank)
    stream = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        train_step(model, opt, imgs, generator=gen)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    calls0 = nat.CALLS
    with ClockSampler(local) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            loss = train_step(model, opt, imgs, generator=gen)
        e1.record(stream)
        torch.cuda.synchronize()
        calls = nat.CALLS - calls0
        dev_s = max_over_ranks(e0.elapsed_time(e1) / 1e3, world)
        barrier(world)
        # e2e: every step copies its images from pinned host memory and reads the loss back
        host = imgs.cpu().pin_memory()
        loss_host = torch.empty((), dtype=torch.float32).pin_memory()
        torch.cuda.synchronize()
        barrier(world)
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for _ in range(steps):
            x = host.to(dev, non_blocking=True)
            loss = train_step(model, opt, x, generator=gen)
            loss_host.copy_(loss.float(), non_blocking=True)
        e3.record(stream)
        torch.cuda.synchronize()
        e2e_s = max_over_ranks(e2.elapsed_time(e3) / 1e3, world)
        # exposed gradient all-reduce: forward + backward with DDP's bucketed
        # all-reduce against the same under no_sync() (no collective), CUDA events,
        # max over ranks
        split = None
        if world > 1:
            def fb(sync):
                with contextlib.nullcontext() if sync else model.no_sync():
                    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                        l, _ = model(imgs, generator=gen)
                    l.backward()
                opt.zero_grad(set_to_none=True)
            ms = {}
            for sync in (True, False):
                fb(sync)
                torch.cuda.synchronize()
                barrier(world)
                a = torch.cuda.Event(enable_timing=True)
                c = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(max(1, min(steps, 5))):
                    fb(sync)
                c.record(stream)
                torch.cuda.synchronize()
                ms[sync] = max_over_ranks(a.elapsed_time(c) / max(1, min(steps, 5)), world)
            split = {"fwd_bwd_ms_with_allreduce": ms[True], "fwd_bwd_ms_without_allreduce": ms[False],
                     "allreduce_exposed_ms": ms[True] - ms[False],
                     "collective": "NCCL all-reduce of fp32 gradients in DDP buckets, overlapped with backward"}
    clocks = clk.summary()
    if rank == 0:
        value = world * per_gpu * steps / dev_s
        line = {"metric": "AFF-small MAE pretraining img/s", "value": value, "unit": "img/s", "n_gpus": world,
                "steps": steps, "warmup": warmup, "ms_per_step": dev_s * 1e3 / steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic N(0,1) images, normalised per image; random-init weights",
                "config": {"workload": "AFF-small MAE pretraining step (config 5)", "global_batch": per_gpu * world,
                           "per_gpu_batch": per_gpu, "img_size": cfg.img_size, "patch": cfg.patch_size,
                           "mask_ratio": cfg.mask_ratio, "nbhd": cfg.nbhd_size, "parallelism": f"ddp{world}",
                           "l2": "working set far above L2 (no flush needed)"},
                "img_per_s_per_gpu": value / world, "final_loss": float(loss),
                "e2e": {"value": world * per_gpu * steps / e2e_s, "unit": "img/s",
                        "h2d_bytes_per_step": host.numel() * host.element_size(), "d2h_bytes_per_step": 4,
                        "ms_per_step": e2e_s * 1e3 / steps},
                "roofline": None, "cpu_baseline": None,
                "cpu_baseline_note": "not run for config 5 (a CPU pretraining step is infeasible)",
                "clocks": clocks, "abi_calls_per_step": calls / steps, "ddp_split": split}
        return line
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling runs)")
    ap.add_argument("--batch", type=int, default=CFG["B"], help="images per GPU (default: config 3's 32)")
    ap.add_argument("--workload", default="attn", choices=["attn", "mae"],
                    help="attn: config 3 neighbourhood attention (default); mae: config 5 pretraining")
    ap.add_argument("--mae-batch", type=int, default=16, help="images per GPU for --workload mae")
    ap.add_argument("--no-mae", action="store_true",
                    help="attn workload: skip the config 5 pretraining leg reported as the nested 'mae' object")
    ap.add_argument("--mae-steps", type=int, default=10, help="timed config 5 steps of the nested 'mae' leg")
    ap.add_argument("--mae-warmup", type=int, default=3, help="warm-up config 5 steps of the nested 'mae' leg")
    ap.add_argument("--order", default="curve", choices=["curve", "morton"],
                    help="cluster order of the config 3 tokens: the reference's anchor scan (default) or Z-order")
    args = ap.parse_args()
    CFG["B"] = args.batch
    CFG["order"] = args.order
    world, rank, local = dist_setup()
    if args.workload == "mae":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference's MAE model needs its Triton "
                                  "GPU kernels and pykeops, which are not installed on the GPU box"}), flush=True)
        else:
            line = run_mae(args, world, rank, local)
            if line is not None:
                print(json.dumps(line), flush=True)
    elif args.impl == "reference":
        run_reference(args, world, rank)
    else:
        line = run_gpu(args, world, rank, local)
        if not args.no_mae:
            # config 5 at the same N: data parallel under DDP when WORLD_SIZE > 1
            torch.cuda.empty_cache()
            m = run_mae(args, world, rank, local, steps=args.mae_steps, warmup=args.mae_warmup)
            if line is not None:
                line["mae"] = {"metric": m["metric"], "img_per_s": m["value"],
                               "img_per_s_per_gpu": m["img_per_s_per_gpu"], "unit": "img/s",
                               "ms_per_step": m["ms_per_step"], "steps": m["steps"], "warmup": m["warmup"],
                               "per_gpu_batch": m["config"]["per_gpu_batch"],
                               "parallelism": m["config"]["parallelism"], "e2e_img_per_s": m["e2e"]["value"],
                               "final_loss": m["final_loss"], "clocks": m["clocks"], "ddp_split": m["ddp_split"],
                               "workload": m["config"]["workload"]}
        if line is not None:
            print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
