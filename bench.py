"""Benchmark of the hexel-kernel hot path on B200: fwd+bwd Mpix/s (and frames/s).

Default workload (--config hexels3d_multiview): one training step over 64
views of a 1,000,000-surfel 3D hexel scene at 1920x1080 -- per view:
preprocess -> depth-ordered binning -> front-to-back compositing -> L2 loss
against the view's target -> backward to the surfel parameters, the views'
gradients summed.  One JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config hexels3d_multiview|hexels3d_single|imagegs_large|imagegs_small|
                              hexels2d]

Multi-GPU (torchrun, one rank per GPU): the 64 views are dealt round-robin
over the ranks, surfels are replicated, and the per-surfel gradients are
summed with one NCCL all-reduce per step (strong scaling: the 64-view batch
is fixed).  The Image-GS configurations split the image into horizontal
stripes of 16-pixel tile rows instead.

The line also reports the single 1080p view with depth/normal outputs
("single_view_surface"), the reference's own CUDA kernels compiled from its
sources (oracle/_ref) timed on the same GPU and inputs ("ref_cuda_sm100a"),
and the CPU restatement of the reference's algorithm on a bounded sample
("cpu_baseline").  `--impl reference` times that CPU restatement alone (the
reference ships no CPU implementation), on the host's cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hexel-kernel_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from multiview import ViewPipeline, fit_step_views, view_groups  # noqa: E402
from sharding import GradBuffer, balance_views, stripe_rows, view_split  # noqa: E402

def l2_loss_grad(*args, **kwargs):
    """gsplat.loss.l2_loss_grad, imported on first use (the reference arm never
    loads this build's library)."""
    from gsplat.loss import l2_loss_grad as fn

    return fn(*args, **kwargs)


def mse_loss(pred, target):
    """gsplat.loss.mse_loss (differentiable), imported on first use."""
    from gsplat.loss import mse_loss as fn

    return fn(pred, target)


# DRAM bytes per launch of the roofline kernels, from the committed ncu
# captures of these configurations (read + write)
TRAFFIC_R3D_BWD_1080 = int((277.773312 + 57.324032) * 1e6)  # render3d_bwd, one 1080p view
TRAFFIC_TOPK_FWD_2048 = int((45.213952 + 163.590144) * 1e6)  # topk_fwd, 2048^2 / 100k
TRAFFIC_HEX_FWD_1024 = int((2.483712 + 7.526656) * 1e6)      # hexel_fwd, 1024^2 / 50k

METRIC = "fwd+bwd Mpix/s"
UNIT = "Mpix/s"
L2_FLUSH_BYTES = 256 << 20
FP32_LANES_PER_SM = 128
NUM_SMS = 148


# ---------------------------------------------------------------------------
# environment helpers
# ---------------------------------------------------------------------------
def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "source": "measured",
                "sm_max_mhz": d.get("sm_max_mhz", 1965.0)}
    return {"hbm_gbs": 6650.0, "source": "fallback", "sm_max_mhz": 1965.0}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed
    region: one nvidia-smi process per node (local rank 0) over all of the
    job's GPUs on the node, so that N ranks do not run N pollers beside the
    timed steps; the other ranks sample nothing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank: int):
        n_local = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
        visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [v for v in visible.split(",") if v.strip().isdigit()] if visible else []
        self.gpus = ids[:n_local] if len(ids) >= n_local else [str(i) for i in range(n_local)]
        self.active = local_rank == 0
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        if not self.active:
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={','.join(self.gpus)}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        # nvidia-smi takes a moment to start: wait (bounded) for its first
        # sample so that short timed regions are covered too
        deadline = time.time() + 5.0
        while not self.lines and time.time() < deadline and self.proc.poll() is None:
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.active:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [],
                    "sampled_by": "local rank 0"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "gpus": len(self.gpus)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# Image-GS fit step
# ---------------------------------------------------------------------------
class ImageGSStep:
    """Device-resident fit step, stage by stage (the same kernels as the
    public autograd API), with CUDA events between stages."""

    STAGES = ("project", "scan", "bin", "raster_fwd", "loss", "raster_bwd", "project_bwd",
              "allreduce")

    def __init__(self, w, world: int, rank: int):
        import gsplat
        from gsplat import csrc
        from gsplat.utils import bin_gaussians_fused, compute_cumulative_intersects, \
            count_tiles_in_rows

        self.gs, self.csrc = gsplat, csrc
        self.bin, self.scan, self.count_rows = (bin_gaussians_fused,
                                                compute_cumulative_intersects,
                                                count_tiles_in_rows)
        self.w = w
        self.world, self.rank = world, rank
        self.rows = stripe_rows(w.tile_bounds[1], world, rank)
        self.H, self.W = w.height, w.width
        self.numel = w.height * w.width * 3
        dev = torch.device("cuda")
        self.m, self.s, self.r, self.c = (w.means2d.to(dev), w.scales2d.to(dev),
                                          w.rotation.to(dev), w.colors.to(dev))
        self.target = w.target.to(dev)
        if self.rows is not None:
            self.r0, self.r1 = self.rows[0] * 16, min(self.rows[1] * 16, self.H)
        else:
            self.r0, self.r1 = 0, self.H
        self.events = [torch.cuda.Event(enable_timing=True) for _ in range(len(self.STAGES) + 1)]
        self.stage_ms = {k: 0.0 for k in self.STAGES}
        self.info = {}

    def run(self, timed: bool):
        ev = self.events
        csrc, w = self.csrc, self.w
        ev[0].record()
        xys, radii, conics, nth = csrc.project_gaussians_2d_scale_rot_forward(
            w.num_points, self.m, self.s, self.r, self.H, self.W, w.tile_bounds)
        ev[1].record()
        if self.rows is not None:
            nth = self.count_rows(xys, radii, w.tile_bounds, self.rows)
        n_isect, cum = self.scan(nth)
        ev[2].record()
        ids, bins = self.bin(w.num_points, n_isect, xys, radii, cum, w.tile_bounds, self.rows)
        ev[3].record()
        img, topk = csrc.nd_rasterize_forward_topk_norm(
            w.tile_bounds, (16, 16, 1), (self.W, self.H, 1), ids, bins, xys, conics, self.c)
        ev[4].record()
        if self.rows is None:
            loss, v_img = l2_loss_grad(img, self.target)
        else:
            v_img = torch.zeros_like(img)
            loss, _ = l2_loss_grad(img[self.r0:self.r1], self.target[self.r0:self.r1],
                                   inv_n=1.0 / self.numel, grad=v_img[self.r0:self.r1])
        ev[5].record()
        v_xy, v_conic, v_colors = csrc.nd_rasterize_backward_topk_norm(
            self.H, self.W, 16, 16, ids, bins, xys, conics, self.c, v_img, topk,
            rows=None if self.rows is None else (self.r0, self.r1))
        ev[6].record()
        _, v_mean, v_scale, v_rot = csrc.project_gaussians_2d_scale_rot_backward(
            w.num_points, self.m, self.s, self.r, self.H, self.W, radii, conics, v_xy, v_conic)
        ev[7].record()
        if self.world > 1:
            import torch.distributed as dist

            packed = torch.cat([v_mean.view(-1), v_scale.view(-1), v_rot.view(-1),
                                v_colors.view(-1), loss.view(1)])
            dist.all_reduce(packed)
        ev[8].record()
        self.info = {"num_intersects": n_isect, "bins": bins}
        self._last = (loss, v_mean, v_scale, v_rot, v_colors)
        return loss

    def collect(self):
        for i, k in enumerate(self.STAGES):
            self.stage_ms[k] += self.events[i].elapsed_time(self.events[i + 1])


def run_ours(args, world, rank, local):
    import workloads
    from gsplat._lib import lib

    w = getattr(workloads, args.config)()
    step = ImageGSStep(w, world, rank)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    for _ in range(args.warmup):
        step.run(False)
    torch.cuda.synchronize()
    # per-stage work of this rank's share (for the roofline)
    bins = step.info["bins"].cpu()
    counts = (bins[:, 1] - bins[:, 0]).to(torch.int64)
    tx, ty, _ = w.tile_bounds
    ty_idx = torch.arange(tx * ty) // tx
    tx_idx = torch.arange(tx * ty) % tx
    px_in_tile = ((torch.clamp(w.height - ty_idx * 16, max=16)) *
                  (torch.clamp(w.width - tx_idx * 16, max=16)))
    pairs = int((counts * px_in_tile).sum())
    n_isect = int(step.info["num_intersects"])

    clocks = ClockSampler(local)
    # the sampler waits for its first sample: start it before the barrier,
    # or the other ranks' first timed step waits for this rank
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    launches0 = lib.dll.hx_launch_count()
    total_ms = 0.0
    start_ev = torch.cuda.Event(enable_timing=True)
    end_ev = torch.cuda.Event(enable_timing=True)
    for _ in range(args.steps):
        flush.zero_()
        start_ev.record()
        step.run(True)
        end_ev.record()
        torch.cuda.synchronize()
        step.collect()
        total_ms += start_ev.elapsed_time(end_ev)
    launches = lib.dll.hx_launch_count() - launches0
    barrier(world)
    clk = clocks.stop()
    total_ms = max_over_ranks(total_ms, world)
    ms_per_step = total_ms / args.steps
    stage_ms = {k: max_over_ranks(v / args.steps, world) for k, v in step.stage_ms.items()}

    # end-to-end: public autograd API from pinned host buffers, loss read back
    e2e = None if args.skip_extras else run_e2e(w, args, world, rank)

    if rank != 0:
        return None
    peaks = measured_peaks()
    mpix = w.height * w.width / 1e6
    value = mpix / (ms_per_step / 1e3)
    sm_mhz = clk.get("sm_mhz") or peaks["sm_max_mhz"]
    fp32_peak_tflops = NUM_SMS * FP32_LANES_PER_SM * 2 * peaks["sm_max_mhz"] * 1e6 / 1e12
    fwd_ms = stage_ms["raster_fwd"]
    fwd_flops = pairs * 14.0
    stages = {k: round(v, 4) for k, v in stage_ms.items()}
    sort_bits = max(1, (tx * ty - 1).bit_length())
    sort_bytes = n_isect * (8 + 16 * ((sort_bits + 7) // 8))
    roofline = {
        "kernel": "topk_fwd_kernel (nd_rasterize_forward_topk_norm)",
        "bound": "fp32",
        "achieved": round(fwd_flops / (fwd_ms / 1e3) / 1e12, 3),
        "peak": round(fp32_peak_tflops, 2),
        "unit": "TFLOP/s",
        "frac": round(fwd_flops / (fwd_ms / 1e3) / 1e12 / fp32_peak_tflops, 4),
        "traffic": TRAFFIC_TOPK_FWD_2048 if args.config == "imagegs_large" else None,
        "traffic_source": ("dram__bytes_read.sum + dram__bytes_write.sum per launch, one ncu "
                           "capture of this configuration (profiles/imagegs_topk_2048_n100k.md)"
                           if args.config == "imagegs_large" else None),
        "peak_source": "nominal FP32 FMA rate, 148 SMs x 128 lanes x 2 x max SM clock "
                       "(no measured FP32 peak in MEASURED_PEAKS.json)",
        "work": f"{pairs} (pixel, candidate) pairs x 14 FLOP",
        "bin_sort_hbm": {
            "achieved_gbs": round(sort_bytes / (stage_ms["bin"] / 1e3) / 1e9, 1),
            "peak_gbs": peaks["hbm_gbs"], "peak_source": peaks["source"],
            "frac": round(sort_bytes / (stage_ms["bin"] / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
            "bytes": sort_bytes,
        },
    }
    line = {
        "metric": METRIC,
        "value": round(value * 1.0, 3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "frames_per_s": round(1e3 / ms_per_step, 3),
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded; the reference publishes no dataset)",
        "config": {
            "workload": w.name,
            "height": w.height, "width": w.width, "num_gaussians": w.num_points,
            "top_k": 10, "tile": 16, "channels": 3,
            "num_intersects": n_isect,
            "parallelism": f"tile-row stripes x{world}" if world > 1 else "single GPU",
            "l2": "flushed between timed steps (256 MB write)",
        },
        "stages_ms": stages,
        "roofline": roofline,
        "e2e": e2e,
        "gpu_launches": int(launches),
        "clocks": clk,
    }
    if world == 1 and not args.skip_extras:
        line["cpu_baseline"] = cpu_baseline(args, w)
        ref = ref_cuda_timing(args, w)
        if ref is not None:
            line["ref_cuda_sm100a"] = ref
    return line


def run_e2e(w, args, world, rank):
    """Same step through the public API (autograd), inputs copied each step
    from pinned host memory and the loss read back."""
    import gsplat

    rows = stripe_rows(w.tile_bounds[1], world, rank)
    host = [t.pin_memory() for t in (w.means2d, w.scales2d, w.rotation, w.colors, w.target)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    if rows is not None:
        r0, r1 = rows[0] * 16, min(rows[1] * 16, w.height)
    else:
        r0, r1 = 0, w.height
    numel = w.height * w.width * 3

    def one():
        m, s, r, c, tgt = (t.to("cuda", non_blocking=True) for t in host)
        for p in (m, s, r, c):
            p.requires_grad_(True)
        xys, radii, conics, nth = gsplat.project_gaussians_2d_scale_rot(m, s, r, w.height, w.width,
                                                                        w.tile_bounds)
        img = gsplat.rasterize_gaussians_sum(xys, radii, conics, nth, c, w.height, w.width,
                                             topk_norm=True, tile_rows=rows)
        d = img[r0:r1] - tgt[r0:r1]
        loss = (d * d).sum() / numel
        loss.backward()
        if world > 1:
            import torch.distributed as dist

            packed = torch.cat([m.grad.view(-1), s.grad.view(-1), r.grad.view(-1),
                                c.grad.view(-1), loss.detach().view(1)])
            dist.all_reduce(packed)
            loss = packed[-1]
        return float(loss.item())

    for _ in range(max(1, args.warmup)):
        one()
    torch.cuda.synchronize()
    barrier(world)
    st = torch.cuda.Event(enable_timing=True)
    en = torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(args.steps):
        one()
    en.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(st.elapsed_time(en) / args.steps, world)
    return {"value": round(w.height * w.width / 1e6 / (ms / 1e3), 3), "unit": UNIT,
            "ms_per_step": round(ms, 4), "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": 4,
            "path": "gsplat.project_gaussians_2d_scale_rot + gsplat.rasterize_gaussians_sum"
                    "(topk_norm=True) + L2 loss + backward"}


# ---------------------------------------------------------------------------
# 2D image hexels (1024x1024, 50,000 hexagons, top-10 normalised compositing)
# ---------------------------------------------------------------------------
# Algorithmic work (FMA = 2): forward 40 FLOP per (pixel, candidate) pair,
# backward 110 FLOP per (pixel, stored id).
HEX2D_FWD_FLOP, HEX2D_BWD_FLOP = 40.0, 110.0


def hexels2d_binning(w, xys, radii):
    """The harness's binning of the hexagons (caller-chosen radii): tile
    counts, prefix sum, sorted ids and tile bins."""
    from gsplat.utils import bin_gaussians_fused, compute_cumulative_intersects, \
        count_tiles_in_rows

    tb = w.tile_bounds
    nth = count_tiles_in_rows(xys, radii, tb, (0, tb[1]))
    ni, cum = compute_cumulative_intersects(nth)
    ids, bins = bin_gaussians_fused(w.num_points, ni, xys, radii, cum, tb)
    return nth, ni, ids, bins


def run_ours_hex2d(args, world, rank, local):
    """c3: one fit step -- binning, top-10 hexagon compositing, L2 loss,
    backward to the hexagons' parameters.  The image is small; every rank
    runs its own replica (no collective), value = ranks x per-GPU rate."""
    import workloads
    from gsplat import csrc
    from gsplat._lib import lib

    w = workloads.hexels2d()
    dev = torch.device("cuda")
    xys, scales, rot, col, radii = (t.to(dev) for t in (w.xys, w.scales, w.rotation, w.colors,
                                                       w.radii))
    target = w.target.to(dev)
    e = torch.empty(0, device=dev)
    H, W, tb = w.height, w.width, w.tile_bounds
    numel = H * W * 3
    zero_hw = torch.zeros((H, W), device=dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    stage_names = ("bin", "raster_fwd", "loss", "raster_bwd")
    stage_ms = {k: 0.0 for k in stage_names}
    info = {}

    def step(timed):
        ev[0].record()
        nth, ni, ids, bins = hexels2d_binning(w, xys, radii)
        ev[1].record()
        img, topk, ws, ent = csrc.nd_rasterize_forward_topk_norm_hexels(
            tb, (16, 16, 1), (W, H, 1), ids, bins, xys, scales, rot, col, w.aa_kernel_size,
            w.softness, e, e)
        ev[2].record()
        loss, v_out = l2_loss_grad(img, target)
        ev[3].record()
        grads = csrc.nd_rasterize_backward_topk_norm_hexels(
            H, W, 16, 16, ids, bins, xys, scales, rot, col, v_out, zero_hw, zero_hw, topk,
            w.aa_kernel_size, w.softness, e, e)
        ev[4].record()
        info.update(ni=ni, bins=bins, topk=topk)
        return loss, grads

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize()
    counts = (info["bins"][:, 1] - info["bins"][:, 0]).to(torch.int64).cpu()
    tx, ty, _ = tb
    t_idx = torch.arange(tx * ty)
    px_in_tile = (torch.clamp(H - (t_idx // tx) * 16, max=16) *
                  torch.clamp(W - (t_idx % tx) * 16, max=16))
    pairs = int((counts * px_in_tile).sum())
    stored = int((info["topk"] >= 0).sum())
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    clocks = ClockSampler(local)
    # the sampler waits for its first sample: start it before the barrier,
    # or the other ranks' first timed step waits for this rank
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    launches0 = lib.dll.hx_launch_count()
    total = 0.0
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(args.steps):
        flush.zero_()
        st.record()
        step(True)
        en.record()
        torch.cuda.synchronize()
        total += st.elapsed_time(en)
        for i, k in enumerate(stage_names):
            stage_ms[k] += ev[i].elapsed_time(ev[i + 1])
    launches = lib.dll.hx_launch_count() - launches0
    barrier(world)
    clk = clocks.stop()
    ms = max_over_ranks(total / args.steps, world)
    stages = {k: round(max_over_ranks(v / args.steps, world), 4) for k, v in stage_ms.items()}
    if rank != 0:
        return None
    peaks = measured_peaks()
    fp32_peak = NUM_SMS * FP32_LANES_PER_SM * 2 * peaks["sm_max_mhz"] * 1e6 / 1e12
    bwd = stored * HEX2D_BWD_FLOP / (stages["raster_bwd"] / 1e3) / 1e12
    fwd = pairs * HEX2D_FWD_FLOP / (stages["raster_fwd"] / 1e3) / 1e12
    line = {
        "metric": METRIC, "value": round(world * H * W / 1e6 / (ms / 1e3), 3), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "frames_per_s": round(world * 1e3 / ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; the reference publishes no dataset)",
        "config": {"workload": w.name, "height": H, "width": W, "num_hexagons": w.num_points,
                   "top_k": 10, "tile": 16, "softness": w.softness,
                   "num_intersects": int(info["ni"]),
                   "parallelism": f"{world} independent replicas" if world > 1 else "single GPU",
                   "l2": "flushed between timed steps (256 MB write)"},
        "stages_ms": stages,
        "roofline": {"kernel": "hexel_fwd_kernel / hexel_bwd_kernel", "bound": "fp32",
                     "achieved": round(fwd, 3), "peak": round(fp32_peak, 2), "unit": "TFLOP/s",
                     "frac": round(fwd / fp32_peak, 4), "traffic": TRAFFIC_HEX_FWD_1024,
                     "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum per "
                                       "launch, one ncu capture of this configuration "
                                       "(profiles/hexels2d_1024_n50k.md)",
                     "work": f"forward {pairs} (pixel, candidate) pairs x {HEX2D_FWD_FLOP:.0f} "
                             f"FLOP; backward {stored} stored ids x {HEX2D_BWD_FLOP:.0f} FLOP",
                     "backward": {"achieved": round(bwd, 3), "frac": round(bwd / fp32_peak, 4)}},
        "gpu_launches": int(launches), "clocks": clk, "e2e": None,
    }
    if world == 1 and not args.skip_extras:
        threads = len(os.sched_getaffinity(0))
        torch.set_num_threads(threads)
        crop = args.cpu_crop_tiles
        secs, mpix = cpu_sample_run_hex2d(w, crop)
        line["cpu_baseline"] = {
            "value": round(mpix / secs, 5), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"one fwd+bwd over a {crop}x{crop}-tile ({mpix:.4f} Mpix) centre crop of "
                      f"{w.name}: binning of the crop's rows, top-10 hexagon compositing and "
                      f"backward; {secs:.2f} s", "seconds": round(secs, 3)}
        ref = ref_cuda_timing_hex2d(args, w)
        if ref is not None:
            line["ref_cuda_sm100a"] = ref
    return line


def cpu_sample_run_hex2d(w, crop_tiles: int):
    """One fwd+bwd of the oracle (2D hexels) over a crop_tiles x crop_tiles
    tile crop at the image centre; returns (seconds, megapixels)."""
    import numpy as np

    from oracle import hexels2d as oh
    from oracle import raster2d as o

    tx, ty, _ = w.tile_bounds
    x0 = max(0, tx // 2 - crop_tiles // 2)
    y0 = max(0, ty // 2 - crop_tiles // 2)
    xs = np.arange(x0, min(tx, x0 + crop_tiles))
    ys = np.arange(y0, min(ty, y0 + crop_tiles))
    tiles = (ys[:, None] * tx + xs[None, :]).reshape(-1)
    t0 = time.perf_counter()
    keys, ids = o.map_intersects(w.xys.numpy(), w.radii.numpy(), None, w.tile_bounds,
                                 tile_rows=(int(ys[0]), int(ys[-1]) + 1))
    _, ids_sorted, bins = o.sort_and_bin(keys, ids.astype(np.int32), tx * ty)
    p = oh.HexParams(xys=w.xys, colors=w.colors, softness=w.softness, aa=w.aa_kernel_size)
    p.scales, p.rotation = w.scales, w.rotation
    img, topk, _, _ = oh.forward(p, torch.from_numpy(ids_sorted), bins, w.height, w.width,
                                 tile_ids=tiles)
    rows = slice(int(ys[0]) * 16, min((int(ys[-1]) + 1) * 16, w.height))
    cols = slice(int(xs[0]) * 16, min((int(xs[-1]) + 1) * 16, w.width))
    v_img = torch.zeros_like(img)
    v_img[rows, cols] = 2.0 * (img[rows, cols] - w.target[rows, cols]) / img.numel()
    topk_crop = torch.full_like(topk, -1)
    topk_crop[rows, cols] = topk[rows, cols]
    zero = torch.zeros((w.height, w.width))
    oh.backward(p, v_img, zero, zero, topk_crop, w.height, w.width)
    secs = time.perf_counter() - t0
    return secs, (rows.stop - rows.start) * (cols.stop - cols.start) / 1e6


def ref_cuda_timing_hex2d(args, w):
    """The reference's 2D hexel kernels (compiled from its sources) on the same
    inputs, with its own binning sequence (map_gaussian_to_intersects,
    torch.sort, get_tile_bin_edges; gsplat/utils.py:118-162) on the same tile
    counts."""
    path = os.path.join(ROOT, "oracle", "_ref", "_ref_gsplat_csrc.so")
    if not os.path.exists(path):
        return None
    import importlib.util

    spec = importlib.util.spec_from_file_location("_ref_gsplat_csrc", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    from gsplat.utils import count_tiles_in_rows

    dev = torch.device("cuda")
    xys, scales, rot, col, radii = (t.to(dev) for t in (w.xys, w.scales, w.rotation, w.colors,
                                                       w.radii))
    target = w.target.to(dev)
    e = torch.empty(0, device=dev)
    H, W, tb, n = w.height, w.width, w.tile_bounds, w.num_points
    numel = H * W * 3
    zero_hw = torch.zeros((H, W), device=dev)
    nth = count_tiles_in_rows(xys, radii, tb, (0, tb[1]))

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    stage_names = ("bin", "raster_fwd", "loss", "raster_bwd")
    stage_ms = {k: 0.0 for k in stage_names}

    def step():
        ev[0].record()
        cum = torch.cumsum(nth, dim=0, dtype=torch.int32)
        ni = int(cum[-1].item())
        isect, gids = ref.map_gaussian_to_intersects(n, ni, xys, radii, cum, tb)
        isect_s, order = torch.sort(isect)
        gids_s = torch.gather(gids, 0, order)
        bins = ref.get_tile_bin_edges(ni, tb[0] * tb[1], isect_s)
        ev[1].record()
        img, topk, ws, ent = ref.nd_rasterize_forward_topk_norm_hexels(
            tb, (16, 16, 1), (W, H, 1), gids_s, bins, xys, scales, rot, col, w.aa_kernel_size,
            w.softness, e, e)
        ev[2].record()
        d = img - target
        loss = (d * d).sum() / numel
        v_out = d * (2.0 / numel)
        ev[3].record()
        ref.nd_rasterize_backward_topk_norm_hexels(H, W, 16, 16, gids_s, bins, xys, scales, rot,
                                                   col, v_out, zero_hw, zero_hw, topk,
                                                   w.aa_kernel_size, w.softness, e, e)
        ev[4].record()
        return loss

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    total = 0.0
    for _ in range(args.steps):
        flush.zero_()
        st.record()
        step()
        en.record()
        torch.cuda.synchronize()
        total += st.elapsed_time(en)
        for i, k in enumerate(stage_names):
            stage_ms[k] += ev[i].elapsed_time(ev[i + 1])
    ms = total / args.steps
    return {"value": round(H * W / 1e6 / (ms / 1e3), 3), "unit": UNIT,
            "ms_per_step": round(ms, 4), "steps": args.steps,
            "stages_ms": {k: round(v / args.steps, 4) for k, v in stage_ms.items()},
            "what": "reference CUDA kernels compiled from its sources for sm_100a "
                    "(-O3 --use_fast_math), its own binning sequence, same inputs and loss"}


# ---------------------------------------------------------------------------
# 3D hexel surfels
# ---------------------------------------------------------------------------
# c5 (multi-view, default): 64 views of the 1M-surfel scene, the RGB-only
# cached training path, loss per view mean((rgb - target)^2), views dealt
# round-robin over the ranks, per-surfel gradients all-reduced once per step.
# c4 (single view): the same scene from view 0 with depth/normal outputs,
# loss mean((rgb - target)^2) + 0.1 mean(depth^2) + 0.1 mean(normal^2).
LAMBDA_DEPTH2, LAMBDA_NORMAL2 = 0.1, 0.1
# Algorithmic work per unit (FMA = 2 FLOP): forward compositing per
# evaluated (pixel, surfel) pair, i.e. list entries visited before the
# pixel terminates (sum of the per-pixel last index); backward compositing
# per contributing (blended) pair.
FWD_FLOP_PER_PAIR = 90.0
BWD_FLOP_PER_PAIR = 260.0


def make_targets(w, views, device):
    """Seeded U[0,1) target image per view (3,H,W)."""
    cam = w.cameras[0]
    out = []
    for v in views:
        g = torch.Generator().manual_seed(20261201 + 7919 * (v + 1))
        out.append(torch.rand((3, cam.height, cam.width), generator=g).to(device))
    return out


class Hexels3DStep:
    """Device-resident fit step over this rank's views through the kernels of
    the public autograd API (cuda_hexels3d._C forward with the backward's
    state saved, then the cached backward), CUDA events between stages."""

    STAGES = ("preprocess", "scan", "bin", "render_fwd", "loss", "render_bwd", "geometry_bwd",
              "accumulate", "allreduce")

    def __init__(self, w, world: int, rank: int, surface: bool, group: int = 1):
        from gsplat.cuda_hexels3d import _C

        self.C = _C
        self.w = w
        self.surface = surface
        self.world, self.rank = world, rank
        self.views = view_split(len(w.cameras), world, rank)
        dev = torch.device("cuda")
        self.dev = dev
        self.params = [t.to(dev) for t in (w.means3d, w.scales, w.rotations, w.colors,
                                           w.color_grads, w.view_grads, w.opacities)]
        self.bg = w.background.to(dev)
        self.cams = [w.cameras[v].to(dev) for v in self.views]
        self.targets = make_targets(w, self.views, dev)
        cam = w.cameras[0]
        self.H, self.W = cam.height, cam.width
        self.empty = torch.empty(0, device=dev)
        self.zero_hw = torch.zeros((self.H, self.W), device=dev)
        self.numel = 3 * self.H * self.W
        # per-step gradient sums, zeroed once per step and all-reduced in place
        self.grads = GradBuffer([p.shape for p in self.params], dev)
        self.acc = self.grads.views
        # the RGB step's views are pipelined over two streams (multiview.py)
        self.pipeline = None if surface else ViewPipeline(self.params, streams=2)
        # the timed step bins the rank's views in groups (view_groups)
        self.group_max = group
        self.group = view_groups(len(self.views), group) if group > 1 else 1
        self.marks: list = []
        self.stage_ms = {k: 0.0 for k in self.STAGES}
        self.info: dict = {}

    def _mark(self, name):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.marks.append((name, ev))

    def _view(self, cam, target, keep_info):
        C, e = self.C, self.empty
        m3, sc, rot, col, cg, vg, op = self.params
        o = C._forward_core(m3, sc, rot, col, cg, e, vg, e, e, op, e, cam.viewmatrix,
                            cam.projmatrix, cam.campos, self.bg, self.W, self.H, cam.tan_fovx,
                            cam.tan_fovy, self.w.softness, 1.0, 1, 1, True, False, False, False,
                            return_surface=self.surface, save=True, save_surface=self.surface,
                            count_contrib=keep_info)
        # the view's mean-squared colour error is added into the step's loss slot
        _, g_color = l2_loss_grad(o["out_color"], target, loss=self.grads.loss)
        gd = ga = gn = e
        loss = None
        if self.surface:
            hw = float(self.H * self.W)
            depth, normals = o["surf_depth"], o["surf_maps"][:3]
            loss = LAMBDA_DEPTH2 * (depth * depth).sum() / hw + \
                LAMBDA_NORMAL2 * (normals * normals).sum() / (3 * hw)
            gd = depth * (2 * LAMBDA_DEPTH2 / hw)
            ga = self.zero_hw
            gn = torch.cat([normals * (2 * LAMBDA_NORMAL2 / (3 * hw)), self.zero_hw[None]])
        self._mark("loss")
        names = ("means3d", "scales", "rotations", "colors", "color_grads", "view_grads",
                 "opacities")
        grads = C._backward_core(m3, e, sc, rot, col, cg, e, vg, e, e, op, e, cam.viewmatrix,
                                 cam.projmatrix, cam.campos, self.bg, g_color, e, gd, ga, gn,
                                 self.W, self.H, cam.tan_fovx, cam.tan_fovy, self.w.softness,
                                 1.0, 1, 1, True, -1, False, False, False, o["saved"],
                                 surf_state=o["surf_state"],
                                 surf_normals=o["normals"] if self.surface else None,
                                 accumulate_into=dict(zip(names, self.acc)),
                                 blend_mask=o["blend_mask"], records=o["records"])
        if keep_info:
            saved = o["saved"]
            self.info.setdefault("num_rendered", []).append(o["num_rendered"])
            self.info.setdefault("evaluated_pairs", []).append(
                int(saved[10].to(torch.int64).sum().item()))
            counts = o["contrib_count"].to(torch.int64).sum((1, 2)).tolist()
            self.info.setdefault("blended_pairs", []).append(int(counts[0]))
            self.info.setdefault("culled_evaluated_pairs", []).append(int(counts[1]))
        return loss, grads

    def run_pipelined(self):
        """The step as a user runs it: views pipelined over two streams
        (multiview.fit_step_views), gradients all-reduced; no per-stage
        events."""
        if self.pipeline is None:
            self.run()
            return self.grads.loss
        self.grads.zero_()
        fit_step_views(self.params, self.cams, self.targets, self.bg, self.w.softness,
                       self.acc, self.grads.loss, self.pipeline, group=self.group)
        self.grads.all_reduce_(self.world)
        return self.grads.loss

    def run(self, keep_info: bool = False):
        """The step with CUDA events between stages, views in order on one
        stream (stage shares, per-view costs, work counts)."""
        if keep_info:
            self.info = {}
        self.marks = []
        self.C.stage_hook = self._mark
        try:
            self._mark("start")
            self.grads.zero_()
            for cam, tgt in zip(self.cams, self.targets):
                # the backward adds this view's gradients into self.acc
                loss, _ = self._view(cam, tgt, keep_info)
                if loss is not None:  # surface terms of the loss
                    self.grads.loss.add_(loss)
                self._mark("accumulate")
            self.grads.all_reduce_(self.world)
            total = self.grads.loss
            self._mark("allreduce")
        finally:
            self.C.stage_hook = None
        return total

    def collect(self):
        for (_, a), (name, b) in zip(self.marks[:-1], self.marks[1:]):
            self.stage_ms[name] += a.elapsed_time(b)

    def view_ms(self):
        """Device time of each of this rank's views in the last run (from the
        previous view's end, or the step's start, to the view's end)."""
        out, start = [], None
        for name, ev in self.marks:
            if name == "start":
                start = ev
            elif name == "accumulate":
                out.append(start.elapsed_time(ev))
                start = ev
        return out

    def rebalance(self):
        """Re-deal the views over the ranks by the device time each took in
        the last run (one all-reduce of a per-view vector; every rank computes
        the same split), then load the cameras and targets of the new set."""
        if self.world == 1:
            return
        import torch.distributed as dist

        nviews = len(self.w.cameras)
        costs = torch.zeros(nviews, dtype=torch.float64, device=self.dev)
        for v, ms in zip(self.views, self.view_ms()):
            costs[v] = ms
        dist.all_reduce(costs)
        views = balance_views(costs.tolist(), self.world)[self.rank]
        if views == self.views:
            return
        have = dict(zip(self.views, self.targets))
        new = [v for v in views if v not in have]
        have.update(zip(new, make_targets(self.w, new, self.dev)))
        self.views = views
        self.cams = [self.w.cameras[v].to(self.dev) for v in views]
        self.targets = [have[v] for v in views]
        if self.group_max > 1:
            self.group = view_groups(len(views), self.group_max)


def time_step_3d(step, steps, warmup, world):
    """Warm-up (the first one collects the work counts), then `steps` timed
    steps between barriers, L2 flushed before each; returns (ms per step,
    stage ms per step, this library's kernel launches in the timed steps),
    times max over ranks."""
    from gsplat._lib import lib

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    for i in range(warmup):
        step.run(keep_info=(i == warmup - 1))
        if i == 1 and world > 1:
            # deal the views by the device time each took in this run (the
            # first run pays one-time set-up and is not representative)
            torch.cuda.synchronize()
            step.rebalance()
    step.run_pipelined()  # the timed form's own first run (stream pools)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    total_ms = 0.0
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = lib.dll.hx_launch_count()
    # an NVTX range over the timed steps (ncu --nvtx --nvtx-include timed_steps/)
    torch.cuda.nvtx.range_push("timed_steps")
    for _ in range(steps):
        flush.zero_()
        st.record()
        step.run_pipelined()
        en.record()
        torch.cuda.synchronize()
        total_ms += st.elapsed_time(en)
    torch.cuda.nvtx.range_pop()
    launches = lib.dll.hx_launch_count() - launches0
    barrier(world)
    ms = max_over_ranks(total_ms / steps, world)
    # stage shares from one more step with events between stages (one stream)
    step.stage_ms = {k: 0.0 for k in step.STAGES}
    flush.zero_()
    step.run()
    torch.cuda.synchronize()
    step.collect()
    stage = {k: max_over_ranks(v, world) for k, v in step.stage_ms.items()}
    return ms, stage, launches


def roofline_3d(step, stage_ms):
    peaks = measured_peaks()
    fp32_peak = NUM_SMS * FP32_LANES_PER_SM * 2 * peaks["sm_max_mhz"] * 1e6 / 1e12
    nv = len(step.views)
    blended = sum(step.info.get("blended_pairs", [0]))
    evaluated = sum(step.info.get("evaluated_pairs", [0]))
    culled = sum(step.info.get("culled_evaluated_pairs", [0]))
    bwd_ms, fwd_ms = stage_ms["render_bwd"], stage_ms["render_fwd"]
    bwd = blended * BWD_FLOP_PER_PAIR / (bwd_ms / 1e3) / 1e12 if bwd_ms > 0 else 0.0
    fwd = evaluated * FWD_FLOP_PER_PAIR / (fwd_ms / 1e3) / 1e12 if fwd_ms > 0 else 0.0
    fwd_c = culled * FWD_FLOP_PER_PAIR / (fwd_ms / 1e3) / 1e12 if fwd_ms > 0 else 0.0
    return {
        "kernel": "render3d_bwd_kernel (rasterize_hexels3d backward compositing)",
        "bound": "fp32",
        "achieved": round(bwd, 3),
        "peak": round(fp32_peak, 2),
        "unit": "TFLOP/s",
        "frac": round(bwd / fp32_peak, 4),
        "traffic": TRAFFIC_R3D_BWD_1080 if nv and step.H == 1080 and not step.surface else None,
        "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum per launch (one view), "
                          "one ncu capture of this configuration "
                          "(profiles/render3d_bwd_1080p_1M.md)",
        "peak_source": "nominal FP32 FMA rate, 148 SMs x 128 lanes x 2 x max SM clock "
                       "(MEASURED_PEAKS.json has no FP32 figure)",
        "work": f"{blended} blended (pixel, surfel) pairs over {nv} views x "
                f"{BWD_FLOP_PER_PAIR:.0f} FLOP per step on rank 0",
        "forward": {"kernel": "render3d_fwd_kernel", "achieved": round(fwd, 3),
                    "frac": round(fwd / fp32_peak, 4),
                    "work": f"{evaluated} pairs visited before each pixel terminates (sum of "
                            f"the last indices) x {FWD_FLOP_PER_PAIR:.0f} FLOP",
                    "after_box_cull": {
                        "achieved": round(fwd_c, 3), "frac": round(fwd_c / fp32_peak, 4),
                        "work": f"{culled} pairs evaluated after the warps' pixel-box cull x "
                                f"{FWD_FLOP_PER_PAIR:.0f} FLOP (the kernel's actual work)"}},
    }


def run_ours_3d(args, world, rank, local):
    w = workload_3d(args.config, args.views)
    surface = args.config == "hexels3d_single"
    step = Hexels3DStep(w, world, rank, surface, args.group)
    clocks = ClockSampler(local)
    clocks.start()
    ms_per_step, stage_ms, launches = time_step_3d(step, args.steps, args.warmup, world)
    clk = clocks.stop()
    nviews = len(w.cameras)
    rendered_rank = sum(step.info.get("num_rendered", [0]))
    e2e = e2e_autograd = None
    if not args.skip_extras:
        e2e_autograd = run_e2e_3d(w, args, world, rank, surface, step.views)
        e2e = e2e_autograd if surface else run_e2e_3d_pipelined(w, args, world, rank,
                                                                step.views, step.group)
    secondary = None
    if world == 1 and not args.skip_extras and not surface:
        secondary = single_view_comparison(args)
    if rank != 0:
        return None
    value = nviews * step.H * step.W / 1e6 / (ms_per_step / 1e3)
    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "frames_per_s": round(nviews / (ms_per_step / 1e3), 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded; the reference publishes no dataset)",
        "config": {
            "workload": w.name,
            "views": nviews, "height": step.H, "width": step.W, "num_surfels": w.num_points,
            "outputs": "rgb + depth + alpha + normal + distortion" if surface else "rgb",
            "color_model": "linear", "view_model": "linear",
            "intersections_per_view": round(rendered_rank / max(1, len(step.views))),
            "view_group": step.group,
            "parallelism": (f"views dealt over {world} GPUs by the device time each took in "
                            "the second warm-up step (longest first to the least-loaded rank), "
                            "surfels replicated, gradients NCCL all-reduced")
                           if world > 1 else "single GPU",
            "l2": "flushed between timed steps (256 MB write)",
        },
        "stages_ms": {k: round(v, 4) for k, v in stage_ms.items()},
        "stages_note": ("one step with CUDA events between stages, views one at a time in "
                        "order on one stream; the timed steps bin the views in groups and "
                        "pipeline the groups over two streams"
                        if step.pipeline is not None else
                        "CUDA events between stages of the timed steps"),
        "roofline": roofline_3d(step, stage_ms),
        "e2e": e2e,
        "gpu_launches": int(launches),
        "clocks": clk,
    }
    if e2e_autograd is not None and e2e_autograd is not e2e:
        line["e2e_autograd_per_view"] = e2e_autograd
    if secondary is not None:
        line["single_view_surface"] = secondary
    if world == 1 and not args.skip_extras and not surface:
        line["configs_2d"] = other_configs_2d(args)
    if world == 1 and not args.skip_extras:
        cpu = cpu_baseline_3d(args, w)
        if cpu is not None:
            line["cpu_baseline"] = cpu
        ref = ref_cuda_timing_3d(args, w, surface)
        if ref is not None:
            line["ref_cuda_sm100a"] = ref
    return line


def other_configs_2d(args):
    """The 2D configurations measured in the same run, device-timed, each
    beside the reference's CUDA kernels on the same inputs: Image-GS
    256x256 / 4,096 and 2048x2048 / 100,000 Gaussians (top-10), 2D hexels
    1024x1024 / 50,000 (top-10).  Each: device-resident fit step
    (projection or binning, compositing, L2 loss, backward), L2 flushed
    between steps."""
    import workloads

    out = {}
    for cfg in ("imagegs_small", "imagegs_large", "hexels2d"):
        sub = argparse.Namespace(**vars(args))
        sub.config, sub.skip_extras = cfg, True
        sub.steps, sub.warmup = max(args.steps, 20), max(args.warmup, 3)
        line = (run_ours_hex2d if cfg == "hexels2d" else run_ours)(sub, 1, 0, 0)
        w = workloads.hexels2d() if cfg == "hexels2d" else getattr(workloads, cfg)()
        ref = ref_cuda_timing_hex2d(sub, w) if cfg == "hexels2d" else ref_cuda_timing(sub, w)
        rl = line.get("roofline", {})
        entry = {"workload": line["config"]["workload"], "value": line["value"],
                 "unit": line["unit"], "ms_per_step": line["ms_per_step"],
                 "steps": line["steps"], "stages_ms": line.get("stages_ms"),
                 "roofline": {k: rl.get(k) for k in ("kernel", "achieved", "peak", "unit",
                                                     "frac")},
                 "clocks": line.get("clocks")}
        if ref is not None:
            entry["ref_cuda_sm100a"] = {"value": ref["value"], "ms_per_step": ref["ms_per_step"]}
            entry["speedup_vs_ref_cuda"] = round(ref["ms_per_step"] / line["ms_per_step"], 3)
        out[cfg] = entry
    return out


def single_view_comparison(args):
    """The 1080p / 1M-surfel single view with depth/normal outputs, ours and
    the reference's CUDA kernels on the same inputs (device-resident, L2
    flushed between steps)."""
    w = workload_3d("hexels3d_single")
    step = Hexels3DStep(w, 1, 0, True)
    ms, stage, _ = time_step_3d(step, max(args.steps, 10), max(args.warmup, 3), 1)
    H, W = step.H, step.W
    out = {"workload": w.name, "ms_per_step": round(ms, 4),
           "value": round(H * W / 1e6 / (ms / 1e3), 3), "unit": UNIT,
           "stages_ms": {k: round(v, 4) for k, v in stage.items()},
           "roofline": roofline_3d(step, stage)}
    del step
    ref = ref_cuda_timing_3d(args, w, True, steps=max(args.steps, 10))
    if ref is not None:
        out["ref_cuda_sm100a"] = ref
    return out


def run_e2e_3d_pipelined(w, args, world, rank, views, group=1):
    """The RGB multi-view step end to end through the repo's multi-view fit
    API (multiview.fit_step_views: this rank's views pipelined over two
    streams, gradients added into one flat buffer, NCCL all-reduce in place)
    with every step's inputs -- the surfel parameters and this rank's target
    images -- copied from pinned host memory and the loss read back.  Inputs
    are double-buffered as a training loop's loader would: while step s
    runs, a copy stream uploads step s + 1's inputs into the other buffer.
    Returns the figures and a per-step breakdown (copy-stream time, compute,
    all-reduce + loss read-back)."""
    dev = torch.device("cuda")
    host_params = [t.pin_memory() for t in (w.means3d, w.scales, w.rotations, w.colors,
                                           w.color_grads, w.view_grads, w.opacities)]
    host_targets = [t.pin_memory() for t in make_targets(w, views, "cpu")]
    h2d = sum(t.numel() * t.element_size() for t in host_params + host_targets)
    cams = [w.cameras[v].to(dev) for v in views]
    bg = w.background.to(dev)
    bufs = [([torch.empty(t.shape, device=dev) for t in host_params],
             [torch.empty(t.shape, device=dev) for t in host_targets]) for _ in range(2)]
    grads = GradBuffer([t.shape for t in host_params], dev)
    pipe = ViewPipeline(bufs[0][0], streams=2)
    main = torch.cuda.current_stream()
    copy = torch.cuda.Stream()
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    ev = {k: torch.cuda.Event(enable_timing=True)
          for k in ("c0", "c1", "s0", "s1", "s2")}
    parts = {"h2d_copy_stream_ms": 0.0, "compute_ms": 0.0, "allreduce_readback_ms": 0.0}

    def upload(b, timed):
        with torch.cuda.stream(copy):
            copy.wait_event(free[b])
            if timed:
                ev["c0"].record(copy)
            for d, h in zip(bufs[b][0] + bufs[b][1], host_params + host_targets):
                d.copy_(h, non_blocking=True)
            if timed:
                ev["c1"].record(copy)
            ready[b].record(copy)

    def step(i, timed):
        b = i % 2
        upload(1 - b, timed)  # the next step's inputs, overlapped with this step
        main.wait_event(ready[b])
        if timed:
            ev["s0"].record(main)
        grads.zero_()
        fit_step_views(bufs[b][0], cams, bufs[b][1], bg, w.softness, grads.views, grads.loss,
                       pipe, group=group)
        free[b].record(main)
        if timed:
            ev["s1"].record(main)
        grads.all_reduce_(world)
        loss = float(grads.loss.item())
        if timed:
            ev["s2"].record(main)
            torch.cuda.synchronize()
            parts["h2d_copy_stream_ms"] += ev["c0"].elapsed_time(ev["c1"])
            parts["compute_ms"] += ev["s0"].elapsed_time(ev["s1"])
            parts["allreduce_readback_ms"] += ev["s1"].elapsed_time(ev["s2"])
        return loss

    upload(0, False)
    i = 0
    for _ in range(max(1, min(args.warmup, 2))):
        step(i, False)
        i += 1
    torch.cuda.synchronize()
    barrier(world)
    steps = max(1, min(args.steps, args.e2e_steps))
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(steps):
        step(i, False)
        i += 1
    en.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(st.elapsed_time(en) / steps, world)
    # one more step with events between its parts (the timed steps carry none)
    step(i, True)
    cam = w.cameras[0]
    return {"value": round(len(w.cameras) * cam.height * cam.width / 1e6 / (ms / 1e3), 3),
            "unit": UNIT, "ms_per_step": round(ms, 4), "steps": steps,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4,
            "breakdown_ms_one_step": {k: round(v, 3) for k, v in parts.items()},
            "path": f"multiview.fit_step_views (this rank's views binned {group} at a time, the "
                    "groups pipelined over two streams, gradients into one flat buffer, NCCL "
                    "all-reduce in place) per step; the "
                    "surfel parameters and the rank's target images copied from pinned host "
                    "memory every step on a copy stream, double-buffered (step s + 1's inputs "
                    "upload while step s runs); the loss read back every step"}


def run_e2e_3d(w, args, world, rank, surface, views=None):
    """The step through gsplat.rasterize_hexels3d (autograd), the surfel
    parameters and this rank's target images copied from pinned host memory
    every step and the loss read back.  `views`: this rank's views (default:
    round-robin)."""
    import gsplat

    if views is None:
        views = view_split(len(w.cameras), world, rank)
    host_params = [t.pin_memory() for t in (w.means3d, w.scales, w.rotations, w.colors,
                                           w.color_grads, w.view_grads, w.opacities)]
    host_targets = [t.pin_memory() for t in make_targets(w, views, "cpu")]
    cams = [w.cameras[v].to("cuda") for v in views]
    h2d = sum(t.numel() * t.element_size() for t in host_params + host_targets)
    bg = w.background.to("cuda")
    # the next view's target image is copied on a side stream while the
    # current view renders (double-buffered, as a training loop's loader would)
    main = torch.cuda.current_stream()
    copy_stream = torch.cuda.Stream()
    bufs = [torch.empty(host_targets[0].shape, device="cuda") for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def prefetch(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[b])
            bufs[b].copy_(host_targets[i], non_blocking=True)
            ready[b].record(copy_stream)

    def one():
        params = [t.to("cuda", non_blocking=True).requires_grad_(True) for t in host_params]
        total = torch.zeros((), device="cuda")
        prefetch(0)
        for i, cam in enumerate(cams):
            if i + 1 < len(cams):
                prefetch(i + 1)
            b = i % 2
            main.wait_event(ready[b])
            tgt = bufs[b]
            out = gsplat.rasterize_hexels3d(
                *params[:7], cam.viewmatrix, cam.projmatrix, cam.campos, bg, cam.width,
                cam.height, cam.tan_fovx, cam.tan_fovy, w.softness, return_surface=surface)
            loss = mse_loss(out[0], tgt)
            free[b].record(main)  # the target is read only by the loss kernel
            if surface:
                depth, normals = out[2], out[4]
                loss = loss + LAMBDA_DEPTH2 * (depth * depth).mean() + \
                    LAMBDA_NORMAL2 * (normals * normals).mean()
            loss.backward()
            total = total + loss.detach()
        if world > 1:
            import torch.distributed as dist

            packed = torch.cat([p.grad.view(-1) for p in params] + [total.view(1)])
            dist.all_reduce(packed)
            total = packed[-1]
        return float(total.item())

    for _ in range(max(1, min(args.warmup, 2))):
        one()
    torch.cuda.synchronize()
    barrier(world)
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, min(args.steps, args.e2e_steps))
    st.record()
    for _ in range(steps):
        one()
    en.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(st.elapsed_time(en) / steps, world)
    cam = w.cameras[0]
    return {"value": round(len(w.cameras) * cam.height * cam.width / 1e6 / (ms / 1e3), 3),
            "unit": UNIT, "ms_per_step": round(ms, 4), "steps": steps,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4,
            "path": "gsplat.rasterize_hexels3d(" + ("return_surface=True" if surface else "")
                    + ") per view + loss.backward(); each view's target copied from pinned "
                    "host memory on a side stream while the previous view renders"}


def ref_cuda_timing_3d(args, w, surface, steps=None):
    """The reference's CUDA kernels (compiled from its sources) on the same
    views, driven by the reference's own call sequence: the cached RGB path
    (rasterize_hexels3d_forward_cached + rasterize_hexels3d_backward_cached,
    gsplat/rasterize_hexels3d.py:957-1035,1363-1517) or, with surface outputs,
    rasterize_hexels3d_forward_all + the uncached rasterize_hexels3d_backward
    (gsplat/rasterize_hexels3d.py:2294-2491)."""
    path = os.path.join(ROOT, "oracle", "_ref", "_ref_hexels3d_C.so")
    if not os.path.exists(path):
        return None
    import importlib.util

    spec = importlib.util.spec_from_file_location("_ref_hexels3d_C", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    dev = torch.device("cuda")
    views = list(range(len(w.cameras)))
    m3, sc, rot, col, cg, vg, op = (t.to(dev) for t in (w.means3d, w.scales, w.rotations,
                                                        w.colors, w.color_grads, w.view_grads,
                                                        w.opacities))
    bg = w.background.to(dev)
    cams = [w.cameras[v].to(dev) for v in views]
    targets = make_targets(w, views, dev)
    H, W = cams[0].height, cams[0].width
    e = torch.empty(0, device=dev)
    zero_hw = torch.zeros((H, W), device=dev)
    numel = 3 * H * W
    hw = float(H * W)

    def step():
        for cam, tgt in zip(cams, targets):
            scal = (W, H, cam.tan_fovx, cam.tan_fovy, w.softness, 1.0, 1, 1, True)
            tens = (m3, sc, rot, col, cg, e, vg, e, e, op, e, cam.viewmatrix, cam.projmatrix,
                    cam.campos, bg)
            if surface:
                out = ref.rasterize_hexels3d_forward_all(*tens, *scal, False, False, False, True,
                                                         -1, False, False, False)
                g_color = (out[0] - tgt) * (2.0 / numel)
                gd = out[5] * (2 * LAMBDA_DEPTH2 / hw)
                gn = torch.cat([out[7][:3] * (2 * LAMBDA_NORMAL2 / (3 * hw)), zero_hw[None]])
                ref.rasterize_hexels3d_backward(m3, e, *tens[1:], g_color, e, gd, zero_hw, gn,
                                                *scal, -1, False, False, False)
            else:
                img, radii, saved = ref.rasterize_hexels3d_forward_cached(*tens, *scal, False,
                                                                          False, False)
                g_color = (img - tgt) * (2.0 / numel)
                ref.rasterize_hexels3d_backward_cached(m3, e, *tens[1:], g_color, e, e, e, e,
                                                       *scal, -1, False, False, False, saved)

    steps = max(1, min(args.steps, args.ref_max_steps)) if steps is None else steps
    for _ in range(min(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    total = 0.0
    for _ in range(steps):
        flush.zero_()
        st.record()
        step()
        en.record()
        torch.cuda.synchronize()
        total += st.elapsed_time(en)
    ms = total / steps
    return {"value": round(len(views) * H * W / 1e6 / (ms / 1e3), 3), "unit": UNIT,
            "ms_per_step": round(ms, 4), "steps": steps,
            "what": "reference CUDA kernels compiled from its sources for sm_100a "
                    "(-O3 --use_fast_math), its own call sequence "
                    + ("(forward_all + uncached backward, surface outputs)" if surface
                       else "(forward_cached + backward_cached)")
                    + ", same inputs and loss"}


def workload_3d(name, views=64):
    import workloads

    if name == "hexels3d_multiview":
        return workloads.hexels3d_multiview(views)
    if name == "hexels3d_single":
        return workloads.hexels3d_single()
    raise ValueError(name)


def cpu_baseline_3d(args, w):
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    secs, mpix, desc, parts = cpu_sample_run_3d(w, args.cpu_crop_tiles_3d)
    return {"value": round(mpix / secs, 5), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": desc, "seconds": round(secs, 3), **parts}


def cpu_sample_run_3d(w, crop_tiles: int):
    """One view's fwd+bwd by the oracle, timed in two parts: the per-view
    fixed work (preprocess of all surfels, binning of the whole frame,
    geometry VJP of all surfels) in full, and the per-pixel work (compositing
    and its backward) over a crop_tiles x crop_tiles tile crop at the centre
    of view 0, extrapolated to the frame by pixel count.  Returns (frame
    seconds, frame megapixels, description, parts)."""
    from oracle import hexels3d as o

    cam = w.cameras[0]
    r = o.sample_fwd_bwd_split(w, cam, crop_tiles, make_targets(w, [0], "cpu")[0])
    desc = (f"view 0 of {w.name}: per-view fixed work timed in full ({r['fixed_s']:.2f} s: "
            f"preprocess of all surfels, binning of the frame, geometry VJP), compositing "
            f"fwd+bwd timed over a {crop_tiles}x{crop_tiles}-tile ({r['crop_mpix']:.4f} Mpix) "
            f"centre crop ({r['pixel_s']:.2f} s) and scaled to the frame by pixel count: "
            f"{r['frame_s']:.1f} s per frame")
    parts = {"fixed_s": round(r["fixed_s"], 3), "crop_pixel_s": round(r["pixel_s"], 3),
             "crop_mpix": round(r["crop_mpix"], 5), "frame_s": round(r["frame_s"], 2)}
    return r["frame_s"], r["frame_mpix"], desc, parts


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (restated reference algorithm) on host cores
# ---------------------------------------------------------------------------
def cpu_sample_run(w, crop_tiles: int):
    """One fwd+bwd of the oracle over a crop of crop_tiles x crop_tiles tiles
    at the image centre; returns (seconds, megapixels)."""
    import numpy as np

    from oracle import raster2d as o

    tx, ty, _ = w.tile_bounds
    x0 = max(0, tx // 2 - crop_tiles // 2)
    y0 = max(0, ty // 2 - crop_tiles // 2)
    xs = np.arange(x0, min(tx, x0 + crop_tiles))
    ys = np.arange(y0, min(ty, y0 + crop_tiles))
    tiles = (ys[:, None] * tx + xs[None, :]).reshape(-1)
    t0 = time.perf_counter()
    m = w.means2d.clone().requires_grad_(False)
    xys, radii, conics, nth = o.project_2d(m, w.scales2d, w.rotation, w.height, w.width,
                                           w.tile_bounds)
    # bin only Gaussians whose rectangle meets the crop
    rx0, ry0, rx1, ry1 = o.tile_rect(xys.numpy(), radii.numpy().astype(np.float32), tx, ty)
    meet = ((radii.numpy() > 0) & (rx1 > xs[0]) & (rx0 <= xs[-1]) & (ry1 > ys[0]) &
            (ry0 <= ys[-1]))
    sub = np.nonzero(meet)[0]
    keys, ids = o.map_intersects(xys.numpy()[sub], radii.numpy()[sub], None, w.tile_bounds,
                                 tile_rows=(int(ys[0]), int(ys[-1]) + 1))
    ids = sub[ids] if ids.size else ids
    _, ids_sorted, bins = o.sort_and_bin(keys, ids.astype(np.int32), tx * ty)
    img, topk, _, _ = o.rasterize_topk_forward(xys, conics, w.colors, torch.from_numpy(ids_sorted),
                                               bins, w.height, w.width, tile_ids=tiles)
    v_img = torch.zeros_like(img)
    rows = slice(int(ys[0]) * 16, min((int(ys[-1]) + 1) * 16, w.height))
    cols = slice(int(xs[0]) * 16, min((int(xs[-1]) + 1) * 16, w.width))
    v_img[rows, cols] = 2.0 * (img[rows, cols] - w.target[rows, cols]) / img.numel()
    topk_crop = torch.full_like(topk, -1)
    topk_crop[rows, cols] = topk[rows, cols]
    v_xy, v_conic, v_colors = o.rasterize_topk_backward(xys, conics, w.colors, v_img, topk_crop,
                                                        w.height, w.width)
    o.project_2d_backward(w.scales2d, w.rotation, w.height, w.width, radii, conics, v_xy, v_conic)
    secs = time.perf_counter() - t0
    mpix = (rows.stop - rows.start) * (cols.stop - cols.start) / 1e6
    return secs, mpix


def cpu_baseline(args, w):
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    crop = max(1, min(args.cpu_crop_tiles, w.tile_bounds[0]))
    secs, mpix = cpu_sample_run(w, crop)
    return {"value": round(mpix / secs, 5), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"one fwd+bwd over a {crop}x{crop}-tile ({mpix:.4f} Mpix) centre crop of "
                      f"{w.name}: projection of all Gaussians, binning of those meeting the "
                      f"crop, top-10 compositing and backward; {secs:.2f} s",
            "seconds": round(secs, 3)}


def run_reference(args, world, rank):
    """Reference arm: the CPU restatement of the reference's algorithm (the
    reference has no CPU implementation), all host threads, a bounded sample
    of the workload per step.  Rank 0 only."""
    if rank != 0:
        return None
    import workloads

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    three_d = args.config.startswith("hexels3d")
    if three_d:
        w = workload_3d(args.config, args.views)
        crop = args.cpu_crop_tiles_3d
        sample = lambda: cpu_sample_run_3d(w, crop)[:2]  # noqa: E731
        cam = w.cameras[0]
        config = {"workload": w.name, "views": len(w.cameras), "height": cam.height,
                  "width": cam.width, "num_surfels": w.num_points,
                  "outputs": "rgb + depth + alpha + normal + distortion"
                  if args.config == "hexels3d_single" else "rgb"}
    elif args.config == "hexels2d":
        w = workloads.hexels2d()
        crop = max(1, min(args.cpu_crop_tiles, w.tile_bounds[0]))
        sample = lambda: cpu_sample_run_hex2d(w, crop)  # noqa: E731
        config = {"workload": w.name, "height": w.height, "width": w.width,
                  "num_hexagons": w.num_points, "top_k": 10, "tile": 16}
    else:
        w = getattr(workloads, args.config)()
        crop = max(1, min(args.cpu_crop_tiles, w.tile_bounds[0]))
        sample = lambda: cpu_sample_run(w, crop)  # noqa: E731
        config = {"workload": w.name, "height": w.height, "width": w.width,
                  "num_gaussians": w.num_points, "top_k": 10, "tile": 16}
    warm = min(args.warmup, 3)  # a CPU sample takes seconds: at most 3 untimed
    for _ in range(warm):
        sample()
    secs_total, mpix_total = 0.0, 0.0
    steps = max(1, min(args.steps, args.ref_max_steps))
    for _ in range(steps):
        s, mp = sample()
        secs_total += s
        mpix_total += mp
    value = mpix_total / secs_total
    return {
        "metric": METRIC, "value": round(value, 5), "unit": UNIT, "impl": "reference",
        "n_gpus": world, "steps": steps, "warmup": warm,
        "ms_per_step": round(secs_total / steps * 1e3, 2),
        "higher_is_better": True, "scaling": "strong" if three_d else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": config,
        "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": threads,
                         "kind": "port",
                         "sample": (f"each step: one view (view 0) fwd+bwd, its fixed work "
                                    f"(preprocess of all surfels, binning of the frame, "
                                    f"geometry VJP) timed in full and its compositing fwd+bwd "
                                    f"timed over a {crop}x{crop}-tile centre crop and scaled to "
                                    f"the frame by pixel count" if three_d else
                                    f"each step: one fwd+bwd over a {crop}x{crop}-tile centre "
                                    f"crop ({mpix_total / steps:.4f} Mpix)")
                                   + "; the reference ships CUDA only, so this is its "
                                   "algorithm restated on the CPU"},
        "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# the reference's own CUDA kernels (built from its sources), same GPU
# ---------------------------------------------------------------------------
def ref_cuda_timing(args, w):
    path = os.path.join(ROOT, "oracle", "_ref", "_ref_gsplat_csrc.so")
    if not os.path.exists(path):
        return None
    import importlib.util

    spec = importlib.util.spec_from_file_location("_ref_gsplat_csrc", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    dev = torch.device("cuda")
    m, s, r, c, tgt = (t.to(dev) for t in (w.means2d, w.scales2d, w.rotation, w.colors, w.target))
    H, W, tb, n = w.height, w.width, w.tile_bounds, w.num_points
    numel = H * W * 3

    def step():
        # the reference's own call sequence (rasterize_sum.py:54-226, utils.py:96-162)
        xys, radii, conics, nth = ref.project_gaussians_2d_scale_rot_forward(n, m, s, r, H, W, tb)
        cum = torch.cumsum(nth, dim=0, dtype=torch.int32)
        ni = int(cum[-1].item())
        isect, gids = ref.map_gaussian_to_intersects(n, ni, xys, radii, cum, tb)
        isect_s, order = torch.sort(isect)
        gids_s = torch.gather(gids, 0, order)
        bins = ref.get_tile_bin_edges(ni, tb[0] * tb[1], isect_s)
        img, topk = ref.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (W, H, 1), gids_s, bins,
                                                       xys, conics, c)
        d = img - tgt
        loss = (d * d).sum() / numel
        v_img = d * (2.0 / numel)
        v_xy, v_conic, v_col = ref.nd_rasterize_backward_topk_norm(H, W, 16, 16, gids_s, bins, xys,
                                                                   conics, c, v_img, topk)
        ref.project_gaussians_2d_scale_rot_backward(n, m, s, r, H, W, radii, conics, v_xy, v_conic)
        return loss

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    total = 0.0
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(args.steps):
        flush.zero_()
        st.record()
        step()
        en.record()
        torch.cuda.synchronize()
        total += st.elapsed_time(en)
    ms = total / args.steps
    return {"value": round(H * W / 1e6 / (ms / 1e3), 3), "unit": UNIT, "ms_per_step": round(ms, 4),
            "what": "reference CUDA kernels compiled from its sources for sm_100a "
                    "(-O3 --use_fast_math), driven by its own Python call sequence"}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="hexels3d_multiview",
                    choices=["hexels3d_multiview", "hexels3d_single", "imagegs_large",
                             "imagegs_small", "hexels2d"])
    ap.add_argument("--views", type=int, default=64,
                    help="views of the multi-view orbit (64 is the benchmark configuration; "
                         "fewer, e.g. 1, for a small profiling case)")
    ap.add_argument("--group", type=int, default=8,
                    help="multi-view step: views binned together per group (1 = per view); "
                         "capped at half of a rank's views")
    ap.add_argument("--cpu-crop-tiles", type=int, default=16)
    ap.add_argument("--cpu-crop-tiles-3d", type=int, default=8)
    ap.add_argument("--ref-max-steps", type=int, default=3)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--skip-extras", action="store_true",
                    help="time the device-resident step only (no e2e, CPU baseline or "
                         "reference CUDA timing), e.g. under a profiler")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0

    world, rank, local = dist_setup(args.gpus)
    try:
        if args.config.startswith("hexels3d"):
            line = run_ours_3d(args, world, rank, local)
        elif args.config == "hexels2d":
            line = run_ours_hex2d(args, world, rank, local)
        else:
            line = run_ours(args, world, rank, local)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
