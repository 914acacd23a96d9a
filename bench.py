"""Benchmark of the r2splat hot path on B200: projection fwd+bwd and voxelization fwd+bwd.

Metric: Gaussian*views/s of projection forward+backward
(``value``) and Mvoxels/s of voxelization forward+backward (``voxelize``), on
benchmark config 2 by default: 500,000 Gaussians, 75 views over 360 degrees,
512x512 detector, 256^3 grid (seeded synthetic inputs, r2s_workloads.py).

One projection step is the reference's explicit training step without the
loss, through the public op API ``r2splat.ops.explicit`` as callers use it:
prepare (parameter transform + softplus), explicit rasterize (projection,
binning, rasterizer), then explicit backward with a seeded N(0,1) upstream
image gradient.  One voxel step is prepare, explicit rasterize of no view
(the op layer requires a projection pass before its backward,
r2splat/ops/explicit.py:255-256 of the reference), explicit voxelize of the
grid and explicit backward with a seeded N(0,1) upstream volume gradient.
The projection pass renders zero views: both op layers return empty buffers
for it without a launch, so the voxel step times voxelization alone.

Multi-GPU (torchrun, one process per GPU, NCCL): by default the job's 75
views are dealt to the ranks, every N-th view starting at the rank
(``--scaling strong``: the same job split over the GPUs), and the
per-Gaussian gradients are summed with one NCCL all-reduce per step;
``--scaling weak`` gives every rank 75 views of a 75*N-view orbit instead.
The voxel grid is split into N z-slabs of whole brick layers, balanced by
each layer's records plus a per-brick cost (strong scaling).  ``value`` is the
whole job's Gaussian*views over the max-over-ranks step time.  Each timed step
lies between its own pair of CUDA events; the 256 MiB L2 flush before each
step lies outside them.

``--rank-shares N`` (one GPU) times each rank's share of an N-GPU strong-scaling
job in turn, with the same step objects and no collective, and prints the
per-rank step times and phases: what limits N GPUs, measured on one.

``--impl reference`` runs the reference implementation of the path on rank 0:
its own Python op layer, unchanged (``baseline/_ref``), over its own CUDA
sources built for sm_100a (``oracle/_ref``), through the same public calls
and on the same workload (config 3 in batches of 20 views, past its int32
record limit, as its callers must).
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
for _p in (os.path.join(ROOT, "bt-3dgs_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

import r2s_shard as shard  # noqa: E402
import r2s_workloads as wl  # noqa: E402

L2_FLUSH_BYTES = 256 << 20
# the projection pass of the voxel step: zero views (the op layer requires a
# projection pass before its backward; with no view it is empty)
VOXEL_STEP_VIEWS = 0
VOXEL_STEP_DETECTOR = 16


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(world, value: float) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_config(cfg, views: int) -> dict:
    """The workload keys both arms print (same dict for the same job)."""
    return {"workload": cfg.name, "n_gaussians": cfg.n_gaussians, "views": views,
            "detector": cfg.detector, "grid": cfg.grid,
            "l2": "256MiB flush between steps, outside the timed events"}


# ---------------------------------------------------------------------------
# end-to-end pipeline: host inputs -> device step -> host outputs
# ---------------------------------------------------------------------------
class HostPipeline:
    """Runs a step on inputs copied from pinned host memory and copies its
    result back, every step inside the timed region.  The copies run on a copy
    stream: the next step's inputs upload while this step computes (a
    double-buffered input pipeline) and the outputs download behind the next
    step into two alternating sets of pinned host buffers, allocated once, as
    a training loop keeps them.  Subclasses set ``self.host`` (pinned host
    inputs) and implement ``step(*device_inputs)`` returning the device
    tensors to download."""

    def _upload(self):
        with torch.cuda.stream(self.copy_stream):
            ins = [h.to(self.dev, non_blocking=True) for h in self.host]
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
        return ins, ev

    def reset_pipeline(self):
        self.copy_stream = torch.cuda.Stream(device=self.dev)
        self.prefetched = None
        # host output buffers survive a reset (allocated in the warm-up steps)
        self.out_sets = getattr(self, "out_sets", None)
        self.out_events = [None, None]
        self.out_turn = 0

    def _host_outputs(self, results):
        """The pinned host buffers of this step (the set the step before last
        used: its download has completed once its event has)."""
        if self.out_sets is None:
            self.out_sets = [[torch.empty(r.shape, dtype=r.dtype, pin_memory=True)
                              for r in results] for _ in range(2)]
        k = self.out_turn
        self.out_turn ^= 1
        if self.out_events[k] is not None:
            self.out_events[k].synchronize()
        return k, self.out_sets[k]

    def step_e2e(self, prefetch_next=True):
        if getattr(self, "copy_stream", None) is None:
            self.reset_pipeline()
        compute = torch.cuda.current_stream()
        ins, ev = self.prefetched if self.prefetched is not None else self._upload()
        self.prefetched = None
        compute.wait_event(ev)
        for t in ins:
            t.record_stream(compute)
        if prefetch_next:
            self.prefetched = self._upload()
        results = self.step(*ins)
        done = torch.cuda.Event()
        done.record(compute)
        self.copy_stream.wait_event(done)
        k, outs = self._host_outputs(results)
        with torch.cuda.stream(self.copy_stream):
            for o, r in zip(outs, results):
                o.copy_(r, non_blocking=True)
                r.record_stream(self.copy_stream)
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
        self.out_events[k] = ev
        return outs

    def bytes_e2e(self):
        h2d = sum(t.numel() * t.element_size() for t in self.host)
        return h2d, self.d2h_bytes


# ---------------------------------------------------------------------------
# this build
# ---------------------------------------------------------------------------
class OursProjection(HostPipeline):
    def __init__(self, cfg, world, rank, dev, scaling):
        from r2splat.ops import explicit as E

        self.E, self.world, self.cfg, self.dev = E, world, cfg, dev
        self.det = cfg.detector
        m, q, s, o = wl.make_gaussians(cfg)
        self.params = [t.to(dev) for t in (m, q, s, o)]
        if scaling == "weak":
            first, count, total, stride = shard.view_shard(cfg.n_views, rank, world)
        else:
            first, count, total, stride = shard.view_split(cfg.n_views, rank, world)
        self.views = count
        vm, K = wl.make_cameras(count, cfg.detector, first=first, count=count, total=total,
                                stride=stride)
        self.vm, self.K = vm.to(dev), K.to(dev)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        self.v_img = torch.randn((count, self.det, self.det), generator=g, device=dev)
        self.host = [t.pin_memory() for t in (m, q, s, o, vm, K)] + [self.v_img.cpu().pin_memory()]
        self.d2h_bytes = sum(t.numel() * t.element_size() for t in (m, q, s, o))
        self.allreduce = shard.GradientAllReduce()

    def step(self, m=None, q=None, s=None, o=None, vm=None, K=None, v_img=None):
        E = self.E
        if m is None:
            m, q, s, o = self.params
            vm, K, v_img = self.vm, self.K, self.v_img
        params = (m, q, s, o)
        for p in params:
            p.grad = None
        st = E.prepare_explicit_gaussians(q, s, o, scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
        res = E.explicit_rasterize(st, m, vm, K, img_w=self.det, img_h=self.det,
                                   tile_size=wl.IMG_TILE, eps2d=wl.EPS2D,
                                   radius_clip=wl.RADIUS_CLIP, absgrad=True)
        res.image.grad = v_img
        E.explicit_backward(st, *params)
        grads = [p.grad for p in params]
        if self.world > 1:
            self.allreduce(grads)
        return grads

    def phases(self):
        """Per-phase device time of one step (CUDA events between the same
        calls the op layer makes), ms."""
        from r2splat.cuda import _wrapper as W

        m, q, s, o = self.params
        C, N, det = self.views, m.size(0), self.det
        nt = (det + wl.IMG_TILE - 1) // wl.IMG_TILE
        stats = torch.empty((C * N, 8), dtype=torch.float32, device=self.dev)
        T = PhaseTimer()
        with torch.no_grad():
            cov, ms, op = W.fused_prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
            T.mark("prepare")
            m2, radii, splats, rects, _ = W.fused_project(m, cov, op, self.vm, self.K, det, det,
                                                          wl.IMG_TILE, nt, nt, wl.EPS2D,
                                                          wl.RADIUS_CLIP)
            T.mark("project")
            # the op layer's binning: all views at once, or contiguous view
            # batches when the records pass the int32 tile offsets (config 3)
            binned = W.fused_bin(rects, C, N, nt * nt, nt, 0, limit=W.MAX_RECORDS_PER_BATCH)
            batches = ([(0, C, binned)] if binned is not None else
                       [(c0, c1, None) for c0, c1 in W.plan_view_batches(rects, C, N)])
            for c0, c1, pre in batches:
                offs, ids, _ = pre if pre is not None else W.fused_bin(
                    rects[c0 * N * 8:c1 * N * 8], c1 - c0, N, nt * nt, nt, 0)
                T.mark("binning (incl. host read of the record count)")
                cull = torch.empty(ids.shape, dtype=torch.int16, device=self.dev)
                W.fused_raster_fwd(splats[c0:c1], offs, ids, c1 - c0, N, det, det, wl.IMG_TILE,
                                   nt, nt, cull=cull)
                T.mark("raster forward")
                W.fused_raster_bwd(splats[c0:c1], offs, ids, self.v_img[c0:c1], c1 - c0, N, det,
                                   det, wl.IMG_TILE, nt, nt, True, out=stats[c0 * N:c1 * N],
                                   cull=cull)
                T.mark("raster backward")
                del offs, ids, cull, pre
            outs = [torch.empty_like(t) for t in (m, q, s, o)]
            v2 = torch.empty((C, N, 2), device=self.dev)
            v2a = torch.empty((C, N, 2), device=self.dev)
            W.fused_explicit_backward(m, q, s, o, wl.SCALE_MIN, wl.SCALE_MAX, self.vm, self.K, det,
                                      det, wl.EPS2D, stats, v2, v2a, None, None, 0, 0, 0, 0.0,
                                      None, False, outs)
            T.mark("explicit backward")
            if self.world > 1:
                self.allreduce(outs)
            T.mark("gradient all-reduce")
        res = T.result()
        res["view_batches"] = len(batches)
        return res


class OursVoxel(HostPipeline):
    def __init__(self, cfg, world, rank, dev, host_params):
        from r2splat.ops import explicit as E

        self.E, self.world, self.dev = E, world, dev
        self.G = G = cfg.grid
        self.nt = (G + wl.VOL_TILE - 1) // wl.VOL_TILE
        rng, ctr = wl.unit_cube_box()
        self.rng, self.ctr = rng.to(dev), ctr.to(dev)
        self.params = [t.to(dev) for t in host_params]
        vm1, K1 = wl.make_cameras(VOXEL_STEP_VIEWS, VOXEL_STEP_DETECTOR)
        self.vm1, self.K1 = vm1.to(dev), K1.to(dev)
        if world > 1:
            # z-slabs balanced by the cost of each brick layer, its records
            # plus a per-brick share (every rank computes the same ranges from
            # the same mapping)
            from r2splat.cuda import _wrapper as W

            with torch.no_grad():
                m, q, s, o = self.params
                cov, _, op = W.fused_prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
                rects = W.fused_map(m, cov, op, self.rng, self.ctr, G, G, G, wl.VOL_TILE,
                                    self.nt, self.nt, self.nt, wl.EPS3D, wl.RADIUS_CLIP)[4]
            self.layers = shard.balanced_layer_ranges(shard.layer_costs(rects, self.nt,
                                                                        self.nt * self.nt),
                                                      world)[rank]
        else:
            self.layers = None
        l0, l1 = self.layers or (0, self.nt)
        z0, z1 = shard.slab_rows(l0, l1, wl.VOL_TILE, G)
        g = torch.Generator(device=dev).manual_seed(200 + rank)
        self.v_vol = torch.randn((z1 - z0, G, G), generator=g, device=dev)
        self.host = [t.pin_memory() for t in host_params] + [self.v_vol.cpu().pin_memory()]
        self.d2h_bytes = sum(t.numel() * t.element_size() for t in host_params)
        self.allreduce = shard.GradientAllReduce()

    def step(self, m=None, q=None, s=None, o=None, v_vol=None):
        E, G = self.E, self.G
        if m is None:
            m, q, s, o = self.params
            v_vol = self.v_vol
        params = (m, q, s, o)
        for p in params:
            p.grad = None
        st = E.prepare_explicit_gaussians(q, s, o, scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
        E.explicit_rasterize(st, m, self.vm1, self.K1, img_w=VOXEL_STEP_DETECTOR,
                             img_h=VOXEL_STEP_DETECTOR, tile_size=wl.IMG_TILE, eps2d=wl.EPS2D,
                             radius_clip=wl.RADIUS_CLIP, absgrad=False)
        vr = E.explicit_voxelize(st, m, self.rng, self.ctr, dim2=G, dim1=G, dim0=G,
                                 tile_size=wl.VOL_TILE, eps3d=wl.EPS3D,
                                 radius_clip=wl.RADIUS_CLIP, z_layers=self.layers)
        vr.volume.grad = v_vol
        E.explicit_backward(st, *params)
        grads = [p.grad for p in params]
        if self.world > 1:
            self.allreduce(grads)
        return grads

    def phases(self):
        """Per-phase device time of one voxel step, ms (the same calls the op
        layer makes, without the empty projection pass)."""
        from r2splat.cuda import _wrapper as W

        m, q, s, o = self.params
        G, nt, N = self.G, self.nt, m.size(0)
        l0, l1 = self.layers or (0, nt)
        T = PhaseTimer()
        with torch.no_grad():
            cov, ms, op = W.fused_prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
            T.mark("prepare")
            m3, c3, r3, vs, rects, _ = W.fused_map(m, cov, op, self.rng, self.ctr, G, G, G,
                                                   wl.VOL_TILE, nt, nt, nt, wl.EPS3D,
                                                   wl.RADIUS_CLIP)
            T.mark("volume mapping")
            offs, fids, _ = W.fused_bin(rects, l1 - l0, N, nt * nt, nt, 1, segment_base=l0)
            order = W.fused_brick_order(offs, fids.numel())
            T.mark("3D binning (incl. host read of the record count) + brick order")
            rows = W.fused_voxel_rows(vs, offs, fids, N, G, G, G, wl.VOL_TILE, nt, nt, nt, l0, l1,
                                      order=order)
            T.mark("row table")
            W.fused_voxel_fwd(vs, offs, fids, N, G, G, G, wl.VOL_TILE, nt, nt, nt, l0, l1,
                              rows=rows, order=order)
            T.mark("voxel forward")
            stats = W.fused_voxel_bwd(vs, offs, fids, self.v_vol, N, G, G, G, wl.VOL_TILE, nt, nt,
                                      nt, l0, l1, rows=rows, order=order)
            T.mark("voxel backward")
            outs = [torch.empty_like(t) for t in (m, q, s, o)]
            W.fused_explicit_backward(m, q, s, o, wl.SCALE_MIN, wl.SCALE_MAX, None, None, 0, 0,
                                      wl.EPS2D, None, None, None, self.rng, self.ctr, G, G, G,
                                      wl.EPS3D, stats, False, outs)
            T.mark("explicit backward")
            if self.world > 1:
                self.allreduce(outs)
            T.mark("gradient all-reduce")
        res = T.result()
        res["layers"] = [l0, l1]
        res["records"] = int(fids.numel())
        return res


class PhaseTimer:
    """CUDA events between consecutive phases on the current stream (ranks
    start together: a barrier first, so no phase absorbs another rank's
    lateness)."""

    def __init__(self):
        torch.cuda.synchronize()
        if torch.distributed.is_available() and torch.distributed.is_initialized():
            torch.distributed.barrier()
            torch.cuda.synchronize()
        self.events = [("start", self._ev())]

    @staticmethod
    def _ev():
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def mark(self, name):
        self.events.append((name, self._ev()))

    def result(self):
        torch.cuda.synchronize()
        out = {}
        for (_, a), (name, b) in zip(self.events, self.events[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)  # a phase repeated per batch sums
        out = {k: round(v, 4) for k, v in out.items()}
        return {"ms": out, "total_ms": round(sum(out.values()), 4)}


# ---------------------------------------------------------------------------
# the reference: its unchanged op layer over its own CUDA build
# ---------------------------------------------------------------------------
class RefProjection:
    def __init__(self, cfg, dev):
        from oracle import ref_stock

        self.S = ref_stock.stock_r2splat().explicit
        self.cfg = cfg
        self.det = cfg.detector
        m, q, s, o = wl.make_gaussians(cfg)
        self.params = [t.to(dev) for t in (m, q, s, o)]
        vm, K = wl.make_cameras(cfg.n_views, cfg.detector)
        self.vm, self.K = vm.to(dev), K.to(dev)
        g = torch.Generator(device=dev).manual_seed(100)
        self.v_img = torch.randn((cfg.n_views, self.det, self.det), generator=g, device=dev)

    # the reference's int32 tile offsets overflow past 2^31 records (config 3):
    # there its callers must render in batches; 20 views per batch fit

    def step(self):
        S = self.S
        m, q, s, o = self.params
        for p in self.params:
            p.grad = None
        C = self.vm.shape[0]
        per = 20 if self.cfg.name.startswith("cfg3") else C
        for c0 in range(0, C, per):
            c1 = min(C, c0 + per)
            st = S.prepare_explicit_gaussians(q, s, o, scale_min=wl.SCALE_MIN,
                                              scale_max=wl.SCALE_MAX)
            res = S.explicit_rasterize(st, m, self.vm[c0:c1], self.K[c0:c1], img_w=self.det,
                                       img_h=self.det, tile_size=wl.IMG_TILE, eps2d=wl.EPS2D,
                                       radius_clip=wl.RADIUS_CLIP, absgrad=True)
            res.image.grad = self.v_img[c0:c1]
            S.explicit_backward(st, m, q, s, o)


class RefVoxel:
    def __init__(self, cfg, dev, proj: RefProjection):
        self.S = proj.S
        self.params = proj.params
        self.G = cfg.grid
        rng, ctr = wl.unit_cube_box()
        self.rng, self.ctr = rng.to(dev), ctr.to(dev)
        vm1, K1 = wl.make_cameras(VOXEL_STEP_VIEWS, VOXEL_STEP_DETECTOR)
        self.vm1, self.K1 = vm1.to(dev), K1.to(dev)
        g = torch.Generator(device=dev).manual_seed(200)
        self.v_vol = torch.randn((self.G,) * 3, generator=g, device=dev)

    def step(self):
        S, G = self.S, self.G
        m, q, s, o = self.params
        for p in self.params:
            p.grad = None
        st = S.prepare_explicit_gaussians(q, s, o, scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
        S.explicit_rasterize(st, m, self.vm1, self.K1, img_w=VOXEL_STEP_DETECTOR,
                             img_h=VOXEL_STEP_DETECTOR, tile_size=wl.IMG_TILE, eps2d=wl.EPS2D,
                             radius_clip=wl.RADIUS_CLIP, absgrad=False)
        vr = S.explicit_voxelize(st, m, self.rng, self.ctr, dim2=G, dim1=G, dim0=G,
                                 tile_size=wl.VOL_TILE, eps3d=wl.EPS3D,
                                 radius_clip=wl.RADIUS_CLIP)
        vr.volume.grad = self.v_vol
        S.explicit_backward(st, m, q, s, o)


# ---------------------------------------------------------------------------
# config 4: the training step (projection + TV sub-volume + losses + Adam)
# ---------------------------------------------------------------------------
TRAIN_VIEWS_PER_STEP = 8
TRAIN_POOL = 32          # orbit views with seeded synthetic targets
TRAIN_TV = 64            # edge of the random TV sub-volume (voxels)
TRAIN_GRID = 256         # full-grid resolution that fixes the sub-volume's voxel size
TRAIN_WEIGHTS = dict(w_l1=0.8, w_ssim=0.2, w_tv=0.05, w_edge=0.1)
TRAIN_LRS = {"means": 1.6e-4, "quats": 1e-3, "scales": 5e-3, "opacities": 5e-2}
TRAIN_KEYS = ["means", "scales", "quats", "opacities"]
TRAIN_SPLIT_EVERY = 100   # binary split of a seeded subset every 100 steps
TRAIN_SPLIT_FRAC = 0.05
TRAIN_SCALE_EPS = 1e-5    # configs/model/binary_tree.yaml:8


def split_mask(step, n, dev):
    """The seeded 5 % subset split at `step` (the same on every rank)."""
    g = torch.Generator(device=dev).manual_seed(5000 + step)
    return torch.rand(n, generator=g, device=dev) < TRAIN_SPLIT_FRAC


def warm_split_path(split_fn, model_cls_or_none, dev):
    """Run one split of a small throwaway model so that the kernels the
    split uses (the library's and torch's, loaded lazily on first launch) are
    loaded before the timed window, as they are in a long training run."""
    tree = TreeParams(*wl.make_gaussians(wl.CONFIGS[0], n=1000), dev)
    if model_cls_or_none is not None:
        m = model_cls_or_none(device=str(dev), min_scale=wl.SCALE_MIN, max_scale=wl.SCALE_MAX,
                              scale_eps=TRAIN_SCALE_EPS)
        for name in vars(tree):
            setattr(m, name, getattr(tree, name))
        tree = m
    opts = {k: torch.optim.Adam([{"params": getattr(tree, k), "name": k}], lr=1e-3, eps=1e-15)
            for k in TRAIN_KEYS}
    for k in TRAIN_KEYS:
        getattr(tree, k).grad = torch.zeros_like(getattr(tree, k))
        opts[k].step()
    state = {"grad2d": torch.zeros(1000, device=dev), "count": torch.zeros(1000, device=dev)}
    split_fn(tree, opts, state, split_mask(0, 1000, dev))
    torch.cuda.synchronize()


def first_train_step(steps, warmup):
    """Number of the first (warm-up) step, chosen so that the split at step
    TRAIN_SPLIT_EVERY falls inside the timed window."""
    return max(1, TRAIN_SPLIT_EVERY - warmup - steps // 2)


class TreeParams:
    """The four raw parameters and the binary-tree buffers of a model (the
    attributes the split reads and replaces)."""

    def __init__(self, m, q, s, o, dev):
        self.means = torch.nn.Parameter(m.to(dev))
        self.quats = torch.nn.Parameter(q.to(dev))
        self.scales = torch.nn.Parameter(s.to(dev))
        self.opacities = torch.nn.Parameter(o.to(dev))
        n = m.shape[0]
        self.parent = torch.full((n,), -1, dtype=torch.int32, device=dev)
        self.level = torch.zeros((n,), dtype=torch.int32, device=dev)
        self.history_means = torch.empty((0, 3), device=dev)
        self.history_scales = torch.empty((0, 3), device=dev)
        self.history_quats = torch.empty((0, 4), device=dev)
        self.history_opacities = torch.empty((0,), device=dev)
        self.history_parent = torch.empty((0,), dtype=torch.int32, device=dev)
        self.history_level = torch.empty((0,), dtype=torch.int32, device=dev)


class TrainData:
    """Seeded synthetic data of the training step: a pool of orbit views with
    target projections of a teacher Gaussian set and edge masks, the per-step
    view choice and the per-step TV sub-box (default.py:444-470 restated:
    a box of TRAIN_TV voxels of a TRAIN_GRID^3 grid over the unit cube, centre
    uniform in the valid range)."""

    def __init__(self, cfg, dev, render_targets):
        self.det = cfg.detector
        vm, K = wl.make_cameras(TRAIN_POOL, cfg.detector)
        self.vm, self.K = vm.to(dev), K.to(dev)
        self.targets = render_targets(self.vm, self.K)  # [P, H, W]
        g = torch.Generator(device=dev).manual_seed(401)
        self.edge = (torch.rand(self.targets.shape, generator=g, device=dev) < 0.2).float()
        self.box = TRAIN_TV / TRAIN_GRID

    def step_views(self, step, rank, world):
        g = torch.Generator().manual_seed(1000 + step)
        views = torch.randperm(TRAIN_POOL, generator=g)[:TRAIN_VIEWS_PER_STEP]
        per = (TRAIN_VIEWS_PER_STEP + world - 1) // world
        return views[rank * per:(rank + 1) * per]

    def step_box(self, step, dev):
        g = torch.Generator().manual_seed(2000 + step)
        half = self.box / 2
        center = (-0.5 + half) + (1.0 - 2 * half) * torch.rand(3, generator=g, dtype=torch.float64)
        return (torch.full((3,), self.box, dtype=torch.float32, device=dev),
                center.float().to(dev))


def _teacher(cfg):
    import dataclasses

    return wl.make_gaussians(dataclasses.replace(cfg, seed=cfg.seed + 40), n=200_000)


class OursTrain:
    def __init__(self, cfg, world, rank, dev):
        from r2splat.ops import explicit as E
        from r2splat.ops import training as T

        self.E, self.T = E, T
        self.cfg, self.world, self.rank, self.dev = cfg, world, rank, dev
        tm, tq, ts, to = (t.to(dev) for t in _teacher(cfg))

        def render(vm, K):
            with torch.no_grad():
                st = E.prepare_explicit_gaussians(tq, ts, to, scale_min=wl.SCALE_MIN,
                                                  scale_max=wl.SCALE_MAX)
                return E.explicit_rasterize(st, tm, vm, K, img_w=cfg.detector,
                                            img_h=cfg.detector, tile_size=wl.IMG_TILE,
                                            eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP,
                                            absgrad=False).image.detach().clone()

        self.data = TrainData(cfg, dev, render)
        self.model = TreeParams(*wl.make_gaussians(cfg), dev)
        self.opts = {k: torch.optim.Adam([{"params": getattr(self.model, k), "name": k}],
                                         lr=TRAIN_LRS[k], eps=1e-15) for k in TRAIN_KEYS}
        self.loss = T.FusedBinaryTreeLossComputer(**TRAIN_WEIGHTS)
        self.densify = {"grad2d": None, "count": None}
        self.allreduce = shard.GradientAllReduce()
        self.step_no = 0
        self.sizes = []  # Gaussians rendered per step
        warm_split_path(lambda m, o, st, mask: T.binary_split(
            m, o, st, mask, TRAIN_KEYS, revised_opacity=True, scale_min=wl.SCALE_MIN,
            scale_max=wl.SCALE_MAX, scale_eps=TRAIN_SCALE_EPS), None, dev)

    def step(self):
        E, T, d, M = self.E, self.T, self.data, self.model
        P = {k: getattr(M, k) for k in TRAIN_KEYS}
        views = d.step_views(self.step_no, self.rank, self.world).to(self.dev)
        rng, ctr = d.step_box(self.step_no, self.dev)
        step_no = self.step_no
        self.step_no += 1
        self.sizes.append(P["means"].shape[0])
        st = E.prepare_explicit_gaussians(P["quats"], P["scales"], P["opacities"],
                                          scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
        res = E.explicit_rasterize(st, P["means"], d.vm[views], d.K[views], img_w=d.det,
                                   img_h=d.det, tile_size=wl.IMG_TILE, eps2d=wl.EPS2D,
                                   radius_clip=wl.RADIUS_CLIP, absgrad=True)
        vox = E.explicit_voxelize(st, P["means"], rng, ctr, dim2=TRAIN_TV, dim1=TRAIN_TV,
                                  dim0=TRAIN_TV, tile_size=wl.VOL_TILE, eps3d=wl.EPS3D,
                                  radius_clip=wl.RADIUS_CLIP)
        out = self.loss(res.image[..., None], d.targets[views][..., None],
                        d.edge[views][..., None], vox.volume)
        if self.world > 1:  # gradients summed over ranks = the one-GPU step's gradients
            objective = shard.data_parallel_objective(
                out, self.loss.w_l1, self.loss.w_ssim, self.loss.w_tv, len(views),
                TRAIN_VIEWS_PER_STEP, self.world)
        else:
            objective = out["total"]
        objective.backward()
        # densification statistics in the backward kernel; every rank adds its
        # own views with the step's global camera count, so the sum of the
        # ranks' states (taken when the strategy reads them) is the one-GPU state
        E.explicit_backward(st, P["means"], P["quats"], P["scales"], P["opacities"],
                            densify=T.DensifyAccumulator(self.densify, absgrad=True,
                                                         n_cameras=TRAIN_VIEWS_PER_STEP))
        if self.world > 1:
            self.allreduce([p.grad for p in P.values()])
        if step_no % TRAIN_SPLIT_EVERY == 0:
            # the strategy's split after the backward, before the optimizer
            # step (src/trainers/binary_tree.py:193-206): the new parameters
            # have no gradient, so that Adam step skips them, as torch's does
            T.binary_split(M, self.opts, self.densify, split_mask(step_no, P["means"].shape[0],
                                                                  self.dev),
                           TRAIN_KEYS, revised_opacity=True, scale_min=wl.SCALE_MIN,
                           scale_max=wl.SCALE_MAX, scale_eps=TRAIN_SCALE_EPS)
        T.adam_step(self.opts)
        for o in self.opts.values():
            o.zero_grad(set_to_none=True)
        return out["total"]


class RefTrain:
    """The same step through the reference's own code: its op layer
    (unchanged, baseline/_ref) over its CUDA build (oracle/_ref), its
    BinaryTreeLossComputer (src/utils/loss.py, unchanged) with autograd, the
    strategy's _update_state (restated in the oracle), its split()
    (src/strategies/binary_tree.py, unchanged) on its BinaryTreeGaussianModel,
    and torch.optim.Adam."""

    def __init__(self, cfg, dev):
        from oracle import r2s_oracle as O
        from oracle import ref_stock

        self.O, self.cfg, self.dev = O, cfg, dev
        self.S = ref_stock.stock_r2splat().explicit
        self.loss = ref_stock.load_loss_module().BinaryTreeLossComputer(**TRAIN_WEIGHTS)
        S = self.S
        tm, tq, ts, to = (t.to(dev) for t in _teacher(cfg))

        def render(vm, K):
            st = S.prepare_explicit_gaussians(tq, ts, to, scale_min=wl.SCALE_MIN,
                                              scale_max=wl.SCALE_MAX)
            return S.explicit_rasterize(st, tm, vm, K, img_w=cfg.detector, img_h=cfg.detector,
                                        tile_size=wl.IMG_TILE, eps2d=wl.EPS2D,
                                        radius_clip=wl.RADIUS_CLIP,
                                        absgrad=False).image.detach().clone()

        self.data = TrainData(cfg, dev, render)
        # the reference's BinaryTreeGaussianModel holds the parameters and the
        # tree, its strategy module's split() splits them
        btm = ref_stock.load_binary_tree_model("stock")
        self.split = ref_stock.load_strategy_module("stock").split
        self.model = btm.BinaryTreeGaussianModel(device=str(dev), min_scale=wl.SCALE_MIN,
                                                 max_scale=wl.SCALE_MAX,
                                                 scale_eps=TRAIN_SCALE_EPS)
        tree = TreeParams(*wl.make_gaussians(cfg), dev)
        for name in ("means", "quats", "scales", "opacities", "parent", "level", "history_means",
                     "history_scales", "history_quats", "history_opacities", "history_parent",
                     "history_level"):
            setattr(self.model, name, getattr(tree, name))
        self.model.trainable_param_keys = list(TRAIN_KEYS)
        self.opts = self.model.build_optimizers(TRAIN_LRS)
        self.densify = {"grad2d": None, "count": None}
        self.step_no = 0
        self.sizes = []
        warm_split_path(lambda m, o, st, mask: self.split(m, o, st, mask, list(TRAIN_KEYS),
                                                          revised_opacity=True),
                        btm.BinaryTreeGaussianModel, dev)

    def step(self):
        d, S, O, M = self.data, self.S, self.O, self.model
        P = {k: getattr(M, k) for k in TRAIN_KEYS}
        views = d.step_views(self.step_no, 0, 1).to(self.dev)
        rng, ctr = d.step_box(self.step_no, self.dev)
        step_no = self.step_no
        self.step_no += 1
        self.sizes.append(P["means"].shape[0])
        st = S.prepare_explicit_gaussians(P["quats"], P["scales"], P["opacities"],
                                          scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
        res = S.explicit_rasterize(st, P["means"], d.vm[views], d.K[views], img_w=d.det,
                                   img_h=d.det, tile_size=wl.IMG_TILE, eps2d=wl.EPS2D,
                                   radius_clip=wl.RADIUS_CLIP, absgrad=True)
        vox = S.explicit_voxelize(st, P["means"], rng, ctr, dim2=TRAIN_TV, dim1=TRAIN_TV,
                                  dim0=TRAIN_TV, tile_size=wl.VOL_TILE, eps3d=wl.EPS3D,
                                  radius_clip=wl.RADIUS_CLIP)
        out = self.loss(res.image[..., None], d.targets[views][..., None],
                        d.edge[views][..., None], vox.volume)
        out["total"].backward()
        S.explicit_backward(st, P["means"], P["quats"], P["scales"], P["opacities"])
        O.densify_state_update(self.densify, res.means2d.absgrad, res.radii.amax(dim=-1), d.det,
                               d.det, len(views))
        if step_no % TRAIN_SPLIT_EVERY == 0:
            self.split(M, self.opts, self.densify, split_mask(step_no, P["means"].shape[0],
                                                             self.dev),
                       list(TRAIN_KEYS), revised_opacity=True)
        for opt in self.opts.values():
            opt.step()
            opt.zero_grad(set_to_none=True)
        return out["total"]


def run_train_bench(args, cfg, dev, world, rank, local, flush):
    """Config 4: whole-job Gaussian*views/s of the training step (8 views per
    step in total, split over the GPUs: strong scaling)."""
    ref = args.impl == "reference"
    if ref:
        try:
            from oracle.ref_stock import stock_available

            if not stock_available():
                print(json.dumps({"impl": "reference", "unavailable":
                                  "reference install baseline/_ref or build oracle/_ref missing"}))
                return
            trainer = RefTrain(cfg, dev)
        except Exception as exc:
            print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"}))
            return
    else:
        trainer = OursTrain(cfg, world, rank, dev)
    trainer.step_no = first_train_step(args.steps, args.warmup)
    with ClockSampler(local) as clk:
        ms = time_steps(trainer.step, args.steps, args.warmup, 1 if ref else world, flush)
    if rank != 0:
        return
    timed_sizes = trainer.sizes[-args.steps:]
    timed_first = trainer.step_no - args.steps
    splits = [k for k in range(timed_first, trainer.step_no) if k % TRAIN_SPLIT_EVERY == 0]
    value = sum(timed_sizes) * TRAIN_VIEWS_PER_STEP / (args.steps * ms * 1e-3)
    line = {
        "metric": "Gaussian*views/s training step (config 4)",
        "value": round(value, 1), "unit": "Gaussian*views/s", "n_gpus": 1 if ref else world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded teacher projections, random edge masks, r2s_workloads)",
        "config": {"workload": cfg.name, "n_gaussians": cfg.n_gaussians,
                   "views_per_step": TRAIN_VIEWS_PER_STEP, "detector": cfg.detector,
                   "tv_subvolume": TRAIN_TV, "loss": TRAIN_WEIGHTS,
                   "step": "prepare + rasterize + 64^3 voxelize + L1/SSIM/edge/TV losses + "
                           "backward with densify stats + grad all-reduce + binary split "
                           "every 100 steps + Adam",
                   "split": f"{TRAIN_SPLIT_FRAC:.0%} seeded subset every {TRAIN_SPLIT_EVERY} "
                            f"steps (longest axis, revised opacity); timed steps "
                            f"{timed_first}-{trainer.step_no - 1} include split(s) at {splits}",
                   "gaussians_per_timed_step": timed_sizes,
                   "l2": "256MiB flush between steps, outside the timed events"},
        "clocks": clk.summary(),
    }
    if ref:
        line["impl"] = "reference"
        line["e2e"] = {"value": round(value, 1), "unit": "Gaussian*views/s",
                       "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
        line["cpu_baseline"] = {"value": round(value, 1), "unit": "Gaussian*views/s", "cores": 0,
                                "kind": "reference",
                                "sample": "the reference's CUDA build and PyTorch code on GPU 0"}
    else:
        # per step: prepare (2), project_splats, binning (4), raster forward;
        # TV sub-volume: map, 3D binning (4), brick order, row table, voxel
        # forward; losses: projection loss and its gradient, TV and its
        # gradient; backward: raster, voxel, explicit backward with the
        # densification statistics; Adam; plus the split's children kernel
        line["gpu_launches"] = args.steps * 24 + len(splits)
    print(json.dumps(line))


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------
def time_steps(fn, steps, warmup, world, flush):
    """Device time per step: each of the K steps between its own pair of
    CUDA events on the compute stream, the 256 MiB L2 flush before each step
    outside the pair, the K steps bracketed by a barrier and a synchronize."""
    for _ in range(warmup):
        flush.zero_()
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(steps)]
    for a, b in pairs:
        flush.zero_()  # inputs and L2: 256 MiB write between steps
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = sum(a.elapsed_time(b) for a, b in pairs) / steps
    return max_over_ranks(world, ms)


def time_e2e(pipe: HostPipeline, steps, warmup, world, flush):
    """Wall time per step of the end-to-end step, inputs uploaded from and
    outputs downloaded to pinned host memory inside the timed region (the
    pipeline is emptied before it, so the first step's upload is timed and no
    upload past the last step is)."""
    for _ in range(warmup):
        flush.zero_()
        pipe.step_e2e(prefetch_next=False)
        torch.cuda.synchronize()
    pipe.reset_pipeline()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(steps):
        flush.zero_()
        pipe.step_e2e(prefetch_next=i + 1 < steps)
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t0) * 1e3 / steps
    barrier(world)
    return max_over_ranks(world, dt)


def kernel_time(fn, reps=3):
    """Average duration of one launch sequence on the current stream."""
    ts = []
    for _ in range(reps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return sum(ts) / len(ts)


def pipe_peaks(dev):
    """FP32 (FFMA) and MUFU ex2 throughput of this GPU at its current clock,
    from the library's calibration kernels (r2s_calib_ffma_f32 /
    r2s_calib_ex2_f32: 148 x 8 CTAs of 256 threads, 8 independent chains per
    thread), best of three CUDA-event timings."""
    import ctypes

    from r2splat.cuda._backend import _C

    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks = n_sm * 8
    out = torch.empty(blocks * 256, device=dev)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    res = {}
    for name, fn, iters, per in (("ffma", _C.r2s_calib_ffma_f32, 16384, 2.0),
                                 ("ex2", _C.r2s_calib_ex2_f32, 4096, 1.0)):
        def launch():
            rc = fn(ctypes.c_void_p(out.data_ptr()), iters, blocks, st)
            if rc:
                raise RuntimeError(f"calibration {name} failed ({rc})")

        launch()
        best = min(kernel_time(launch, 1) for _ in range(3))
        ops = blocks * 256 * 8 * iters
        res[name] = ops * per / (best * 1e-3)
    return {"fp32_tflops": round(res["ffma"] / 1e12, 2),
            "ex2_per_s": round(res["ex2"], -8), "sm_count": n_sm,
            "how": "r2s_calib_*: 8 CTAs of 256 threads per SM, 8 independent FFMA (2 FLOP) or "
                   "FMUL+ex2.approx chains per thread, best of 3 CUDA-event timings"}


# DRAM traffic of one raster_bwd16_kernel launch per view: the ncu capture of
# `bench.py --views 8` (one kernel, one launch, --set full),
# dram__bytes_read.sum + dram__bytes_write.sum = 530.231 MB + 105.894 MB for 8
# views (traffic grows with the views).
BWD16_DRAM_BYTES_PER_VIEW = (530.231296e6 + 105.893632e6) / 8
# FP32 work per evaluated pixel of raster_bwd16_kernel<true> (absolute
# gradients on), counted from its inner loop: 7 FFMA (the exponent: 2; the row
# moment R1; the two conic products a dx + b dy, b dx + c dy; the two absolute
# sums), 1 FMUL (v e) and 2 FADD (the column and row sums): 10 FP32-pipe
# instructions, 17 FLOP, and 1 MUFU ex2.  The keep test (z >= 0) and the
# cut-off band's running min of |z| run on the ALU pipe and are not counted.
BWD16_FLOP_PER_PAIR = 17
BWD16_FP32_INST_PER_PAIR = 10


def evaluated_pairs(cull: torch.Tensor) -> int:
    """Pixels raster_bwd16_kernel evaluates for the records of one binning:
    16 per walked line, where a record walks the rows or the columns of its
    culled box inside the tile, whichever are fewer (the culling table of the
    forward: c_lo | c_hi << 4 | r_lo << 8 | r_hi << 12)."""
    v = cull.to(torch.int32) & 0xFFFF
    cols = ((v >> 4) & 15) - (v & 15) + 1
    rows = ((v >> 12) & 15) - ((v >> 8) & 15) + 1
    live = (cols > 0) & (rows > 0)
    lines = torch.minimum(cols, rows).clamp_min(0) * live
    return int(lines.sum(dtype=torch.int64).item()) * 16


def dominant_kernel_roofline(proj: OursProjection, hbm_peak, peak_kind, peaks):
    """The raster backward (the largest share of the step) on its own launch.

    It is bound by the SM's FP32 pipe and instruction issue, not by HBM:
    ``achieved`` is the FP32 work on the pixels it evaluates (the walked lines
    of each record's culled box, ``evaluated_pairs``; 17 FLOP each) per second,
    against the FFMA throughput this bench measures on the same GPU
    (``pipe_peaks``).  The reference's pair count (every pixel of every
    record's tile, n_isects x 256) is reported beside it, as are the MUFU ex2
    rate (one ex2 per evaluated pair) and the HBM view: compulsory bytes per
    launch (flatten ids 4 B per record, splat record 32 B and statistics 32 B
    per (view, Gaussian), upstream image 4 B per pixel, offsets 4 B per tile)
    against the measured copy bandwidth, and the DRAM traffic of the ncu
    capture."""
    from r2splat.cuda import _wrapper as W

    E = proj.E
    m, q, s, o = proj.params
    st = E.prepare_explicit_gaussians(q, s, o, scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
    E.explicit_rasterize(st, m, proj.vm, proj.K, img_w=proj.det, img_h=proj.det,
                         tile_size=wl.IMG_TILE, eps2d=wl.EPS2D, radius_clip=wl.RADIUS_CLIP,
                         absgrad=True)
    pb = st.projection.buffers
    C, N = pb.means2d.shape[:2]
    ntx, nty = pb.tile_offsets.size(2), pb.tile_offsets.size(1)
    batches = pb.view_batches or [(0, C, pb.flatten_ids)]
    culls = pb.cull if isinstance(pb.cull, list) else [pb.cull]
    n_isects = sum(ids.numel() for _, _, ids in batches)
    pairs_eval = sum(evaluated_pairs(c) for c in culls)
    stats = torch.empty((C * N, 8), dtype=torch.float32, device=pb.splats.device)

    def launch():
        for (c0, c1, ids), cull in zip(batches, culls):
            W.fused_raster_bwd(pb.splats[c0:c1], pb.tile_offsets[c0:c1], ids, proj.v_img[c0:c1],
                               c1 - c0, N, proj.det, proj.det, wl.IMG_TILE, ntx, nty, True,
                               out=stats[c0 * N:c1 * N], cull=cull)

    launch()
    ms = kernel_time(launch)
    t = ms * 1e-3
    alg_bytes = (n_isects * 4 + C * N * (32 + 32) + C * proj.det * proj.det * 4
                 + C * ntx * nty * 4)
    cfg2_shaped = proj.cfg.name.startswith("cfg2")
    tflops = pairs_eval * BWD16_FLOP_PER_PAIR / t / 1e12
    fp32_peak = peaks["fp32_tflops"]
    lane_ops_peak = fp32_peak * 1e12 / 2  # FFMA lane-instructions per second
    return {
        "kernel": "raster_bwd16_kernel<true>",
        "bound": "fp32",
        "achieved": round(tflops, 2),
        "peak": fp32_peak,
        "unit": "TFLOP/s",
        "frac": round(tflops / fp32_peak, 4),
        "peak_source": "measured in this run (FFMA calibration kernel, same GPU and clock)",
        "traffic": round(BWD16_DRAM_BYTES_PER_VIEW * C) if cfg2_shaped else None,
        "traffic_source": ("ncu capture at 8 views (profiles/raster_bwd16_cfg2_8views.md), "
                           "scaled by views" if cfg2_shaped else "no ncu capture of this "
                           "configuration"),
        "alg_bytes": alg_bytes,
        "launches": len(batches),
        "ms_per_launch": round(ms, 3),
        "n_isects": n_isects,
        "pairs_evaluated": pairs_eval,
        "pairs_reference": n_isects * wl.IMG_TILE * wl.IMG_TILE,
        "flop_per_pair": BWD16_FLOP_PER_PAIR,
        "fp32_pipe": {"inst_per_pair": BWD16_FP32_INST_PER_PAIR,
                      "frac": round(pairs_eval * BWD16_FP32_INST_PER_PAIR / t / lane_ops_peak, 4)},
        "sfu": {"achieved_ex2_per_s": round(pairs_eval / t, -6),
                "peak_ex2_per_s": peaks["ex2_per_s"],
                "frac": round(pairs_eval / t / peaks["ex2_per_s"], 4)},
        "hbm": {"achieved_gbs": round(alg_bytes / t / 1e9, 1), "peak_gbs": hbm_peak,
                "peak_source": peak_kind, "frac": round(alg_bytes / t / 1e9 / hbm_peak, 4)},
    }


def _training_inputs(cfg, dev):
    """Config-sized inputs of the training rows after the backward: the four
    parameter groups with gradients and Adam optimizers (eps 1e-15 and the
    per-group learning rates of the reference's model config), and one step's
    screen-space gradients and radii for the densification statistics."""
    N, C = cfg.n_gaussians, cfg.n_views
    g = torch.Generator(device=dev).manual_seed(300)
    shapes = {"means": (N, 3), "quats": (N, 4), "scales": (N, 3), "opacities": (N,)}
    lrs = {"means": 1.6e-4, "quats": 1e-3, "scales": 5e-3, "opacities": 5e-2}
    params = {k: torch.nn.Parameter(torch.randn(v, generator=g, device=dev)) for k, v in shapes.items()}
    for p in params.values():
        p.grad = torch.randn(p.shape, generator=g, device=dev) * 1e-3
    opts = {k: torch.optim.Adam([{"params": p, "name": k}], lr=lrs[k], eps=1e-15)
            for k, p in params.items()}
    grads2d = torch.rand((C, N, 2), generator=g, device=dev) * 1e-3
    radii = torch.randint(0, 40, (C, N), generator=g, device=dev, dtype=torch.int32)
    return opts, grads2d, radii


def training_rows(cfg, dev, reference: bool, reps: int = 10):
    """Device time of one Adam step over all parameter groups, one step's
    densification statistics and one loss forward+backward (config-sized),
    ours or the reference's PyTorch code (torch.optim.Adam; the strategy's
    _update_state; BinaryTreeLossComputer with torch's default conv settings)."""
    opts, grads2d, radii = _training_inputs(cfg, dev)
    C, N = radii.shape
    state = {"grad2d": None, "count": None, "radii": None}
    g = torch.Generator(device=dev).manual_seed(301)
    det, grid = cfg.detector, 64  # the 64^3 TV sub-volume of the reference trainer
    renders = torch.rand((C, det, det, 1), generator=g, device=dev).requires_grad_(True)
    targets = torch.rand((C, det, det, 1), generator=g, device=dev)
    edge_mask = (torch.rand((C, det, det, 1), generator=g, device=dev) < 0.2).float()
    vol = torch.rand((grid, grid, grid), generator=g, device=dev).requires_grad_(True)
    weights = dict(w_l1=0.8, w_ssim=0.2, w_tv=0.05, w_edge=0.1)
    if reference:
        from oracle import r2s_oracle as O
        from oracle import ref_stock

        computer = ref_stock.load_loss_module().BinaryTreeLossComputer(**weights)

        def adam():
            for o in opts.values():
                o.step()

        def densify():
            O.densify_state_update(state, grads2d, radii, cfg.detector, cfg.detector, C,
                                   track_radii=True)

        def loss():
            renders.grad = vol.grad = None
            computer(renders, targets, edge_mask, vol)["total"].backward()
    else:
        from r2splat.ops import training as T

        def adam():
            T.adam_step(opts)

        info = {"means2d": torch.zeros(1), "radii": radii, "width": cfg.detector,
                "height": cfg.detector, "n_cameras": C}
        info["means2d"].absgrad = grads2d

        def densify():
            T.update_densify_state(state, info, track_radii=True)

        computer = T.FusedBinaryTreeLossComputer(**weights)

        def loss():
            renders.grad = vol.grad = None
            computer(renders, targets, edge_mask, vol)["total"].backward()
    out = {}
    for name, fn in (("adam", adam), ("densify", densify), ("loss_fwd_bwd", loss)):
        fn()
        out[name + "_ms"] = round(kernel_time(fn, reps), 4)
    out["groups"] = ("adam: means [N,3], quats [N,4], scales [N,3], opacities [N]; densify: [C,N] "
                     "pairs; loss: L1+SSIM+edge on [C,H,W] projections + TV on a 64^3 volume")
    return out


def cpu_baseline(cfg, seconds_budget=15.0):
    """Dense PyTorch-on-CPU evaluation of the same formulas (the CPU oracle):
    projection forward + autograd backward of a sample of Gaussians on one
    full-size view; Gaussian*views/s of that sample."""
    from oracle import r2s_oracle as O

    threads = torch.get_num_threads()
    vm, K = wl.make_cameras(1, cfg.detector, total=cfg.n_views)
    n = 256
    while True:
        m, q, s, o = wl.make_gaussians(cfg, n=n)
        params = [t.clone().requires_grad_(True) for t in (m, q, s, o)]
        t0 = time.perf_counter()
        img, *_ = O.projection_forward(*params, vm, K, width=cfg.detector, height=cfg.detector,
                                       tile=wl.IMG_TILE, eps2d=wl.EPS2D, clip=wl.RADIUS_CLIP,
                                       smin=wl.SCALE_MIN, smax=wl.SCALE_MAX, chunk=64)
        img.backward(torch.ones_like(img))
        dt = time.perf_counter() - t0
        if dt * 2.2 > seconds_budget or n >= 16384:
            break
        n *= 2
    return {"value": round(n / dt, 1), "unit": "Gaussian*views/s", "cores": threads,
            "kind": "port",
            "sample": f"{n} Gaussians of {cfg.name} distributions x 1 view at {cfg.detector}^2, "
                      f"dense over all pixels with tile-membership mask, fwd+autograd bwd, "
                      f"{dt:.1f} s"}


def run_reference(args, cfg, dev, local, flush):
    try:
        from oracle.ref_stock import stock_available

        if not stock_available():
            print(json.dumps({"impl": "reference", "unavailable":
                              "reference install baseline/_ref or build oracle/_ref missing"}))
            return
        proj = RefProjection(cfg, dev)
        vox = RefVoxel(cfg, dev, proj)
    except Exception as exc:  # the reference cannot be loaded
        print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"}))
        return
    with ClockSampler(local) as clk:
        ms = time_steps(proj.step, args.steps, args.warmup, 1, flush)
        vms = time_steps(vox.step, args.steps, args.warmup, 1, flush)
    del proj, vox
    torch.cuda.empty_cache()
    train = training_rows(cfg, dev, reference=True)
    value = cfg.n_gaussians * cfg.n_views / (ms * 1e-3)
    line = {
        "metric": "Gaussian*views/s projection fwd+bwd (and Mvoxels/s voxelize fwd+bwd)",
        "impl": "reference", "value": round(value, 1), "unit": "Gaussian*views/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, r2s_workloads)",
        "config": job_config(cfg, cfg.n_views),
        "voxelize": {"value": round(cfg.grid ** 3 / (vms * 1e-3) / 1e6, 2),
                     "unit": "Mvoxels/s", "ms_per_step": round(vms, 3)},
        "cpu_baseline": {"value": round(value, 1), "unit": "Gaussian*views/s", "cores": 0,
                         "kind": "reference",
                         "sample": "the reference's op layer over its CUDA build (it ships no "
                                   "CPU implementation), full workload on GPU 0"},
        "e2e": {"value": round(value, 1), "unit": "Gaussian*views/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "implementation": "reference r2splat.ops (baseline/_ref, unchanged) over its CUDA "
                          "sources built for sm_100a (oracle/_ref)",
        "training": train,
        "clocks": clk.summary(),
    }
    print(json.dumps(line))


def run_rank_shares(args, cfg, dev, flush):
    """Each rank's share of an N-GPU strong-scaling job, timed in turn on one
    GPU: the projection with the rank's views (view r, r + N, ...), the voxel
    step with the rank's z-slab (the same split the N-GPU run computes), each
    a step object of the N-GPU run with its gradient all-reduce left out.
    The largest rank time against the one-GPU time / N bounds the N-GPU
    efficiency before the all-reduce; the phases name what limits it."""
    n = args.rank_shares
    if n < 1:
        raise SystemExit("--rank-shares needs N >= 1")
    ranks = []
    with ClockSampler(0) as clk:
        for world, rank in [(1, 0)] + [(n, r) for r in range(n)]:
            proj = OursProjection(cfg, world, rank, dev, "strong")
            proj.world = 1  # no collective: one process
            ms = time_steps(proj.step, args.steps, args.warmup, 1, flush)
            proj.phases()
            pph = proj.phases()
            views = proj.views
            del proj
            torch.cuda.empty_cache()
            vox = OursVoxel(cfg, world, rank, dev, wl.make_gaussians(cfg))
            vox.world = 1
            vms = time_steps(vox.step, args.steps, args.warmup, 1, flush)
            vox.phases()
            vph = vox.phases()
            del vox
            torch.cuda.empty_cache()
            ranks.append({"world": world, "rank": rank, "views": views,
                          "projection_ms": round(ms, 3), "voxel_ms": round(vms, 3),
                          "layers": vph["layers"], "records": vph["records"],
                          "projection_phases": pph["ms"], "voxel_phases": vph["ms"]})
    one, shares = ranks[0], ranks[1:]
    p_max = max(r["projection_ms"] for r in shares)
    v_max = max(r["voxel_ms"] for r in shares)
    print(json.dumps({
        "mode": f"rank shares of a {n}-GPU strong-scaling job, timed in turn on one GPU",
        "config": job_config(cfg, cfg.n_views), "steps": args.steps, "warmup": args.warmup,
        "projection": {"one_gpu_ms": one["projection_ms"], "largest_share_ms": p_max,
                       "efficiency_before_allreduce": round(one["projection_ms"] / n / p_max, 4)},
        "voxelize": {"one_gpu_ms": one["voxel_ms"], "largest_share_ms": v_max,
                     "efficiency_before_allreduce": round(one["voxel_ms"] / n / v_max, 4)},
        "ranks": ranks, "clocks": clk.summary()}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--scaling", choices=("strong", "weak"), default="strong",
                    help="strong: the job's views split over the GPUs; weak: every GPU "
                         "renders the config's views of a larger orbit")
    ap.add_argument("--views", type=int, default=None,
                    help="override the job's views (small profiling cases)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rank-shares", type=int, default=None, metavar="N",
                    help="one GPU: time each rank's share of an N-GPU strong-scaling job "
                         "in turn (no collective) and print the per-rank step times")
    args = ap.parse_args()
    if args.impl == "reference" and int(os.environ.get("RANK", "0")) != 0:
        return  # the reference arm runs on rank 0 only
    if args.impl == "reference":
        os.environ["WORLD_SIZE"] = "1"
    world, rank, local = init_dist()
    dev = torch.device("cuda", local)
    cfg = wl.CONFIGS[args.config]
    if args.views is not None:
        import dataclasses

        cfg = dataclasses.replace(cfg, n_views=args.views,
                                  name=f"{cfg.name}-views{args.views}")
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    hbm_peak, peak_kind = _peaks()
    if args.config == 4:
        run_train_bench(args, cfg, dev, world, rank, local, flush)
        return
    if args.rank_shares is not None:
        if world != 1 or args.impl != "ours":
            raise SystemExit("--rank-shares runs this build on one GPU")
        run_rank_shares(args, cfg, dev, flush)
        return
    if args.impl == "reference":
        run_reference(args, cfg, dev, local, flush)
        return

    proj = OursProjection(cfg, world, rank, dev, args.scaling)
    job_views = cfg.n_views * (world if args.scaling == "weak" else 1)
    with ClockSampler(local) as clk:
        ms = time_steps(proj.step, args.steps, args.warmup, world, flush)
        e2e_ms = time_e2e(proj, args.steps, max(1, args.warmup // 2), world, flush)
        peaks = pipe_peaks(dev)
        roof = (dominant_kernel_roofline(proj, hbm_peak, peak_kind, peaks)
                if rank == 0 else None)
        proj.phases()  # the first call sizes the allocator's blocks for these calls
        proj_phases = proj.phases()
        h2d, d2h = proj.bytes_e2e()
        del proj
        torch.cuda.empty_cache()
        vox = OursVoxel(cfg, world, rank, dev, wl.make_gaussians(cfg))
        vms = time_steps(vox.step, args.steps, args.warmup, world, flush)
        v_e2e_ms = time_e2e(vox, args.steps, max(1, args.warmup // 2), world, flush)
        vox.phases()
        vox_phases = vox.phases()
        vh2d, vd2h = vox.bytes_e2e()
    del vox
    torch.cuda.empty_cache()
    phases = {"projection": proj_phases, "voxelize": vox_phases}
    if world > 1:
        import torch.distributed as dist

        gathered = [None] * world
        dist.all_gather_object(gathered, phases)
        phases = {"per_rank": gathered}
    train = training_rows(cfg, dev, reference=False) if rank == 0 else None
    value = cfg.n_gaussians * job_views / (ms * 1e-3)
    e2e_value = cfg.n_gaussians * job_views / (e2e_ms * 1e-3)
    vox_value = cfg.grid ** 3 / (vms * 1e-3) / 1e6
    barrier(world)
    # our kernels per timed step: projection = prepare (covariances, then the
    # softplus opacities), project_splats, binning (count, column scan, scan,
    # place), raster forward, raster backward, explicit backward (binning to
    # raster backward once per view batch; with several batches, the first
    # binning's count, column scan and scan also run once for all views, as
    # the op layer first tries one binning); voxel =
    # prepare (two), map, binning (count, column scan, scan, place), brick
    # order, row table, voxel forward, voxel backward, explicit backward (the
    # zero-view projection pass launches nothing)
    n_batches = proj_phases["view_batches"]
    gpu_launches = args.steps * (4 + 6 * n_batches + (3 if n_batches > 1 else 0))
    vox_launches = args.steps * 12
    if rank != 0:
        return
    line = {
        "metric": "Gaussian*views/s projection fwd+bwd (and Mvoxels/s voxelize fwd+bwd)",
        "value": round(value, 1), "unit": "Gaussian*views/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, r2s_workloads)",
        "config": job_config(cfg, job_views),
        "parallelism": (f"{job_views} views dealt over {world} GPU(s) + NCCL gradient all-reduce; "
                        f"voxel grid in {world} balanced z-slab(s)"),
        "voxelize": {"value": round(vox_value, 2), "unit": "Mvoxels/s",
                     "ms_per_step": round(vms, 3), "scaling": "strong (z-slabs)",
                     "gpu_launches": vox_launches,
                     "e2e": {"value": round(cfg.grid ** 3 / (v_e2e_ms * 1e-3) / 1e6, 2),
                             "unit": "Mvoxels/s", "h2d_bytes_per_step": vh2d,
                             "d2h_bytes_per_step": vd2h, "ms_per_step": round(v_e2e_ms, 3)}},
        "e2e": {"value": round(e2e_value, 1), "unit": "Gaussian*views/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 3)},
        "roofline": roof,
        "pipe_peaks": peaks,
        "phases": phases,
        "training": train,
        "gpu_launches": gpu_launches,
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg)
    print(json.dumps(line))


def shutdown():
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    try:
        main()
    finally:
        shutdown()
