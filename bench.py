"""Benchmark of the r2splat hot path on B200: projection fwd+bwd and voxelization fwd+bwd.

Metric: Gaussian*views/s of projection forward+backward
(``value``) and Mvoxels/s of voxelization forward+backward (``voxelize``), on
benchmark config 2 by default: 500,000 Gaussians, 75 views over 360 degrees,
512x512 detector, 256^3 grid (seeded synthetic inputs, r2s_workloads.py).

One step of the projection path is the reference's explicit training step
without the loss: prepare (parameter transform + softplus), explicit
rasterize (projection, binning, rasterizer), then explicit backward with a
seeded N(0,1) upstream image gradient, all through ``r2splat.ops``.  One
voxel step is prepare, voxelize of the grid and the voxel VJP chain down to
the raw parameters.

Multi-GPU (torchrun, one process per GPU): every rank renders its own 75
views of a 75*N-view orbit of the same Gaussians (weak scaling) and the
per-Gaussian gradients are summed with one NCCL all-reduce per step; the
voxel grid is split into N z-slabs (strong scaling of that secondary
metric).  ``value`` is the whole job: N*75*500k Gaussian*views / max-over-
ranks step time.

``--impl reference`` times the reference implementation of the path -- the
reference's own CUDA sources built for sm_100a (``oracle/_ref``) driven in
the reference op layer's call order -- on rank 0 with the same workload.
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


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------
class OursProjection:
    def __init__(self, cfg, world, rank, dev):
        from r2splat.ops import explicit as E

        self.E = E
        self.world = world
        self.cfg = cfg
        self.det = cfg.detector
        m, q, s, o = wl.make_gaussians(cfg)
        self.host = [t.pin_memory() for t in (m, q, s, o)]
        self.params = [t.to(dev) for t in (m, q, s, o)]
        first, count, total, stride = shard.view_shard(cfg.n_views, rank, world)
        vm, K = wl.make_cameras(count, cfg.detector, first=first, count=count, total=total,
                                stride=stride)
        self.vm, self.K = vm.to(dev), K.to(dev)
        self.host_cams = (vm.pin_memory(), K.pin_memory())
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        self.v_img = torch.randn((cfg.n_views, self.det, self.det), generator=g, device=dev)
        self.host_vimg = self.v_img.cpu().pin_memory()
        self.allreduce = shard.GradientAllReduce()

    def step(self, params=None, vm=None, K=None, v_img=None):
        E = self.E
        params = self.params if params is None else params
        vm = self.vm if vm is None else vm
        K = self.K if K is None else K
        v_img = self.v_img if v_img is None else v_img
        for p in params:
            p.grad = None
            p.requires_grad_(True)
        st = E.prepare_explicit_gaussians(params[1], params[2], params[3],
                                          scale_min=wl.SCALE_MIN, scale_max=wl.SCALE_MAX)
        res = E.explicit_rasterize(st, params[0], vm, K, img_w=self.det, img_h=self.det,
                                   tile_size=wl.IMG_TILE, eps2d=wl.EPS2D,
                                   radius_clip=wl.RADIUS_CLIP, absgrad=True)
        res.image.grad = v_img
        E.explicit_backward(st, *params)
        if self.world > 1:
            self.allreduce([p.grad for p in params])
        return res

    def _upload(self):
        """H2D of one step's inputs (raw parameters, cameras, upstream image
        gradient) on the copy stream; returns the device tensors and an event."""
        dev = self.params[0].device
        with torch.cuda.stream(self.copy_stream):
            ins = [h.to(dev, non_blocking=True) for h in self.host]
            ins += [c.to(dev, non_blocking=True) for c in self.host_cams]
            ins.append(self.host_vimg.to(dev, non_blocking=True))
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
        return ins, ev

    def reset_pipeline(self):
        self.copy_stream = torch.cuda.Stream(device=self.params[0].device)
        self.prefetched = None

    def step_e2e(self, prefetch_next=True):
        """Same step with host-resident inputs and outputs: H2D of the raw
        parameters, cameras and upstream image gradient, D2H of the four
        parameter gradients.  The copies run on a copy stream: the next step's
        inputs upload while this step computes (a double-buffered input
        pipeline) and the gradients download behind the next step; every copy
        of a timed step happens inside the timed region."""
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
        params, (vm, K, v_img) = ins[:4], ins[4:]
        self.step(params, vm, K, v_img)
        done = torch.cuda.Event()
        done.record(compute)
        self.copy_stream.wait_event(done)
        with torch.cuda.stream(self.copy_stream):
            outs = [p.grad.to("cpu", non_blocking=True) for p in params]
            for p in params:
                p.grad.record_stream(self.copy_stream)
        return outs

    def bytes_e2e(self):
        h2d = sum(t.numel() * t.element_size() for t in self.host) + sum(
            t.numel() * t.element_size() for t in self.host_cams) + self.host_vimg.numel() * 4
        d2h = sum(t.numel() * t.element_size() for t in self.host)
        return h2d, d2h


class OursVoxel:
    def __init__(self, cfg, world, rank, dev, params):
        from r2splat.cuda import _wrapper as W

        self.W = W
        self.world = world
        self.G = cfg.grid
        self.nt = (self.G + wl.VOL_TILE - 1) // wl.VOL_TILE
        self.params = params
        rng, ctr = wl.unit_cube_box()
        self.rng, self.ctr = rng.to(dev), ctr.to(dev)
        # z-slabs balanced by records per brick layer (every rank computes the
        # same ranges from the same mapping)
        with torch.no_grad():
            m, q, s, o = params
            cov, _, op = W.fused_prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
            rects = W.fused_map(m, cov, op, self.rng, self.ctr, self.G, self.G, self.G,
                                wl.VOL_TILE, self.nt, self.nt, self.nt, wl.EPS3D,
                                wl.RADIUS_CLIP)[4]
        self.l0, self.l1 = shard.balanced_layer_ranges(shard.layer_weights(rects, self.nt),
                                                       world)[rank]
        z0, z1 = shard.slab_rows(self.l0, self.l1, wl.VOL_TILE, self.G)
        g = torch.Generator(device=dev).manual_seed(200 + rank)
        self.v_vol = torch.randn((z1 - z0, self.G, self.G), generator=g, device=dev)
        self.allreduce = shard.GradientAllReduce()

    def step(self):
        W = self.W
        m, q, s, o = self.params
        G, nt = self.G, self.nt
        with torch.no_grad():
            cov, ms, op = W.fused_prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
            m3, c3, r3, vs, rects, _ = W.fused_map(m, cov, op, self.rng, self.ctr, G, G, G,
                                                   wl.VOL_TILE, nt, nt, nt, wl.EPS3D,
                                                   wl.RADIUS_CLIP)
            S = self.l1 - self.l0
            offs, fids, _ = W.fused_bin(rects, S, m.size(0), nt * nt, nt, 1, segment_base=self.l0)
            rows = W.fused_voxel_rows(vs, offs, fids, m.size(0), G, G, G, wl.VOL_TILE, nt, nt, nt,
                                      self.l0, self.l1)
            vol = W.fused_voxel_fwd(vs, offs, fids, m.size(0), G, G, G, wl.VOL_TILE, nt, nt, nt,
                                    self.l0, self.l1, rows=rows)
            stats = W.fused_voxel_bwd(vs, offs, fids, self.v_vol, m.size(0), G, G, G,
                                      wl.VOL_TILE, nt, nt, nt, self.l0, self.l1, rows=rows)
            outs = [torch.empty_like(t) for t in (m, q, s, o)]
            W.fused_explicit_backward(m, q, s, o, wl.SCALE_MIN, wl.SCALE_MAX, None, None, 0, 0,
                                      wl.EPS2D, None, None, None, self.rng, self.ctr, G, G, G,
                                      wl.EPS3D, stats, False, outs)
            if self.world > 1:
                self.allreduce(outs)
        return vol


# ---------------------------------------------------------------------------
# reference implementation (the reference's CUDA build, reference call order)
# ---------------------------------------------------------------------------
class RefProjection:
    def __init__(self, cfg, dev):
        from oracle.ref_harness import ReferencePipeline

        self.ref = ReferencePipeline()
        self.cfg = cfg
        self.det = cfg.detector
        m, q, s, o = wl.make_gaussians(cfg)
        self.params = [t.to(dev) for t in (m, q, s, o)]
        vm, K = wl.make_cameras(cfg.n_views, cfg.detector)
        self.vm, self.K = vm.to(dev), K.to(dev)
        g = torch.Generator(device=dev).manual_seed(100)
        self.v_img = torch.randn((cfg.n_views, self.det, self.det), generator=g, device=dev)

    # the reference's int32 tile offsets overflow past 2^31 records (config 3):
    # there it runs in batches of 20 views, as its users must

    def step(self):
        m, q, s, o = self.params
        cov, ms, op = self.ref.prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
        C = self.vm.shape[0]
        per = 20 if self.cfg.name.startswith("cfg3") else C
        for c0 in range(0, C, per):
            c1 = min(C, c0 + per)
            p = self.ref.rasterize_forward(m, cov, op, self.vm[c0:c1], self.K[c0:c1], self.det,
                                           self.det, wl.IMG_TILE, wl.EPS2D, wl.RADIUS_CLIP)
            self.ref.explicit_backward(p, self.v_img[c0:c1], None, None, m, q, s, o, cov, op,
                                       wl.SCALE_MIN, wl.SCALE_MAX, absgrad=True)
        return p


class RefVoxel:
    def __init__(self, cfg, dev, proj: RefProjection):
        self.ref = proj.ref
        self.params = proj.params
        self.G = cfg.grid
        rng, ctr = wl.unit_cube_box()
        self.rng, self.ctr = rng.to(dev), ctr.to(dev)
        g = torch.Generator(device=dev).manual_seed(200)
        self.v_vol = torch.randn((self.G,) * 3, generator=g, device=dev)

    def step(self):
        m, q, s, o = self.params
        G = self.G
        cov, ms, op = self.ref.prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
        v = self.ref.voxelize_forward(m, cov, ms, op, self.rng, self.ctr, G, G, G, wl.VOL_TILE,
                                      wl.EPS3D, wl.RADIUS_CLIP)
        self.ref.explicit_backward(None, None, v, self.v_vol, m, q, s, o, cov, op, wl.SCALE_MIN,
                                   wl.SCALE_MAX)
        return v


# ---------------------------------------------------------------------------
# config 4: the training step (projection + TV sub-volume + losses + Adam)
# ---------------------------------------------------------------------------
TRAIN_VIEWS_PER_STEP = 8
TRAIN_POOL = 32          # orbit views with seeded synthetic targets
TRAIN_TV = 64            # edge of the random TV sub-volume (voxels)
TRAIN_GRID = 256         # full-grid resolution that fixes the sub-volume's voxel size
TRAIN_WEIGHTS = dict(w_l1=0.8, w_ssim=0.2, w_tv=0.05, w_edge=0.1)
TRAIN_LRS = {"means": 1.6e-4, "quats": 1e-3, "scales": 5e-3, "opacities": 5e-2}


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
        m, q, s, o = wl.make_gaussians(cfg)
        self.params = {k: torch.nn.Parameter(t.to(dev)) for k, t in
                       zip(("means", "quats", "scales", "opacities"), (m, q, s, o))}
        self.opts = {k: torch.optim.Adam([{"params": p, "name": k}], lr=TRAIN_LRS[k], eps=1e-15)
                     for k, p in self.params.items()}
        self.loss = T.FusedBinaryTreeLossComputer(**TRAIN_WEIGHTS)
        self.densify = {"grad2d": None, "count": None}
        self.allreduce = shard.GradientAllReduce()
        self.step_no = 0

    def step(self):
        E, T, d, P = self.E, self.T, self.data, self.params
        views = d.step_views(self.step_no, self.rank, self.world).to(self.dev)
        rng, ctr = d.step_box(self.step_no, self.dev)
        self.step_no += 1
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
        T.adam_step(self.opts)
        for o in self.opts.values():
            o.zero_grad(set_to_none=True)
        return out["total"]


class RefTrain:
    """The same step through the reference's kernels (oracle/_ref in its op
    layer's order) and its PyTorch code: BinaryTreeLossComputer with autograd,
    the strategy's _update_state, torch.optim.Adam."""

    def __init__(self, cfg, dev):
        from oracle import r2s_oracle as O
        from oracle.ref_harness import ReferencePipeline

        self.O, self.ref, self.cfg, self.dev = O, ReferencePipeline(), cfg, dev
        tm, tq, ts, to = (t.to(dev) for t in _teacher(cfg))

        def render(vm, K):
            cov, ms, op = self.ref.prepare(tq, ts, to, wl.SCALE_MIN, wl.SCALE_MAX)
            return self.ref.rasterize_forward(tm, cov, op, vm, K, cfg.detector, cfg.detector,
                                              wl.IMG_TILE, wl.EPS2D, wl.RADIUS_CLIP)["output"]

        self.data = TrainData(cfg, dev, render)
        m, q, s, o = wl.make_gaussians(cfg)
        self.params = {k: torch.nn.Parameter(t.to(dev)) for k, t in
                       zip(("means", "quats", "scales", "opacities"), (m, q, s, o))}
        self.opts = {k: torch.optim.Adam([{"params": p, "name": k}], lr=TRAIN_LRS[k], eps=1e-15)
                     for k, p in self.params.items()}
        self.densify = {"grad2d": None, "count": None}
        self.step_no = 0

    def step(self):
        d, P, R, O = self.data, self.params, self.ref, self.O
        views = d.step_views(self.step_no, 0, 1).to(self.dev)
        rng, ctr = d.step_box(self.step_no, self.dev)
        self.step_no += 1
        m, q, s, o = (P[k].detach() for k in ("means", "quats", "scales", "opacities"))
        cov, ms, op = R.prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
        p = R.rasterize_forward(m, cov, op, d.vm[views], d.K[views], d.det, d.det, wl.IMG_TILE,
                                wl.EPS2D, wl.RADIUS_CLIP)
        v = R.voxelize_forward(m, cov, ms, op, rng, ctr, TRAIN_TV, TRAIN_TV, TRAIN_TV,
                               wl.VOL_TILE, wl.EPS3D, wl.RADIUS_CLIP)
        image = p["output"].detach().requires_grad_(True)
        volume = v["output"].detach().requires_grad_(True)
        out = O.binary_tree_losses(image[..., None], d.targets[views][..., None],
                                   d.edge[views][..., None], volume, **TRAIN_WEIGHTS)
        out["total"].backward()
        g = R.explicit_backward(p, image.grad, v, volume.grad, m, q, s, o, cov, op,
                                wl.SCALE_MIN, wl.SCALE_MAX, absgrad=True)
        for k, gk in (("means", "means"), ("quats", "quats"), ("scales", "scales"),
                      ("opacities", "opacities")):
            P[k].grad = g[gk]
        O.densify_state_update(self.densify, g["means2d_abs"], p["radii"].amax(dim=-1), d.det,
                               d.det, len(views))
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
            from oracle.ref_harness import reference_available

            if not reference_available():
                print(json.dumps({"impl": "reference", "unavailable":
                                  "reference sm_100a build oracle/_ref missing"}))
                return
            trainer = RefTrain(cfg, dev)
        except Exception as exc:
            print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"}))
            return
    else:
        trainer = OursTrain(cfg, world, rank, dev)
    with ClockSampler(local) as clk:
        ms = time_steps(trainer.step, args.steps, args.warmup, 1 if ref else world, flush)
    if rank != 0:
        return
    value = cfg.n_gaussians * TRAIN_VIEWS_PER_STEP / (ms * 1e-3)
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
                           "backward with fused densify stats + grad all-reduce + Adam",
                   "split": "binary split every 100 steps lies outside the timed window",
                   "l2": "256MiB flush between steps"},
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
        line["gpu_launches"] = args.steps * 21
    print(json.dumps(line))


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------
def time_steps(fn, steps, warmup, world, flush):
    for _ in range(warmup):
        flush.zero_()
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        flush.zero_()  # inputs and L2: 256 MiB write between steps
        fn()
    b.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = a.elapsed_time(b) / steps
    return max_over_ranks(world, ms)


def time_e2e(proj, steps, warmup, world, flush):
    """Wall time per step of the end-to-end step, inputs uploaded from and
    gradients downloaded to pinned host memory inside the timed region (the
    pipeline is emptied before it, so the first step's upload is timed and no
    upload past the last step is)."""
    for _ in range(warmup):
        flush.zero_()
        proj.step_e2e(prefetch_next=False)
        torch.cuda.synchronize()
    proj.reset_pipeline()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(steps):
        flush.zero_()
        proj.step_e2e(prefetch_next=i + 1 < steps)
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


# DRAM traffic of one raster_bwd16_kernel launch per view, from the ncu
# capture of `bench.py --views 8` (dram__bytes_read.sum + dram__bytes_write.sum
# = 441.2 MB + 103.9 MB for 8 views; traffic grows with the views).
BWD16_DRAM_BYTES_PER_VIEW = (441.213952e6 + 103.907328e6) / 8


def dominant_kernel_roofline(proj: OursProjection, hbm_peak, peak_kind, clock_mhz):
    """Raster backward (the largest share of the step) on its own launch.

    Algorithmic (compulsory) bytes per launch: the flatten ids (4 B per
    intersection record), every (view, Gaussian) splat record once (32 B) and
    its statistics once (32 B), the upstream image (4 B per pixel) and the
    tile offsets (4 B per tile).  The kernel is bound by the SM pipes, not by
    HBM.  `sfu` and `fp32` count the algorithmic pairs P2 = n_isects x
    tile_size^2 (the reference evaluates every pixel of a record's tile, one
    exponential and 30 FP32 flops each) against 16 ex2 per clock per SM at
    the sampled SM clock and against the nominal FP32 peak.  The kernel
    itself evaluates fewer pairs (only the rows or columns a record's
    ellipse reaches inside the tile), so these fractions can exceed 1."""
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
    stats = torch.empty((C * N, 8), dtype=torch.float32, device=pb.splats.device)

    def launch():
        for (c0, c1, ids), cull in zip(batches, culls):
            W.fused_raster_bwd(pb.splats[c0:c1], pb.tile_offsets[c0:c1], ids, proj.v_img[c0:c1],
                               c1 - c0, N, proj.det, proj.det, wl.IMG_TILE, ntx, nty, True,
                               out=stats[c0 * N:c1 * N], cull=cull)

    launch()
    ms = kernel_time(launch)
    alg_bytes = (n_isects * 4 + C * N * (32 + 32) + C * proj.det * proj.det * 4
                 + C * ntx * nty * 4)
    cfg2_shaped = proj.cfg.name.startswith("cfg2")
    achieved = alg_bytes / (ms * 1e-3) / 1e9
    pairs = n_isects * wl.IMG_TILE * wl.IMG_TILE
    mhz = clock_mhz or 1965.0
    sfu_peak = 148 * 16 * mhz * 1e6
    fp32_peak = 148 * 128 * 2 * mhz * 1e6 / 1e12
    tflops = pairs * 30 / (ms * 1e-3) / 1e12
    return {
        "kernel": "raster_bwd16_kernel<true>",
        "bound": "hbm",
        "achieved": round(achieved, 1),
        "peak": hbm_peak,
        "unit": "GB/s",
        "frac": round(achieved / hbm_peak, 4),
        "peak_source": peak_kind,
        "traffic": round(BWD16_DRAM_BYTES_PER_VIEW * C) if cfg2_shaped else None,
        "alg_bytes": alg_bytes,
        "traffic_source": ("ncu capture at 8 views, scaled by views" if cfg2_shaped
                           else "no ncu capture of this configuration"),
        "launches": len(batches),
        "ms_per_launch": round(ms, 3),
        "n_isects": n_isects,
        "sfu": {"achieved_ex2_per_s": round(pairs / (ms * 1e-3), -6),
                "peak_ex2_per_s": round(sfu_peak, -6), "frac": round(pairs / (ms * 1e-3) / sfu_peak, 4),
                "pairs": pairs, "pairs_basis": "algorithmic n_isects x 256; the kernel culls",
                "clock_mhz": mhz},
        "fp32": {"achieved_tflops": round(tflops, 2), "peak_tflops_nominal": round(fp32_peak, 1),
                 "frac": round(tflops / fp32_peak, 4), "flops_per_pair": 30},
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

        def adam():
            for o in opts.values():
                o.step()

        def densify():
            O.densify_state_update(state, grads2d, radii, cfg.detector, cfg.detector, C,
                                   track_radii=True)

        def loss():
            renders.grad = vol.grad = None
            O.binary_tree_losses(renders, targets, edge_mask, vol, **weights)["total"].backward()
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
            "sample": f"{n} Gaussians of config-{2} distributions x 1 view at {cfg.detector}^2, "
                      f"dense over all pixels with tile-membership mask, fwd+autograd bwd, "
                      f"{dt:.1f} s"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--views", type=int, default=None,
                    help="override the views per GPU (small profiling cases)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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

    if args.impl == "reference":
        try:
            from oracle.ref_harness import reference_available

            if not reference_available():
                print(json.dumps({"impl": "reference", "unavailable":
                                  "reference sm_100a build oracle/_ref missing"}))
                return
            proj = RefProjection(cfg, dev)
            vox = RefVoxel(cfg, dev, proj)
        except Exception as exc:  # reference build cannot be loaded
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
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, r2s_workloads)",
            "config": {"workload": cfg.name, "n_gaussians": cfg.n_gaussians,
                       "views": cfg.n_views, "detector": cfg.detector, "grid": cfg.grid,
                       "l2": "256MiB flush between steps"},
            "voxelize": {"value": round(cfg.grid ** 3 / (vms * 1e-3) / 1e6, 2),
                         "unit": "Mvoxels/s", "ms_per_step": round(vms, 3)},
            "cpu_baseline": {"value": round(value, 1), "unit": "Gaussian*views/s", "cores": 0,
                             "kind": "reference",
                             "sample": "the reference's CUDA build (it ships no CPU "
                                       "implementation), full workload on GPU 0"},
            "e2e": {"value": round(value, 1), "unit": "Gaussian*views/s",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "training": train,
            "clocks": clk.summary(),
        }
        print(json.dumps(line))
        return

    proj = OursProjection(cfg, world, rank, dev)
    with ClockSampler(local) as clk:
        ms = time_steps(proj.step, args.steps, args.warmup, world, flush)
        e2e_ms = time_e2e(proj, args.steps, max(1, args.warmup // 2), world, flush)
        roof = dominant_kernel_roofline(proj, hbm_peak, peak_kind, clk.summary()["sm_mhz"]) \
            if rank == 0 else None
        vox = OursVoxel(cfg, world, rank, dev, proj.params)
        torch.cuda.empty_cache()
        vms = time_steps(vox.step, args.steps, args.warmup, world, flush)
    del vox
    torch.cuda.empty_cache()
    train = training_rows(cfg, dev, reference=False) if rank == 0 else None
    value = world * cfg.n_gaussians * cfg.n_views / (ms * 1e-3)
    e2e_value = world * cfg.n_gaussians * cfg.n_views / (e2e_ms * 1e-3)
    h2d, d2h = proj.bytes_e2e()
    barrier(world)
    # our kernels per timed step: projection = prepare, project_splats, binning
    # (count, column scan, scan, place), raster forward, raster backward,
    # explicit backward; voxel = prepare, map, binning (4), row table, voxel
    # forward, voxel backward, explicit backward
    gpu_launches = args.steps * 9
    vox_launches = args.steps * 10
    if rank != 0:
        return
    line = {
        "metric": "Gaussian*views/s projection fwd+bwd (and Mvoxels/s voxelize fwd+bwd)",
        "value": round(value, 1), "unit": "Gaussian*views/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, r2s_workloads)",
        "config": {"workload": cfg.name, "n_gaussians": cfg.n_gaussians,
                   "views_per_gpu": cfg.n_views, "detector": cfg.detector, "grid": cfg.grid,
                   "parallelism": f"views x{world} (weak) + grad all-reduce; voxel z-slabs x{world}",
                   "l2": "256MiB flush between steps"},
        "voxelize": {"value": round(cfg.grid ** 3 / (vms * 1e-3) / 1e6, 2), "unit": "Mvoxels/s",
                     "ms_per_step": round(vms, 3), "scaling": "strong (z-slabs)",
                     "gpu_launches": vox_launches},
        "e2e": {"value": round(e2e_value, 1), "unit": "Gaussian*views/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 3)},
        "roofline": roof,
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
