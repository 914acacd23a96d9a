"""Multi-process sharding of the path on CPU (gloo, world size 2): views per
rank with a gradient all-reduce equal the single-process gradient over all
views; the z-slabs of the voxel grid tile the full volume and their gradient
sum equals the full gradient.  The per-rank compute is the CPU oracle; the
sharding and the collective are the ones bench.py runs over NCCL."""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

from _helpers import ROOT

WORLD = 2
VIEWS_PER_RANK = 2
STRONG_VIEWS = 3  # an odd job: ranks hold 2 and 1 views
DET = 32
GRID = 32
TILE3 = 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_paths():
    for p in (os.path.join(ROOT, "bt-3dgs_b200"), ROOT):
        if p not in sys.path:
            sys.path.insert(0, p)


def _params():
    import r2s_workloads as wl

    m, q, s, o = wl.make_gaussians(wl.CONFIGS[0], n=48)
    return [t.double().requires_grad_(True) for t in (m, q, s, o)]


def _projection_grads(params, first, count, total, stride=1):
    import r2s_workloads as wl
    from oracle import r2s_oracle as O

    vm, K = wl.make_cameras(count, DET, first=first, count=count, total=total, stride=stride)
    img, *_ = O.projection_forward(*params, vm.double(), K.double(), width=DET, height=DET,
                                   tile=wl.IMG_TILE, eps2d=wl.EPS2D, clip=wl.RADIUS_CLIP,
                                   smin=wl.SCALE_MIN, smax=wl.SCALE_MAX)
    g = torch.Generator().manual_seed(5)
    v = torch.randn((total, DET, DET), generator=g, dtype=torch.float64)[first::stride][:count]
    return torch.autograd.grad((img * v).sum(), params)


def _voxel_slab(params, l0, l1):
    import r2s_workloads as wl
    from oracle import r2s_oracle as O

    m, q, s, o = params
    cov, _ = O.parameter_transform(q, s, wl.SCALE_MIN, wl.SCALE_MAX)
    opac = O.softplus(o)
    rng, ctr = wl.unit_cube_box()
    m3, c3, r3 = O.volume_mapping(m, cov, rng.double(), ctr.double(), GRID, GRID, GRID, wl.EPS3D,
                                  wl.RADIUS_CLIP)
    nt = GRID // TILE3
    rects, valid, _ = O.brick_rects_3d(m3.detach().numpy(), r3.numpy(), TILE3, nt, nt, nt)
    return O.voxelize_slab(m3, c3, opac, rects, valid, GRID, GRID, GRID, TILE3, l0, l1)


def _worker(rank, port, out_path):
    _setup_paths()
    import torch.distributed as dist

    import r2s_shard as shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        params = _params()
        first, count, total, stride = shard.view_shard(VIEWS_PER_RANK, rank, WORLD)
        grads = [g.clone() for g in _projection_grads(params, first, count, total, stride)]
        shard.GradientAllReduce()(grads)
        # strong split: a job of STRONG_VIEWS views dealt over the ranks
        first, count, total, stride = shard.view_split(STRONG_VIEWS, rank, WORLD)
        sgrads = [g.clone() for g in _projection_grads(params, first, count, total, stride)]
        shard.GradientAllReduce()(sgrads)

        l0, l1 = shard.layer_range(GRID // TILE3, rank, WORLD)
        slab = _voxel_slab(params, l0, l1)
        g = torch.Generator().manual_seed(9)
        v_full = torch.randn((GRID, GRID, GRID), generator=g, dtype=torch.float64)
        z0, z1 = shard.slab_rows(l0, l1, TILE3, GRID)
        vgrads = [t.clone() for t in torch.autograd.grad((slab * v_full[z0:z1]).sum(), params)]
        shard.GradientAllReduce()(vgrads)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(WORLD)]
        dist.all_gather(sizes, torch.tensor([slab.shape[0]]))
        slabs = [torch.zeros((int(n), GRID, GRID), dtype=torch.float64) for n in sizes]
        dist.all_gather(slabs, slab.detach().contiguous())
        if rank == 0:
            torch.save({"grads": grads, "sgrads": sgrads, "vgrads": vgrads,
                        "volume": torch.cat(slabs)}, out_path)
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def sharded(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("multirank") / "rank0.pt")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, _free_port_once(), out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return torch.load(out)


_PORT = []


def _free_port_once():
    if not _PORT:
        _PORT.append(_free_port())
    return _PORT[0]


def test_layer_ranges_tile_the_grid():
    _setup_paths()
    import r2s_shard as shard

    for n_layers in (1, 4, 7, 32):
        for world in (1, 2, 3, 8):
            rows = []
            for r in range(world):
                l0, l1 = shard.layer_range(n_layers, r, world)
                assert 0 <= l0 <= l1 <= n_layers
                rows.extend(range(l0, l1))
            assert rows == list(range(n_layers))
    assert shard.slab_rows(3, 4, 8, 30) == (24, 30)
    assert shard.slab_rows(4, 4, 8, 30) == (32, 32)
    with pytest.raises(ValueError):
        shard.layer_range(4, 2, 2)


def test_view_shards_cover_the_orbit():
    _setup_paths()
    import r2s_shard as shard

    seen = []
    for r in range(4):
        first, count, total, stride = shard.view_shard(75, r, 4)
        assert total == 300 and count == 75 and stride == 4
        seen.extend(range(first, first + stride * count, stride))
    assert sorted(seen) == list(range(300))


def test_view_splits_partition_the_job():
    _setup_paths()
    import r2s_shard as shard

    for n_views, world in ((75, 1), (75, 2), (75, 8), (3, 2), (5, 8)):
        seen, counts = [], []
        for r in range(world):
            first, count, total, stride = shard.view_split(n_views, r, world)
            assert total == n_views and stride == world
            seen.extend(range(first, first + stride * count, stride))
            counts.append(count)
        assert sorted(seen) == list(range(n_views))
        assert max(counts) - min(counts) <= 1
    with pytest.raises(ValueError):
        shard.view_split(75, 8, 8)


def test_strong_split_gradient_allreduce_equals_single_process(sharded):
    _setup_paths()
    params = _params()
    full = _projection_grads(params, 0, STRONG_VIEWS, STRONG_VIEWS)
    for a, b in zip(sharded["sgrads"], full):
        torch.testing.assert_close(a, b, rtol=1e-10, atol=1e-12)


def test_projection_gradient_allreduce_equals_single_process(sharded):
    _setup_paths()
    params = _params()
    full = _projection_grads(params, 0, VIEWS_PER_RANK * WORLD, VIEWS_PER_RANK * WORLD)
    for a, b in zip(sharded["grads"], full):
        torch.testing.assert_close(a, b, rtol=1e-10, atol=1e-12)


def test_voxel_slabs_equal_the_full_volume_and_gradient(sharded):
    _setup_paths()
    params = _params()
    nt = GRID // TILE3
    full = _voxel_slab(params, 0, nt)
    torch.testing.assert_close(sharded["volume"], full.detach(), rtol=1e-12, atol=1e-14)
    g = torch.Generator().manual_seed(9)
    v_full = torch.randn((GRID, GRID, GRID), generator=g, dtype=torch.float64)
    ref = torch.autograd.grad((full * v_full).sum(), params)
    for a, b in zip(sharded["vgrads"], ref):
        torch.testing.assert_close(a, b, rtol=1e-10, atol=1e-12)


def test_balanced_layer_ranges():
    _setup_paths()
    import r2s_shard as shard

    # clustered load like the config-2 voxel grid: a bump in the middle layers
    w = [0.06, 0.09, 0.14, 0.2, 0.29, 0.38, 0.49, 0.6, 0.71, 0.8, 0.87, 0.91, 0.94, 0.95, 0.94,
         0.94, 0.95, 0.97, 1.01, 1.04, 1.06, 1.05, 1.0, 0.9, 0.78, 0.63, 0.49, 0.36, 0.25, 0.16,
         0.1, 0.06]
    for world in (1, 2, 3, 8, 40):
        ranges = shard.balanced_layer_ranges(w, world)
        assert len(ranges) == world
        assert ranges[0][0] == 0 and ranges[-1][1] == len(w)
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        loads = [sum(w[l0:l1]) for l0, l1 in ranges]
        if world <= len(w):
            assert max(loads) <= sum(w) / world + max(w) + 1e-9
    even = [sum(w[l0:l1]) for l0, l1 in (shard.layer_range(len(w), r, 8) for r in range(8))]
    balanced = [sum(w[l0:l1]) for l0, l1 in shard.balanced_layer_ranges(w, 8)]
    assert max(balanced) < 0.75 * max(even)
    assert shard.balanced_layer_ranges([0.0] * 4, 2) == [(0, 2), (2, 4)]


def test_layer_weights_from_packed_rects():
    _setup_paths()
    import r2s_shard as shard

    def pack(lo, hi):
        return lo | (hi << 16)

    rows = [(pack(0, 2), pack(1, 4), pack(0, 3), 0),   # area 2*3, layers 0..2
            (pack(1, 2), pack(0, 1), pack(2, 4), 0),   # area 1, layers 2..3
            (pack(3, 3), pack(0, 1), pack(0, 4), 0)]   # empty in x
    rects = torch.tensor(rows, dtype=torch.int64).to(torch.int32).contiguous().view(torch.uint8)
    assert shard.layer_weights(rects, 4) == [6.0, 6.0, 7.0, 1.0]
    extra = shard.BRICK_COST_RECORDS * 9
    assert shard.layer_costs(rects, 4, 9) == [6.0 + extra, 6.0 + extra, 7.0 + extra, 1.0 + extra]


@pytest.mark.parametrize("split", [(4, 4), (3, 5), (1, 2, 5)])
def test_data_parallel_objective_sums_to_the_single_process_gradient(split):
    """Ranks holding view blocks of one training step backpropagate
    data_parallel_objective; the summed gradients equal the gradients of the
    full loss (BinaryTreeLossComputer over all views, TV once, and the
    hierarchy term of the replicated parameters with the reference trainer's
    default weight 0.05, configs/trainer/binary_tree.yaml:25)."""
    import r2s_shard as shard
    from oracle import r2s_oracle as O

    w = dict(w_l1=0.8, w_ssim=0.2, w_tv=0.05, w_edge=0.1)
    w_h = 0.05
    g = torch.Generator().manual_seed(4)
    C, H = sum(split), 24
    renders = torch.rand(C, H, H, 1, generator=g, dtype=torch.float64)
    targets = torch.rand(C, H, H, 1, generator=g, dtype=torch.float64)
    edge = (torch.rand(C, H, H, 1, generator=g) < 0.3).double()
    vol = torch.rand(10, 10, 10, generator=g, dtype=torch.float64)
    means = torch.rand(50, 3, generator=g, dtype=torch.float64)
    parents = torch.rand(50, 3, generator=g, dtype=torch.float64)

    def hierarchy(m):  # a nonzero penalty of the replicated parameters
        return torch.relu((m - parents).norm(dim=-1) - 0.3).square().mean()

    r_full = renders.clone().requires_grad_(True)
    v_full = vol.clone().requires_grad_(True)
    m_full = means.clone().requires_grad_(True)
    assert hierarchy(means) > 0
    (O.binary_tree_losses(r_full, targets, edge, v_full, **w)["total"]
     + w_h * hierarchy(m_full)).backward()

    grad_r = torch.zeros_like(renders)
    grad_v = torch.zeros_like(vol)
    grad_m = torch.zeros_like(means)
    v0 = 0
    for n in split:
        r = renders[v0:v0 + n].clone().requires_grad_(True)
        v = vol.clone().requires_grad_(True)
        m = means.clone().requires_grad_(True)
        out = O.binary_tree_losses(r, targets[v0:v0 + n], edge[v0:v0 + n], v, **w)
        out["edge_weight"] = torch.tensor(w["w_edge"], dtype=torch.float64)
        out["hierarchy"] = hierarchy(m)
        shard.data_parallel_objective(out, w["w_l1"], w["w_ssim"], w["w_tv"], n, C,
                                      len(split), w_hierarchy=w_h).backward()
        grad_r[v0:v0 + n] = r.grad
        grad_v += v.grad
        grad_m += m.grad
        v0 += n
    torch.testing.assert_close(grad_r, r_full.grad, rtol=1e-12, atol=1e-15)
    torch.testing.assert_close(grad_v, v_full.grad, rtol=1e-12, atol=1e-15)
    torch.testing.assert_close(grad_m, m_full.grad, rtol=1e-12, atol=1e-15)
