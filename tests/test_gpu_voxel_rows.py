"""The voxel row table (r2s_voxel_rows_f32): the 8-voxel-brick forward and
backward that read it agree with the same kernels culling by the box alone
-- the forward bit for bit (the table only skips half-bricks with no passing
voxel), the backward to float rounding -- on full and ragged grids and on a
z-slab of the global binning."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dims,layers", [((48, 48, 48), None), ((37, 29, 45), None),
                                         ((40, 40, 64), (3, 7))])
def test_row_table_matches_box_culling(dims, layers):
    import r2s_workloads as wl
    from r2splat.cuda import _wrapper as W

    dim2, dim1, dim0 = dims
    m, q, s, o = (t.cuda() for t in wl.make_gaussians(wl.CONFIGS[1], n=20000, seed=4))
    cov, _, op = W.fused_prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
    rng, ctr = (t.cuda() for t in wl.unit_cube_box())
    nt2, nt1, nt0 = (dim2 + 7) // 8, (dim1 + 7) // 8, (dim0 + 7) // 8
    _, _, _, vs, rects, _ = W.fused_map(m, cov, op, rng, ctr, dim2, dim1, dim0, 8, nt2, nt1, nt0,
                                        wl.EPS3D, wl.RADIUS_CLIP)
    l0, l1 = layers if layers else (0, nt0)
    offs, fids, _ = W.fused_bin(rects, l1 - l0, m.size(0), nt1 * nt2, nt2, 1, segment_base=l0)
    assert fids.numel() > 0
    rows = W.fused_voxel_rows(vs, offs, fids, m.size(0), dim2, dim1, dim0, 8, nt2, nt1, nt0, l0, l1)
    assert rows.shape == (fids.numel(), 2)
    for _ in range(2):  # the table is read-only: two calls in a row agree
        v_rows = W.fused_voxel_fwd(vs, offs, fids, m.size(0), dim2, dim1, dim0, 8, nt2, nt1, nt0,
                                   l0, l1, rows=rows)
        v_box = W.fused_voxel_fwd(vs, offs, fids, m.size(0), dim2, dim1, dim0, 8, nt2, nt1, nt0,
                                  l0, l1)
        assert torch.equal(v_rows, v_box) and v_box.abs().max() > 0
    g = torch.Generator(device="cuda").manual_seed(2)
    v_vol = torch.randn(v_box.shape, generator=g, device="cuda")
    st_rows = W.fused_voxel_bwd(vs, offs, fids, v_vol, m.size(0), dim2, dim1, dim0, 8, nt2, nt1,
                                nt0, l0, l1, rows=rows)
    st_box = W.fused_voxel_bwd(vs, offs, fids, v_vol, m.size(0), dim2, dim1, dim0, 8, nt2, nt1,
                               nt0, l0, l1)
    rel = ((st_rows.double() - st_box.double()).norm() / st_box.double().norm()).item()
    assert rel < 1e-6, rel
    # every slice byte is a valid range or the empty marker
    b = rows.view(torch.uint8).reshape(-1, 8).long()
    lo, hi = b & 15, b >> 4
    assert bool(((lo <= hi) & (hi <= 7) | (b == 0x0F)).all())


@pytest.mark.parametrize("dims,layers", [((48, 48, 48), None), ((40, 40, 64), (3, 7))])
def test_brick_order_is_a_longest_first_permutation(dims, layers):
    """r2s_brick_order lists every brick once, in non-increasing
    floor(log2(records)) groups; the row table, forward and backward launched
    in that order give the key-order results (the forward bit for bit)."""
    import r2s_workloads as wl
    from r2splat.cuda import _wrapper as W

    dim2, dim1, dim0 = dims
    m, q, s, o = (t.cuda() for t in wl.make_gaussians(wl.CONFIGS[1], n=20000, seed=5))
    cov, _, op = W.fused_prepare(q, s, o, wl.SCALE_MIN, wl.SCALE_MAX)
    rng, ctr = (t.cuda() for t in wl.unit_cube_box())
    nt2, nt1, nt0 = (dim2 + 7) // 8, (dim1 + 7) // 8, (dim0 + 7) // 8
    _, _, _, vs, rects, _ = W.fused_map(m, cov, op, rng, ctr, dim2, dim1, dim0, 8, nt2, nt1, nt0,
                                        wl.EPS3D, wl.RADIUS_CLIP)
    l0, l1 = layers if layers else (0, nt0)
    N = m.size(0)
    offs, fids, _ = W.fused_bin(rects, l1 - l0, N, nt1 * nt2, nt2, 1, segment_base=l0)
    order = W.fused_brick_order(offs, fids.numel())
    n_keys = offs.numel()
    assert torch.equal(order.sort().values.long(), torch.arange(n_keys, device="cuda"))
    counts = torch.diff(torch.cat([offs.long(), torch.tensor([fids.numel()], device="cuda")]))
    # bit length of the count (floor(log2 c) + 1, 0 for empty bricks), exactly
    groups = torch.frexp(counts.double()).exponent.long() * (counts > 0)
    g_ord = groups[order.long()]
    assert bool((g_ord[:-1] >= g_ord[1:]).all()), "order is not longest-first by group"
    args = (vs, offs, fids, N, dim2, dim1, dim0, 8, nt2, nt1, nt0, l0, l1)
    rows_k = W.fused_voxel_rows(*args)
    rows_o = W.fused_voxel_rows(*args, order=order)
    assert torch.equal(rows_k, rows_o)
    v_k = W.fused_voxel_fwd(*args, rows=rows_k)
    v_o = W.fused_voxel_fwd(*args, rows=rows_o, order=order)
    assert torch.equal(v_k, v_o) and v_k.abs().max() > 0
    g = torch.Generator(device="cuda").manual_seed(3)
    v_vol = torch.randn(v_k.shape, generator=g, device="cuda")
    st_k = W.fused_voxel_bwd(vs, offs, fids, v_vol, N, dim2, dim1, dim0, 8, nt2, nt1, nt0, l0, l1,
                             rows=rows_k)
    st_o = W.fused_voxel_bwd(vs, offs, fids, v_vol, N, dim2, dim1, dim0, 8, nt2, nt1, nt0, l0, l1,
                             rows=rows_o, order=order)
    rel = ((st_o.double() - st_k.double()).norm() / st_k.double().norm()).item()
    assert rel < 1e-6, rel
