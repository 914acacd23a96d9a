"""Binary-tree split against the reference's own ``split``.

The reference's ``split`` (src/strategies/binary_tree.py:92-149, unchanged,
loaded by oracle/ref_stock.py) and this build's ``binary_split`` are applied
to two identical reference ``BinaryTreeGaussianModel`` instances with Adam
optimizers that have taken a step (non-zero moments), strategy statistics and
a non-empty tree history.  Everything the split touches is compared: the four
parameters (children's values within 1e-6, every copied row bit-exact), the
binary-tree buffers and history, the optimizer moments and their keying, and
the strategy state.
"""
import pytest
import torch

from _helpers import rel_l2

pytestmark = pytest.mark.gpu

LRS = {"means": 1.6e-4, "quats": 1e-3, "scales": 5e-3, "opacities": 5e-2}
KEYS = ["means", "scales", "quats", "opacities"]


@pytest.fixture(scope="module")
def mods():
    from oracle import ref_stock

    assert ref_stock.stock_available(), "baseline/_ref or oracle/_ref missing"
    return ref_stock.load_binary_tree_model("stock"), ref_stock.load_strategy_module("stock")


def _model(btm, n, seed):
    g = torch.Generator().manual_seed(seed)
    m = btm.BinaryTreeGaussianModel(device="cuda", min_scale=5e-4, max_scale=1.0, scale_eps=1e-5)
    raw_scales = torch.randn(n, 3, generator=g) * 1.5 - 3.0
    raw_scales[:7] = raw_scales[:7, :1]           # all three axes equal: first axis wins
    raw_scales[7:14, 2] = raw_scales[7:14, 1]     # a tie between the last two axes
    m.means = torch.nn.Parameter((torch.rand(n, 3, generator=g) - 0.5).cuda())
    m.scales = torch.nn.Parameter(raw_scales.cuda())
    m.quats = torch.nn.Parameter(torch.randn(n, 4, generator=g).cuda())
    m.opacities = torch.nn.Parameter((torch.randn(n, generator=g) * 2.0).cuda())
    m.trainable_param_keys = list(KEYS)
    h = n // 3
    m.parent = torch.randint(-1, h, (n,), generator=g, dtype=torch.int32).cuda()
    m.level = torch.randint(0, 5, (n,), generator=g, dtype=torch.int32).cuda()
    m.history_means = torch.rand(h, 3, generator=g).cuda()
    m.history_scales = torch.randn(h, 3, generator=g).cuda()
    m.history_quats = torch.randn(h, 4, generator=g).cuda()
    m.history_opacities = torch.randn(h, generator=g).cuda()
    m.history_parent = torch.randint(-1, h, (h,), generator=g, dtype=torch.int32).cuda()
    m.history_level = torch.randint(0, 4, (h,), generator=g, dtype=torch.int32).cuda()
    opts = m.build_optimizers(LRS)
    for k in KEYS:  # one Adam step: non-zero first and second moments
        p = getattr(m, k)
        p.grad = torch.randn(p.shape, generator=g).cuda()
        opts[k].step()
        opts[k].zero_grad(set_to_none=True)
    state = {"grad2d": torch.rand(n, generator=g).cuda(), "count": torch.rand(n, generator=g).cuda(),
             "radii": torch.rand(n, generator=g).cuda(), "scene_scale": 1.0}
    return m, opts, state


@pytest.mark.parametrize("revised", [True, False])
@pytest.mark.parametrize("frac", [0.05, 0.0, 1.0])
def test_binary_split_matches_reference_split(mods, revised, frac):
    from r2splat.ops import training as T

    btm, strat = mods
    n = 20_000
    ref, ref_opts, ref_state = _model(btm, n, 3)
    ours, our_opts, our_state = _model(btm, n, 3)
    g = torch.Generator(device="cuda").manual_seed(41)
    mask = torch.rand(n, generator=g, device="cuda") < frac
    mask[:14] = frac > 0  # the tie cases are split whenever anything is
    strat.split(ref, ref_opts, ref_state, mask, list(KEYS), revised_opacity=revised)
    T.binary_split(ours, our_opts, our_state, mask, list(KEYS), revised_opacity=revised)
    S = int(mask.sum())
    rest = int(n - S)
    for k in KEYS:
        a, b = getattr(ours, k), getattr(ref, k)
        assert isinstance(a, torch.nn.Parameter) and a.shape == b.shape == (n + S,) + b.shape[1:]
        assert torch.equal(a[:rest], b[:rest]), f"{k}: copied rows differ"
        if S:
            e = rel_l2(a[rest:], b[rest:])
            assert e < 1e-6, f"{k}: children rel-L2 {e:.3e}"
        # optimizer: the new parameter is the group's, its moments moved with it
        opt_a, opt_b = our_opts[k], ref_opts[k]
        assert opt_a.param_groups[0]["params"][0] is a
        assert set(opt_a.state.keys()) == {a}
        sa, sb = opt_a.state[a], opt_b.state[b]
        assert sorted(sa) == sorted(sb)
        for key in sa:
            assert torch.equal(torch.as_tensor(sa[key]), torch.as_tensor(sb[key])), f"{k}/{key}"
    for name in ("parent", "level", "history_means", "history_scales", "history_quats",
                 "history_opacities", "history_parent", "history_level"):
        a, b = getattr(ours, name), getattr(ref, name)
        assert a.dtype == b.dtype and torch.equal(a, b), name
    assert set(our_state) == set(ref_state)
    for k, v in ref_state.items():
        if isinstance(v, torch.Tensor):
            assert torch.equal(our_state[k], v), k
        else:
            assert our_state[k] == v
