"""Parity of the sm_100a kernels with the reference (GPU).

Every call goes through the C ABI (granulelayer_b200/_native.py ->
libgranule_b200.so).  Two checkers: the golden fixtures made by the
reference's own code (tests/golden/make_golden.py) and the CPU oracle
(oracle/oracle.py) on the same inputs.  Tolerances are the hot path's
parity bar: forward rtol 1e-5 / atol 1e-6; dX, dW, db rtol 1e-4 / atol 1e-5.
"""
import numpy as np
import pytest
import torch

from conftest import assert_close, case_names, case_params, load_case
from granulelayer_b200 import PhysicalPlan, SparsePoolingLayer
from granulelayer_b200 import _native
from granulelayer_b200.layout import SparseLayout, init_parameters
from oracle import oracle as O

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def _layer_for(meta, idx, w, b, plan=None):
    lay = SparsePoolingLayer(meta["D"], meta["H"], meta["G"], shared_neurons=None,
                             pooling={"type": meta["pool"], "activation": meta["act"]}, dtype=torch.float32,
                             seed=meta["seed"], bias_std=meta["bias_std"], plan=plan)
    with torch.no_grad():
        lay.indices.copy_(idx)
        lay.weight.copy_(w)
        lay.bias.copy_(b)
    return lay.cuda()


def _run(lay, x, dy):
    xg = torch.as_tensor(x).cuda().requires_grad_(True)
    y = lay(xg)
    (y * torch.as_tensor(dy).cuda()).sum().backward()
    torch.cuda.synchronize()
    return y.detach().cpu(), xg.grad.cpu(), lay.weight.grad.cpu(), lay.bias.grad.cpu()


@pytest.mark.parametrize("accum", ["fixed", "fp32"])
@pytest.mark.parametrize("name", case_names())
def test_matches_reference_golden(name, accum):
    meta, arr = load_case(name)
    L, idx, w, b = case_params(meta, arr)
    lay = _layer_for(meta, idx, w, b, plan=PhysicalPlan(b200_dx_accum=accum))
    y, dx, dw, db = _run(lay, arr["x"], arr["dy"])
    assert lay.last_info["dx_accumulation"] == ("int32 fixed point" if accum == "fixed" else "fp32 atomics")
    gs = arr["dw"].shape[0]
    c = L.counts_tensor("cpu").numpy()
    _, odw, odb, sdx, sdw, sdb = O.backward(arr["x"], idx.numpy(), w.numpy(), b.numpy(), c, arr["dy"],
                                            meta["pool"], meta["act"], slack=True)
    assert_close(y, arr["y"], what="y", **FWD)
    assert_close(dx, arr["dx"], what="dx", slack=sdx, **BWD)
    assert_close(dw[:gs], arr["dw"], what="dw", slack=sdw[:gs], **BWD)
    assert_close(db[:gs], arr["db"], what="db", slack=sdb[:gs], **BWD)
    # all groups against the oracle
    assert_close(dw, odw, what="dw(all groups)", slack=sdw, **BWD)
    assert_close(db, odb, what="db(all groups)", slack=sdb, **BWD)


@pytest.mark.parametrize("accum", ["fixed", "fp32"])
@pytest.mark.parametrize("tf", [1, 2, 4, 8])
@pytest.mark.parametrize("tb", [1, 2, 4, 8])
def test_token_tiles(tf, tb, accum):
    meta, arr = load_case("ragged_b37")
    L, idx, w, b = case_params(meta, arr)
    lay = _layer_for(meta, idx, w, b, plan=PhysicalPlan(b200_fwd_tokens=tf, b200_dx_tokens=tb, b200_dx_accum=accum))
    y, dx, dw, db = _run(lay, arr["x"], arr["dy"])
    _, _, _, sdx, sdw, _ = O.backward(arr["x"], idx.numpy(), w.numpy(), b.numpy(), L.counts_tensor("cpu").numpy(),
                                      arr["dy"], slack=True)
    assert_close(y, arr["y"], what="y", **FWD)
    assert_close(dx, arr["dx"], what="dx", slack=sdx, **BWD)
    assert_close(dw[:16], arr["dw"], what="dw", slack=sdw[:16], **BWD)


def _rand_layer(D, H, G, seed=0, bias_std=0.2, device="cuda"):
    L = SparseLayout(D, H, G, 8, 8, False)
    idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=seed, bias_std=bias_std)
    return L, idx.to(device), w.to(device), b.to(device)


@pytest.mark.parametrize("pool", [_native.POOL_MEAN, _native.POOL_SUM])
def test_group_range_sharding(pool):
    """A call on groups [g0, g1) gives exactly the columns of the full call."""
    L, idx, w, b = _rand_layer(128, 5000, 13, seed=3)
    counts = L.counts_tensor("cuda")
    x = torch.randn(40, 128, device="cuda")
    full = torch.empty(40, 13, device="cuda")
    _native.fwd(x, idx, w, b, counts, full, L.blocks_per_group, 0, 13, pool, 1)
    for g0, g1 in [(0, 5), (5, 13), (7, 8)]:
        part = torch.full((40, g1 - g0), float("nan"), device="cuda")
        _native.fwd(x, idx, w, b, counts, part, L.blocks_per_group, g0, g1, pool, 1)
        assert torch.equal(part, full[:, g0:g1])


def _bounds(L, idx, w, counts, g0, g1):
    wm = torch.empty(g1 - g0, device="cuda")
    rm = torch.empty(g1 - g0, device="cuda", dtype=torch.int32)
    _native.group_absmax(w, counts, L.blocks_per_group, g0, g1, wm)
    _native.group_index_maxcount(idx, counts, L.input_dim, L.blocks_per_group, g0, g1, rm)
    return wm, rm


@pytest.mark.parametrize("fixed", [True, False])
def test_backward_group_range_sums_to_full(fixed):
    L, idx, w, b = _rand_layer(96, 4000, 9, seed=4)
    counts = L.counts_tensor("cuda").to(torch.int32)
    x = torch.randn(33, 96, device="cuda")
    gp = torch.randn(33, 9, device="cuda")
    NB = L.blocks_per_group
    dx_full = torch.zeros(33, 96, device="cuda")
    dw_full, db_full = torch.zeros_like(w), torch.zeros_like(b)
    kw = dict(zip(("wabsmax", "rowmax"), _bounds(L, idx, w, counts, 0, 9))) if fixed else {}
    _native.bwd(x, idx, w, b, counts, gp, dx_full, dw_full, db_full, NB, 0, 9, 0, 1, **kw)
    dx_sum = torch.zeros_like(dx_full)
    dw_p, db_p = torch.zeros_like(w), torch.zeros_like(b)
    for g0, g1 in [(0, 4), (4, 9)]:
        kw = dict(zip(("wabsmax", "rowmax"), _bounds(L, idx, w, counts, g0, g1))) if fixed else {}
        _native.bwd(x, idx, w, b, counts, gp[:, g0:g1].contiguous(), dx_sum, dw_p, db_p, NB, g0, g1, 0, 1, **kw)
    assert_close(dx_sum, dx_full, what="dx", **BWD)
    assert_close(dw_p, dw_full, what="dw", **BWD)
    assert_close(db_p, db_full, what="db", **BWD)


def test_main_grad_accumulates_across_steps():
    meta, arr = load_case("batch1")
    L, idx, w, b = case_params(meta, arr)
    lay = _layer_for(meta, idx, w, b)
    lay.enable_main_grad()
    x = torch.randn(16, meta["D"], device="cuda")
    lay(x).sum().backward()
    g1 = lay.weight.main_grad.clone()
    assert lay.weight.grad is None
    lay(x).sum().backward()
    assert_close(lay.weight.main_grad, 2 * g1, 1e-5, 1e-9, "main_grad")
    lay.zero_main_grad()
    assert float(lay.weight.main_grad.abs().max()) == 0.0


def test_forward_is_bitwise_deterministic():
    meta, arr = load_case("cfg1_mean_relu")
    L, idx, w, b = case_params(meta, arr)
    lay = _layer_for(meta, idx, w, b)
    x = torch.as_tensor(arr["x"]).cuda()
    with torch.no_grad():
        a, c = lay(x), lay(x)
    assert torch.equal(a, c)


def test_inplace_param_update_between_fwd_and_bwd_is_rejected():
    meta, arr = load_case("batch1")
    L, idx, w, b = case_params(meta, arr)
    lay = _layer_for(meta, idx, w, b)
    y = lay(torch.randn(4, meta["D"], device="cuda"))
    with torch.no_grad():
        lay.weight.add_(1.0)
    with pytest.raises(RuntimeError):
        y.sum().backward()


def test_strided_input_and_leading_dims():
    meta, arr = load_case("ragged_b37")
    L, idx, w, b = case_params(meta, arr)
    lay = _layer_for(meta, idx, w, b)
    x = torch.as_tensor(arr["x"]).cuda()
    wide = torch.zeros(x.shape[0], x.shape[1] + 7, device="cuda")
    wide[:, 3:3 + x.shape[1]] = x
    with torch.no_grad():
        y_strided = lay(wide[:, 3:3 + x.shape[1]])
        y3 = lay(x[:36].reshape(4, 9, -1))
    assert_close(y_strided.cpu(), arr["y"], what="y(strided)", **FWD)
    assert y3.shape == (4, 9, meta["G"])
    assert_close(y3.reshape(36, -1).cpu(), arr["y"][:36], what="y(3d)", **FWD)


def test_empty_batch():
    meta, arr = load_case("batch1")
    L, idx, w, b = case_params(meta, arr)
    lay = _layer_for(meta, idx, w, b)
    x = torch.zeros(0, meta["D"], device="cuda", requires_grad=True)
    y = lay(x)
    assert y.shape == (0, meta["G"])
    y.sum().backward()
    assert x.grad.shape == (0, meta["D"])


@pytest.mark.parametrize("D", [9, 17, 4096, 16384, 28000])
def test_wide_and_narrow_inputs_against_oracle(D):
    H, G, B = 2500, 5, 19
    L, idx, w, b = _rand_layer(D, H, G, seed=D)
    counts = L.counts_tensor("cpu").numpy()
    x = torch.randn(B, D)
    dy = torch.randn(B, G)
    lay = SparsePoolingLayer(D, H, G, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=D,
                             bias_std=0.2).cuda()
    y, dx, dw, db = _run(lay, x.numpy(), dy.numpy())
    pre = O.forward(x.numpy(), idx.cpu().numpy(), w.cpu().numpy(), b.cpu().numpy(), counts)
    odx, odw, odb, sdx, sdw, sdb = O.backward(x.numpy(), idx.cpu().numpy(), w.cpu().numpy(), b.cpu().numpy(),
                                              counts, dy.numpy(), slack=True)
    assert_close(y, pre, what="y", **FWD)
    assert_close(dx, odx, what="dx", slack=sdx, **BWD)
    assert_close(dw, odw, what="dw", slack=sdw, **BWD)
    assert_close(db, odb, what="db", slack=sdb, **BWD)


def test_no_hidden_activation_is_materialized():
    """[B, H] in fp32 would be 2 GiB here; forward + backward must stay far below
    (the reference's test_recomputation.py:67-85)."""
    B, H = 256, 2_000_000
    lay = SparsePoolingLayer(1024, H, 1024, shared_neurons=None, pooling="mean", dtype=torch.float32,
                             device="cuda")
    lay.enable_main_grad()
    x = torch.randn(B, 1024, device="cuda", requires_grad=True)
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    lay(x).square().mean().backward()
    torch.cuda.synchronize()
    extra = torch.cuda.max_memory_allocated() - base
    assert extra < B * H * 4 / 20, f"peak extra {extra / 2**20:.0f} MiB suggests materialization"
    assert lay.last_info["checkpoint_bytes"] == B * 1024 * 4


@pytest.mark.parametrize("D,H,G", [(64, 3001, 8), (4096, 200_000, 4), (777, 5000, 13)])
def test_group_bounds_match_torch(D, H, G):
    L, idx, w, b = _rand_layer(D, H, G, seed=11)
    counts = L.counts_tensor("cuda").to(torch.int32)
    wm, rm = _bounds(L, idx, w, counts, 0, G)
    valid = L.valid_mask("cuda").view(G, -1)
    w_valid = torch.where(valid[..., None], w.view(G, -1, 8).abs(), torch.zeros((), device="cuda"))
    assert torch.equal(wm, w_valid.amax(dim=(1, 2)))
    hist = torch.zeros(G, D, device="cuda", dtype=torch.int64)
    iv = torch.where(valid[..., None], idx.view(G, -1, 8).long(), torch.full((), D, device="cuda"))
    hist2 = torch.zeros(G, D + 1, device="cuda", dtype=torch.int64)
    hist2.scatter_add_(1, iv.view(G, -1), torch.ones_like(iv.view(G, -1)))
    assert torch.equal(rm.long(), hist2[:, :D].amax(1))
    # the forward's optional output equals the standalone bound
    pre = torch.empty(5, G, device="cuda")
    wm2 = torch.empty(G, device="cuda")
    _native.fwd(torch.randn(5, D, device="cuda"), idx, w, b, counts, pre, L.blocks_per_group, 0, G, 0, 1,
                wabsmax=wm2)
    assert torch.equal(wm2, wm)


@pytest.mark.parametrize("accum", ["fixed", "fp32"])
@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
def test_nonfinite_upstream_gradient_reaches_dx(accum, bad):
    meta, arr = load_case("ragged_b37")
    L, idx, w, b = case_params(meta, arr)
    lay = _layer_for(meta, idx, w, b, plan=PhysicalPlan(b200_dx_accum=accum))
    dy = arr["dy"].copy()
    dy[3, 2] = bad
    y, dx, dw, db = _run(lay, arr["x"], dy)
    assert not bool(torch.isfinite(dx[3]).all()), "token 3 must see the non-finite coefficient"
    keep = [t for t in range(dx.shape[0]) if t != 3]
    sdx = O.backward(arr["x"], idx.numpy(), w.numpy(), b.numpy(), L.counts_tensor("cpu").numpy(), arr["dy"],
                     slack=True)[3]
    assert_close(dx[keep], arr["dx"][keep], what="dx(other tokens)", slack=sdx[keep], **BWD)


@pytest.mark.parametrize("B", [1, 32, 67])
def test_windowed_indices_against_oracle(B):
    """Config-5 geometry, reduced: D = 16384, 12,288 neurons per group, supergroups of 4096 neurons
    drawing from 512-wide windows (layout.windowed_indices)."""
    from granulelayer_b200.layout import windowed_indices

    D, G = 16384, 3
    H = G * 12288
    lay = SparsePoolingLayer(D, H, G, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=4,
                             bias_std=0.1)
    with torch.no_grad():
        lay.indices.copy_(windowed_indices(lay.layout, "cpu", window=512, supergroup=4096, seed=4))
    idx, w, b = lay.indices.clone(), lay.weight.detach().clone(), lay.bias.detach().clone()
    counts = lay.layout.counts_tensor("cpu").numpy()
    gen = torch.Generator().manual_seed(B)
    x = torch.randn(B, D, generator=gen)
    dy = torch.randn(B, G, generator=gen)
    y, dx, dw, db = _run(lay.cuda(), x.numpy(), dy.numpy())
    pre = O.forward(x.numpy(), idx.numpy(), w.numpy(), b.numpy(), counts)
    odx, odw, odb, sdx, sdw, sdb = O.backward(x.numpy(), idx.numpy(), w.numpy(), b.numpy(), counts, dy.numpy(),
                                              slack=True)
    assert_close(y, pre, what="y", **FWD)
    assert_close(dx, odx, what="dx", slack=sdx, **BWD)
    assert_close(dw, odw, what="dw", slack=sdw, **BWD)
    assert_close(db, odb, what="db", slack=sdb, **BWD)


def test_feature_map_matches_torch():
    """gl_group_feature_map: the sorted distinct features of each group's valid records, and the
    records as positions in that list."""
    from granulelayer_b200.layout import windowed_indices

    L = SparseLayout(16384, 3 * 12288 + 77, 4, 8, 8, False)
    idx = windowed_indices(L, "cpu", window=512, supergroup=4096, seed=5)
    counts = L.counts_tensor("cpu").to(torch.int32)
    di, dc = idx.cuda(), counts.cuda()
    nf = torch.empty(L.groups, dtype=torch.int32, device="cuda")
    _native.group_feature_map(di, dc, L.input_dim, L.blocks_per_group, 0, L.groups, nf)
    cap = int(nf.max())
    fmap = torch.full((L.groups, cap), -1, dtype=torch.int16, device="cuda")
    lidx = torch.empty_like(di)
    _native.group_feature_map(di, dc, L.input_dim, L.blocks_per_group, 0, L.groups, nf, fmap, lidx)
    valid = L.valid_mask("cpu").view(L.groups, L.blocks_per_group, 8)
    for g in range(L.groups):
        used = torch.unique(idx[g][valid[g]].long())
        n_g = int(counts[g])
        assert int(nf[g]) == used.numel() <= 512 * (n_g // 4096 + 2)   # windows a group can straddle
        assert torch.equal(fmap[g, :used.numel()].cpu().long(), used)
        pos = torch.searchsorted(used, idx[g][valid[g]].long())
        assert torch.equal(lidx[g][valid[g]].cpu().long(), pos)


@pytest.mark.parametrize("B", [1, 40, 300])
@pytest.mark.parametrize("accum", ["fixed", "fp32"])
def test_input_locality_path(B, accum):
    """Windowed indices at D = 16384: the runtime stages only each group's features (token tiles of
    32 forward / 8 backward instead of 2 / 1); results match the oracle and the full-row path."""
    from granulelayer_b200.layout import windowed_indices

    D, G = 16384, 3
    H = G * 12288
    outs = []
    for loc in ("auto", "off"):
        lay = SparsePoolingLayer(D, H, G, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=6,
                                 bias_std=0.1, plan=PhysicalPlan(b200_locality=loc, b200_dx_accum=accum))
        with torch.no_grad():
            lay.indices.copy_(windowed_indices(lay.layout, "cpu", window=512, supergroup=4096, seed=6))
        idx, w, b = lay.indices.clone(), lay.weight.detach().clone(), lay.bias.detach().clone()
        lay = lay.cuda()
        gen = torch.Generator().manual_seed(B)
        x = torch.randn(B, D, generator=gen)
        dy = torch.randn(B, G, generator=gen)
        outs.append(_run(lay, x.numpy(), dy.numpy()))
        assert (lay._runtime().locality() is not None) == (loc == "auto")
    counts = SparseLayout(D, H, G, 8, 8, False).counts_tensor("cpu").numpy()
    pre = O.forward(x.numpy(), idx.numpy(), w.numpy(), b.numpy(), counts)
    odx, odw, odb, sdx, sdw, sdb = O.backward(x.numpy(), idx.numpy(), w.numpy(), b.numpy(), counts, dy.numpy(),
                                              slack=True)
    for (y, dx, dw, db) in outs:
        assert_close(y, pre, what="y", **FWD)
        assert_close(dx, odx, what="dx", slack=sdx, **BWD)
        assert_close(dw, odw, what="dw", slack=sdw, **BWD)
        assert_close(db, odb, what="db", slack=sdb, **BWD)


def test_uniform_indices_keep_the_full_row_path():
    lay = SparsePoolingLayer(4096, 3 * 24576, 3, shared_neurons=None, pooling="mean", dtype=torch.float32,
                             seed=1).cuda()
    lay(torch.randn(4, 4096, device="cuda"))
    assert lay._runtime().locality() is None
