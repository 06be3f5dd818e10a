"""Deterministic reduction (PhysicalPlan.reduction = "deterministic") on the GPU: the Mode-B
backward with single-owner dW / db and exact int64 dX accumulation is bitwise repeatable, matches
the float64 oracle (dX, dW, db rtol 1e-4 / atol 1e-5) and the fast backward within that tolerance,
and the runtime resolves the policy as the reference does (README "Deterministic execution")."""
import warnings

import pytest
import torch

from conftest import assert_close, modeb_as_mode_a
from granulelayer_b200 import PhysicalPlan, SparsePoolingLayer
from oracle import oracle as O

pytestmark = pytest.mark.gpu

BWD = dict(rtol=1e-4, atol=1e-5)


def _layer(C, packed, pool="mean", act="relu", reduction="deterministic", H=30000, D=512, G=6, seed=3):
    return SparsePoolingLayer(D, H, G, shared_neurons=C, weight_layout="packed" if packed else "canonical",
                              pooling={"type": pool, "activation": act}, dtype=torch.float32, seed=seed,
                              bias_std=0.2, plan=PhysicalPlan(reduction=reduction)).cuda()


def _grads(lay, x, dy):
    lay.weight.grad = lay.bias.grad = None
    xg = x.clone().requires_grad_(True)
    lay(xg).backward(dy)
    torch.cuda.synchronize()
    return xg.grad.clone(), lay.weight.grad.clone(), lay.bias.grad.clone()


@pytest.mark.parametrize("C,packed", [(8, True), (16, False), (64, True), (64, False)])
@pytest.mark.parametrize("pool,act", [("mean", "relu"), ("sum", "identity"), ("mean", "gelu")])
def test_bitwise_repeatable_and_correct(C, packed, pool, act):
    lay = _layer(C, packed, pool, act)
    gen = torch.Generator().manual_seed(C)
    x = torch.randn(37, 512, generator=gen).cuda()
    dy = torch.randn(37, 6, generator=gen).cuda()
    a = _grads(lay, x, dy)
    b = _grads(lay, x, dy)
    assert lay.last_info["reduction"]["mode"] == "deterministic"
    assert lay.last_info["backward_kernel"] == "gl_bwd_shared_det_f32"
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    L = lay.layout
    ia, wa, ba = modeb_as_mode_a(L, lay.indices.cpu(), lay.weight.detach().cpu(), lay.bias.detach().cpu())
    counts = L.counts_tensor("cpu").numpy()
    dx, dw, db, sdx, sdw, sdb = O.backward(x.cpu().numpy(), ia.numpy(), wa.numpy(), ba.numpy(), counts,
                                           dy.cpu().numpy(), pool, act, slack=True)
    shape_w, shape_b = (L.groups, L.blocks_per_group, L.block, 8), (L.groups, L.blocks_per_group, L.block)
    dw, sdw = torch.from_numpy(dw).reshape(shape_w), torch.from_numpy(sdw).reshape(shape_w)
    db, sdb = torch.from_numpy(db).reshape(shape_b), torch.from_numpy(sdb).reshape(shape_b)
    if L.packed:
        dw, sdw, db, sdb = L.pack_weights(dw), L.pack_weights(sdw), L.pack_bias(db), L.pack_bias(sdb)
    assert_close(a[0].cpu(), dx, what="dx", slack=sdx, **BWD)
    assert_close(a[1].cpu(), dw, what="dw", slack=sdw, **BWD)
    assert_close(a[2].cpu(), db, what="db", slack=sdb, **BWD)
    lay.plan = PhysicalPlan(reduction="fast")
    f = _grads(lay, x, dy)
    for u, v, what in zip(a, f, ("dx", "dw", "db")):
        assert_close(u.cpu(), v.cpu().double(), what=what, **BWD)


def test_repeatable_across_layers_and_main_grad():
    """Two layers built alike give bit-identical gradients, and bit-identical main_grad after two
    accumulating steps (the deterministic dW adds each token tile's sums in a fixed order)."""
    x = torch.randn(64, 512, generator=torch.Generator().manual_seed(5)).cuda()
    dy = torch.randn(64, 6, generator=torch.Generator().manual_seed(6)).cuda()
    l1, l2 = _layer(8, True), _layer(8, True)
    g1, g2 = _grads(l1, x, dy), _grads(l2, x, dy)
    for u, v in zip(g1, g2):
        assert torch.equal(u, v)
    for lay in (l1, l2):
        lay.enable_main_grad()
        lay(x).backward(dy)
        assert torch.equal(lay.weight.main_grad, g1[1])
        lay(x).backward(dy)
    assert torch.equal(l1.weight.main_grad, l2.weight.main_grad)
    assert torch.equal(l1.bias.main_grad, l2.bias.main_grad)
    assert_close(l1.weight.main_grad.cpu(), 2 * g1[1].cpu().double(), what="main_grad", **BWD)


def test_non_finite_upstream_gradient_marks_its_token():
    lay = _layer(8, True)
    x = torch.randn(5, 512, generator=torch.Generator().manual_seed(1)).cuda()
    dy = torch.randn(5, 6, generator=torch.Generator().manual_seed(2)).cuda()
    dy[2, 3] = float("inf")
    dx, _, _ = _grads(lay, x, dy)
    assert torch.isnan(dx[2]).all()
    assert torch.isfinite(dx[[0, 1, 3, 4]]).all()


def test_policy_resolution():
    x = torch.randn(4, 512).cuda()
    mode_a = SparsePoolingLayer(512, 6000, 6, shared_neurons=None, pooling="mean", dtype=torch.float32,
                                plan=PhysicalPlan(reduction="deterministic")).cuda()
    with pytest.raises(ValueError, match="Mode-A"):
        mode_a(x)
    with pytest.raises(ValueError, match="max"):
        _layer(8, True, pool="max", act="identity")(x)
    lay = _layer(8, True, reduction="auto")
    torch.use_deterministic_algorithms(True)
    try:
        lay(x.requires_grad_(True)).sum().backward()
        assert lay.last_info["reduction"]["mode"] == "deterministic"
        with pytest.raises(ValueError):
            SparsePoolingLayer(512, 6000, 6, shared_neurons=None, pooling="mean", dtype=torch.float32).cuda()(x)
    finally:
        torch.use_deterministic_algorithms(False)
    torch.use_deterministic_algorithms(True, warn_only=True)
    try:
        with warnings.catch_warnings(record=True) as rec:
            warnings.simplefilter("always")
            SparsePoolingLayer(512, 6000, 6, shared_neurons=None, pooling="mean", dtype=torch.float32).cuda()(x)
        assert any("deterministic" in str(r.message) for r in rec)
    finally:
        torch.use_deterministic_algorithms(False)
