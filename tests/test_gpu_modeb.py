"""Mode B (shared index records) on the GPU: the reference's own float64 results for canonical and
fragment-packed layers (tests/golden/fwdbwd_modeb_*.npz), and the oracle on the equivalent Mode-A
tensors for larger random layers.  Tolerances: forward rtol 1e-5 / atol 1e-6; dX, dW, db
rtol 1e-4 / atol 1e-5 (plus the oracle's ReLU-boundary allowance where it is used)."""
import hashlib

import pytest
import torch

from conftest import assert_close, load_case, modeb_as_mode_a, modeb_case_names, modeb_case_params
from granulelayer_b200 import PhysicalPlan, SparsePoolingLayer
from oracle import oracle as O

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def _layer(D, H, G, C, packed, seed, bias_std, pool="mean", act="relu", plan=None):
    return SparsePoolingLayer(D, H, G, shared_neurons=C, weight_layout="packed" if packed else "canonical",
                              pooling={"type": pool, "activation": act}, dtype=torch.float32, seed=seed,
                              bias_std=bias_std, plan=plan).cuda()


def _run(lay, x, dy):
    xg = torch.as_tensor(x).cuda().requires_grad_(True)
    y = lay(xg)
    y.backward(torch.as_tensor(dy).cuda())
    torch.cuda.synchronize()
    return y.detach().cpu(), xg.grad.cpu(), lay.weight.grad.cpu(), lay.bias.grad.cpu()


@pytest.mark.parametrize("name", modeb_case_names())
def test_matches_reference_golden(name):
    meta, arr = load_case(name)
    lay = _layer(meta["D"], meta["H"], meta["G"], meta["C"], meta["packed"], meta["seed"], meta["bias_std"],
                 meta["pool"], meta["act"])
    assert hashlib.sha256(lay.indices.cpu().numpy().tobytes()).hexdigest() == meta["idx_sha"]
    assert hashlib.sha256(lay.weight.detach().cpu().numpy().tobytes()).hexdigest() == meta["w_sha"]
    assert lay.explain()["forward"]["kernel"] == "gl_fwd_shared_f32"
    y, dx, dw, db = _run(lay, arr["x"], arr["dy"])
    gs = arr["dw"].shape[0]
    assert_close(y, arr["y"], what="y", **FWD)
    assert_close(dx, arr["dx"], what="dx", **BWD)
    assert_close(dw[:gs], arr["dw"], what="dw", **BWD)
    assert_close(db[:gs], arr["db"], what="db", **BWD)


def _oracle(lay, x, dy, pool="mean", act="relu"):
    L = lay.layout
    ia, wa, ba = modeb_as_mode_a(L, lay.indices.cpu(), lay.weight.detach().cpu(), lay.bias.detach().cpu())
    counts = L.counts_tensor("cpu").numpy()
    pre = O.forward(x, ia.numpy(), wa.numpy(), ba.numpy(), counts, pool, act)
    dx, dw, db, sdx, sdw, sdb = O.backward(x, ia.numpy(), wa.numpy(), ba.numpy(), counts, dy, pool, act, slack=True)
    shape_w = (L.groups, L.blocks_per_group, L.block, 8)
    shape_b = (L.groups, L.blocks_per_group, L.block)
    dw, sdw = torch.from_numpy(dw).reshape(shape_w), torch.from_numpy(sdw).reshape(shape_w)
    db, sdb = torch.from_numpy(db).reshape(shape_b), torch.from_numpy(sdb).reshape(shape_b)
    if L.packed:
        dw, sdw, db, sdb = L.pack_weights(dw), L.pack_weights(sdw), L.pack_bias(db), L.pack_bias(sdb)
    return pre, dx, dw, db, sdx, sdw, sdb


@pytest.mark.parametrize("C,packed", [(8, False), (8, True), (16, True), (32, False), (64, False), (64, True)])
@pytest.mark.parametrize("B", [1, 37, 130])
def test_random_layers_against_oracle(C, packed, B):
    D, H, G = 4096, 2 * 24576 + 333, 3     # ragged: the last group has a partial block
    lay = _layer(D, H, G, C, packed, seed=C + B, bias_std=0.2)
    gen = torch.Generator().manual_seed(B)
    x = torch.randn(B, D, generator=gen).numpy()
    dy = torch.randn(B, G, generator=gen).numpy()
    y, dx, dw, db = _run(lay, x, dy)
    pre, odx, odw, odb, sdx, sdw, sdb = _oracle(lay, x, dy)
    assert_close(y, pre, what="y", **FWD)
    assert_close(dx, odx, what="dx", slack=sdx, **BWD)
    assert_close(dw, odw, what="dw", slack=sdw, **BWD)
    assert_close(db, odb, what="db", slack=sdb, **BWD)


@pytest.mark.parametrize("tf,tb", [(1, 1), (2, 2), (4, 4), (8, 2)])
@pytest.mark.parametrize("act", ["gelu", "identity"])
def test_token_tiles_and_activations(tf, tb, act):
    D, H, G, B = 1000, 5000, 4, 21
    plan = PhysicalPlan(b200_fwd_tokens=tf, b200_dx_tokens=tb)
    lay = _layer(D, H, G, 16, True, seed=3, bias_std=0.3, act=act, plan=plan)
    gen = torch.Generator().manual_seed(tf * 10 + tb)
    x = torch.randn(B, D, generator=gen).numpy()
    dy = torch.randn(B, G, generator=gen).numpy()
    y, dx, dw, db = _run(lay, x, dy)
    pre, odx, odw, odb, sdx, sdw, sdb = _oracle(lay, x, dy, act=act)
    assert_close(y, pre, what="y", **FWD)
    assert_close(dx, odx, what="dx", slack=sdx, **BWD)
    assert_close(dw, odw, what="dw", slack=sdw, **BWD)
    assert_close(db, odb, what="db", slack=sdb, **BWD)


def test_sum_pool_and_main_grad():
    D, H, G, B = 512, 9000, 5, 33
    lay = _layer(D, H, G, 64, False, seed=4, bias_std=0.1, pool="sum")
    lay.enable_main_grad()
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(B, D, generator=gen).cuda()
    dy = torch.randn(B, G, generator=gen).cuda()
    lay(x).backward(dy)
    w1 = lay.weight.main_grad.clone()
    assert lay.weight.grad is None
    lay(x).backward(dy)
    # accumulation (+=): dW is summed with fp32 atomics in varying order, so the dW parity bar applies
    assert_close(lay.weight.main_grad, 2 * w1.double(), what="main_grad", **BWD)
    pre, _, odw, _, _, sdw, _ = _oracle(lay, x.cpu().numpy(), dy.cpu().numpy(), pool="sum")
    assert_close(lay(x).detach(), pre, what="y", **FWD)
    assert_close(w1, odw, what="dw", slack=sdw, **BWD)


def test_padding_slots_get_no_gradient():
    lay = _layer(256, 1000, 3, 64, True, seed=2, bias_std=0.1)   # 333/334 neurons per group: partial blocks
    x = torch.randn(16, 256).cuda()
    lay(x).sum().backward()
    L = lay.layout
    pad = ~L.valid_mask("cuda").view(L.groups, L.blocks_per_group, L.block)
    gw = L.unpack_weights(lay.weight.grad)
    gb = L.unpack_bias(lay.bias.grad)
    assert float(gw[pad].abs().max()) == 0.0 and float(gb[pad].abs().max()) == 0.0


@pytest.mark.parametrize("C,packed", [(8, True), (64, False)])
def test_supergroup_connectivity_layer(C, packed):
    """Mode-B layers with input-supergroup connectivity run on the Mode-B kernels."""
    from granulelayer_b200.supergroups import ConnectivityPlan

    D, H, G, B = 512, 30000, 6, 29
    lay = SparsePoolingLayer(D, H, G, shared_neurons=C, weight_layout="packed" if packed else "canonical",
                             pooling="mean", dtype=torch.float32, seed=2, bias_std=0.1,
                             connectivity=ConnectivityPlan(64, 3, seed=7)).cuda()
    gen = torch.Generator().manual_seed(C)
    x = torch.randn(B, D, generator=gen).numpy()
    dy = torch.randn(B, G, generator=gen).numpy()
    y, dx, dw, db = _run(lay, x, dy)
    pre, odx, odw, odb, sdx, sdw, sdb = _oracle(lay, x, dy)
    assert_close(y, pre, what="y", **FWD)
    assert_close(dx, odx, what="dx", slack=sdx, **BWD)
    assert_close(dw, odw, what="dw", slack=sdw, **BWD)
    assert_close(db, odb, what="db", slack=sdb, **BWD)
