"""Top-K mean pooling on the GPU (Mode A and Mode B): the forwards' per-warp key lists and block
merge, the slots they select, and the k-event backward, against the reference's float64 fixtures
(tests/golden/fwdbwd_topk_*.npz) and the float64 oracle (oracle/pool_oracle.py).  Tolerances:
forward rtol 1e-5 / atol 1e-6; dX, dW, db rtol 1e-4 / atol 1e-5; selected slots exact."""
import numpy as np
import pytest
import torch

from conftest import assert_close, load_case, modeb_as_mode_a, topk_case_names
from granulelayer_b200 import PhysicalPlan, SparsePoolingLayer
from oracle import pool_oracle as P

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def _layer(D, H, G, C, packed, seed, bias_std, k, act, policy="auto", plan=None):
    return SparsePoolingLayer(D, H, G, shared_neurons=C, weight_layout="packed" if packed else "canonical",
                              pooling={"type": "topk_mean", "k": k, "activation": act}, checkpoint_policy=policy,
                              dtype=torch.float32, seed=seed, bias_std=bias_std, plan=plan).cuda()


def _run(lay, x, dy):
    xg = torch.as_tensor(x).cuda().requires_grad_(True)
    y = lay(xg)
    y.backward(torch.as_tensor(dy).cuda())
    torch.cuda.synchronize()
    return y.detach().cpu(), xg.grad.cpu(), lay.weight.grad.cpu(), lay.bias.grad.cpu()


def _oracle(lay, x, dy, k, act):
    L = lay.layout
    idx, w, b = lay.indices.cpu(), lay.weight.detach().cpu(), lay.bias.detach().cpu()
    if L.shared_indices:
        idx, w, b = modeb_as_mode_a(L, idx, w, b)
    counts = L.counts_tensor("cpu").numpy()
    y, slots = P.topk_forward(x, idx.numpy(), w.numpy(), b.numpy(), counts, k, act)
    dx, dw, db = P.topk_backward(x, idx.numpy(), w.numpy(), b.numpy(), counts, dy, k, act, slots=slots)
    dwc = torch.from_numpy(dw).reshape(L.groups, L.blocks_per_group, L.block, 8)
    dbc = torch.from_numpy(db).reshape(L.groups, L.blocks_per_group, L.block)
    if L.packed:
        dwc, dbc = L.pack_weights(dwc), L.pack_bias(dbc)
    return y, slots, dx, dwc, dbc


def _slots(lay, x):
    out = lay._runtime().forward(torch.as_tensor(x).cuda(), lay.weight.detach(), lay.bias.detach(), track_ids=True)
    B = x.shape[0]
    return out["winner"].view(B, lay.layout.groups, -1).cpu().numpy()


@pytest.mark.parametrize("name", topk_case_names())
def test_matches_reference_golden(name):
    meta, arr = load_case(name)
    lay = _layer(meta["D"], meta["H"], meta["G"], meta["C"], meta["packed"], meta["seed"], meta["bias_std"],
                 meta["k"], meta["act"])
    assert lay.effective_policy == "save_winners"
    slots = _slots(lay, arr["x"])
    counts = lay.layout.counts_tensor("cpu").numpy()
    live = np.arange(meta["k"])[None, None, :] < np.minimum(counts, meta["k"])[None, :, None]
    assert np.array_equal(np.where(live, slots, -1), np.where(live, arr["topk"], -1))
    assert (slots[~np.broadcast_to(live, slots.shape)] == -1).all()
    y, dx, dw, db = _run(lay, arr["x"], arr["dy"])
    gs = arr["dw"].shape[0]
    assert_close(y, arr["y"], what="y", **FWD)
    assert_close(dx, arr["dx"], what="dx", **BWD)
    assert_close(dw[:gs], arr["dw"], what="dw", **BWD)
    assert_close(db[:gs], arr["db"], what="db", **BWD)


@pytest.mark.parametrize("C,packed", [(None, False), (8, True), (64, False)])
@pytest.mark.parametrize("k,act", [(1, "relu"), (4, "identity"), (32, "gelu"), (64, "identity")])
@pytest.mark.parametrize("policy", ["save_winners", "minimal_stats"])
def test_random_layers_against_oracle(C, packed, k, act, policy):
    D, H, G, B = 512, 20000, 10, 37
    lay = _layer(D, H, G, C, packed, seed=5, bias_std=0.2, k=k, act=act, policy=policy)
    gen = torch.Generator().manual_seed(7 + k)
    x = torch.randn(B, D, generator=gen).numpy()
    dy = torch.randn(B, G, generator=gen).numpy()
    y, dx, dw, db = _run(lay, x, dy)
    assert lay.last_info["recomputed_stats"] == (policy == "minimal_stats")
    oy, oslots, odx, odw, odb = _oracle(lay, x, dy, k, act)
    assert np.array_equal(_slots(lay, x), oslots)
    assert_close(y, oy, what="y", **FWD)
    assert_close(dx, odx, what="dx", **BWD)
    assert_close(dw, odw, what="dw", **BWD)
    assert_close(db, odb, what="db", **BWD)


@pytest.mark.parametrize("tokens", [1, 2, 4])
def test_token_tiles_and_ties(tokens):
    """Every token tile selects the same slots; duplicate neurons (equal z) are broken by the smaller
    slot, as the reference's stable sort does."""
    plan = PhysicalPlan(b200_fwd_tokens=tokens)
    D, H, G, B, k = 64, 4000, 4, 9, 8
    for C, packed in ((None, False), (16, True)):
        lay = _layer(D, H, G, C, packed, seed=3, bias_std=0.1, k=k, act="identity", plan=plan)
        with torch.no_grad():   # every neuron's twin: the same record, weights and bias in the next block
            L = lay.layout
            if L.shared_indices:
                iw = L.to_canonical(lay.indices, lay.weight, lay.bias)
                ci, cw, cb = [t.clone() for t in iw]
                ci[:, 1::2], cw[:, 1::2], cb[:, 1::2] = ci[:, 0::2], cw[:, 0::2], cb[:, 0::2]
                lay.indices.copy_(L.pack_indices(ci))
                lay.weight.copy_(L.pack_weights(cw))
                lay.bias.copy_(L.pack_bias(cb))
            else:
                lay.indices[:, 1::2] = lay.indices[:, 0::2].clone()
                lay.weight[:, 1::2] = lay.weight[:, 0::2].clone()
                lay.bias[:, 1::2] = lay.bias[:, 0::2].clone()
        x = torch.randn(B, D, generator=torch.Generator().manual_seed(tokens)).numpy()
        oy, oslots, _, _, _ = _oracle(lay, x, np.zeros((B, G), np.float32), k, "identity")
        assert np.array_equal(_slots(lay, x), oslots)
        y = lay(torch.as_tensor(x).cuda()).detach().cpu()
        assert_close(y, oy, what="y", **FWD)
