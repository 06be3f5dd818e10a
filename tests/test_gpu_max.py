"""Max pooling on the GPU (Mode A and Mode B): the forward's max and winners, and the winner-event
backward, against the reference's float64 fixtures (tests/golden/fwdbwd_max_*.npz) and the max
oracle (oracle/pool_oracle.py).  Tolerances: forward rtol 1e-5 / atol 1e-6; dX, dW, db
rtol 1e-4 / atol 1e-5; winners exact."""
import numpy as np
import pytest
import torch

from conftest import assert_close, load_case, max_case_names, modeb_as_mode_a
from granulelayer_b200 import SparsePoolingLayer
from oracle import pool_oracle as P

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def _layer(D, H, G, C, packed, seed, bias_std, act, policy="auto"):
    return SparsePoolingLayer(D, H, G, shared_neurons=C, weight_layout="packed" if packed else "canonical",
                              pooling={"type": "max", "activation": act}, checkpoint_policy=policy,
                              dtype=torch.float32, seed=seed, bias_std=bias_std).cuda()


def _run(lay, x, dy):
    xg = torch.as_tensor(x).cuda().requires_grad_(True)
    y = lay(xg)
    y.backward(torch.as_tensor(dy).cuda())
    torch.cuda.synchronize()
    return y.detach().cpu(), xg.grad.cpu(), lay.weight.grad.cpu(), lay.bias.grad.cpu()


def _mode_a_view(lay):
    L = lay.layout
    idx, w, b = lay.indices.cpu(), lay.weight.detach().cpu(), lay.bias.detach().cpu()
    if L.shared_indices:
        return modeb_as_mode_a(L, idx, w, b)
    return idx, w, b


def _to_layout(L, dw, db):
    dwc = torch.from_numpy(np.asarray(dw)).reshape(L.groups, L.blocks_per_group, L.block, 8)
    dbc = torch.from_numpy(np.asarray(db)).reshape(L.groups, L.blocks_per_group, L.block)
    if L.packed:
        return L.pack_weights(dwc), L.pack_bias(dbc)
    return dwc, dbc


@pytest.mark.parametrize("name", max_case_names())
def test_matches_reference_golden(name):
    meta, arr = load_case(name)
    lay = _layer(meta["D"], meta["H"], meta["G"], meta["C"], meta["packed"], meta["seed"], meta["bias_std"],
                 meta["act"])
    assert lay.effective_policy == "save_winners"
    out = lay._runtime().forward(torch.from_numpy(arr["x"]).cuda(), lay.weight.detach(), lay.bias.detach(),
                                 track_ids=True)
    assert np.array_equal(out["winner"].cpu().numpy(), arr["winner"])
    y, dx, dw, db = _run(lay, arr["x"], arr["dy"])
    gs = arr["dw"].shape[0]
    assert_close(y, arr["y"], what="y", **FWD)
    assert_close(dx, arr["dx"], what="dx", **BWD)
    assert_close(dw[:gs], arr["dw"], what="dw", **BWD)
    assert_close(db[:gs], arr["db"], what="db", **BWD)


@pytest.mark.parametrize("C,packed", [(None, False), (8, True), (64, False)])
@pytest.mark.parametrize("policy", ["save_winners", "minimal_stats"])
@pytest.mark.parametrize("act", ["relu", "identity"])
def test_random_layers_against_oracle(C, packed, policy, act):
    D, H, G, B = 512, 20000, 10, 37
    lay = _layer(D, H, G, C, packed, seed=5, bias_std=0.2, act=act, policy=policy)
    gen = torch.Generator().manual_seed(7)
    x = torch.randn(B, D, generator=gen).numpy()
    dy = torch.randn(B, G, generator=gen).numpy()
    y, dx, dw, db = _run(lay, x, dy)
    assert lay.last_info["recomputed_stats"] == (policy == "minimal_stats")
    idx, w, b = _mode_a_view(lay)
    counts = lay.layout.counts_tensor("cpu").numpy()
    oy, win = P.max_forward(x, idx.numpy(), w.numpy(), b.numpy(), counts, act)
    odx, odw, odb = P.max_backward(x, idx.numpy(), w.numpy(), b.numpy(), counts, dy, act, winner=win)
    odw, odb = _to_layout(lay.layout, odw, odb)
    assert_close(y, oy, what="y", **FWD)
    assert_close(dx, odx, what="dx", **BWD)
    assert_close(dw, odw, what="dw", **BWD)
    assert_close(db, odb, what="db", **BWD)


def test_max_with_input_locality():
    """Windowed indices at D = 16384 take the locality path for max too."""
    from granulelayer_b200.layout import windowed_indices

    D, G, B = 16384, 2, 6
    lay = SparsePoolingLayer(D, G * 12288, G, shared_neurons=None, pooling={"type": "max", "activation": "relu"},
                             dtype=torch.float32, seed=3, bias_std=0.1)
    with torch.no_grad():
        lay.indices.copy_(windowed_indices(lay.layout, "cpu", window=512, supergroup=4096, seed=3))
    idx, w, b = lay.indices.clone(), lay.weight.detach().clone(), lay.bias.detach().clone()
    lay = lay.cuda()
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(B, D, generator=gen).numpy()
    dy = torch.randn(B, G, generator=gen).numpy()
    y, dx, dw, db = _run(lay, x, dy)
    assert lay._runtime().locality() is not None
    counts = lay.layout.counts_tensor("cpu").numpy()
    oy, win = P.max_forward(x, idx.numpy(), w.numpy(), b.numpy(), counts, "relu")
    odx, odw, odb = P.max_backward(x, idx.numpy(), w.numpy(), b.numpy(), counts, dy, "relu", winner=win)
    assert_close(y, oy, what="y", **FWD)
    assert_close(dx, odx, what="dx", **BWD)
    assert_close(dw, odw, what="dw", **BWD)
    assert_close(db, odb, what="db", **BWD)


def test_max_main_grad_accumulates():
    lay = _layer(256, 6000, 4, None, False, seed=2, bias_std=0.1, act="relu")
    lay.enable_main_grad()
    x = torch.randn(16, 256, generator=torch.Generator().manual_seed(3)).cuda()
    dy = torch.randn(16, 4, generator=torch.Generator().manual_seed(4)).cuda()
    lay(x).backward(dy)
    w1 = lay.weight.main_grad.clone()
    lay(x).backward(dy)
    assert_close(lay.weight.main_grad, 2 * w1.double(), what="main_grad", **BWD)
