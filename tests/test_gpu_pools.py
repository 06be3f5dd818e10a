"""LogMeanExp, power-mean and softmax-weighted pooling on the GPU (Mode A and Mode B): the
forwards' online states and the dense backward from the reference's coefficients, against the
reference's float64 fixtures (tests/golden/fwdbwd_smooth_*.npz) and the float64 oracle
(oracle/pool_oracle.py).  Tolerances: forward rtol 1e-5 / atol 1e-6; dX, dW, db rtol 1e-4 /
atol 1e-5."""
import numpy as np
import pytest
import torch

from conftest import assert_close, load_case, modeb_as_mode_a, oracle_params, smooth_case_names
from granulelayer_b200 import PhysicalPlan, SparsePoolingLayer
from oracle import pool_oracle as P

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def _layer(D, H, G, C, packed, seed, bias_std, pooling, policy="auto", plan=None):
    return SparsePoolingLayer(D, H, G, shared_neurons=C, weight_layout="packed" if packed else "canonical",
                              pooling=pooling, checkpoint_policy=policy, dtype=torch.float32, seed=seed,
                              bias_std=bias_std, plan=plan).cuda()


def _run(lay, x, dy):
    xg = torch.as_tensor(x).cuda().requires_grad_(True)
    y = lay(xg)
    y.backward(torch.as_tensor(dy).cuda())
    torch.cuda.synchronize()
    return y.detach().cpu(), xg.grad.cpu(), lay.weight.grad.cpu(), lay.bias.grad.cpu()


def _oracle(lay, x, dy, kind, act, **kw):
    L = lay.layout
    idx, w, b = lay.indices.cpu(), lay.weight.detach().cpu(), lay.bias.detach().cpu()
    if L.shared_indices:
        idx, w, b = modeb_as_mode_a(L, idx, w, b)
    counts = L.counts_tensor("cpu").numpy()
    y = P.smooth_forward(x, idx.numpy(), w.numpy(), b.numpy(), counts, kind, act, **kw)
    dx, dw, db = P.smooth_backward(x, idx.numpy(), w.numpy(), b.numpy(), counts, dy, kind, act, **kw)
    dwc = torch.from_numpy(dw).reshape(L.groups, L.blocks_per_group, L.block, 8)
    dbc = torch.from_numpy(db).reshape(L.groups, L.blocks_per_group, L.block)
    if L.packed:
        dwc, dbc = L.pack_weights(dwc), L.pack_bias(dbc)
    return y, dx, dwc, dbc


@pytest.mark.parametrize("name", smooth_case_names())
def test_matches_reference_golden(name):
    meta, arr = load_case(name)
    pooling = dict(type=meta["pool"], activation=meta["act"], **meta["params"])
    lay = _layer(meta["D"], meta["H"], meta["G"], meta["C"], meta["packed"], meta["seed"], meta["bias_std"], pooling)
    y, dx, dw, db = _run(lay, arr["x"], arr["dy"])
    gs = arr["dw"].shape[0]
    assert_close(y, arr["y"], what="y", **FWD)
    assert_close(dx, arr["dx"], what="dx", **BWD)
    assert_close(dw[:gs], arr["dw"], what="dw", **BWD)
    assert_close(db[:gs], arr["db"], what="db", **BWD)


POOLS = [
    ("logmeanexp", {"temperature": 0.7}, "identity"),
    ("logmeanexp", {"temperature": 3.0}, "gelu"),
    ("power_mean", {"p": 2.0}, "relu"),
    ("power_mean", {"p": 2.5}, "relu"),
    ("power_mean", {"p": 8.0}, "relu"),
    ("softmax_weighted", {"beta": 1.3}, "identity"),
    ("softmax_weighted", {"beta": 0.4}, "relu"),
]


@pytest.mark.parametrize("C,packed", [(None, False), (8, True), (64, False)])
@pytest.mark.parametrize("kind,params,act", POOLS)
def test_random_layers_against_oracle(C, packed, kind, params, act):
    D, H, G, B = 512, 20000, 10, 37
    lay = _layer(D, H, G, C, packed, seed=5, bias_std=0.2, pooling=dict(type=kind, activation=act, **params))
    gen = torch.Generator().manual_seed(7)
    x = torch.randn(B, D, generator=gen).numpy()
    dy = torch.randn(B, G, generator=gen).numpy()
    y, dx, dw, db = _run(lay, x, dy)
    kw = oracle_params({"params": params})
    oy, odx, odw, odb = _oracle(lay, x, dy, kind, act, **kw)
    assert_close(y, oy, what="y", **FWD)
    assert_close(dx, odx, what="dx", **BWD)
    assert_close(dw, odw, what="dw", **BWD)
    assert_close(db, odb, what="db", **BWD)


@pytest.mark.parametrize("tokens", [1, 2, 4, 8])
def test_token_tiles(tokens):
    """Every forward token tile of both modes gives the same pooled values."""
    plan = PhysicalPlan(b200_fwd_tokens=tokens, b200_dx_tokens=min(tokens, 8))
    D, H, G, B = 300, 9000, 6, 21
    gen = torch.Generator().manual_seed(tokens)
    x = torch.randn(B, D, generator=gen).numpy()
    dy = torch.randn(B, G, generator=gen).numpy()
    for C, packed in ((None, False), (16, True)):
        lay = _layer(D, H, G, C, packed, seed=3, bias_std=0.1,
                     pooling=dict(type="softmax_weighted", beta=0.9, activation="identity"), plan=plan)
        y, dx, dw, db = _run(lay, x, dy)
        oy, odx, odw, odb = _oracle(lay, x, dy, "softmax_weighted", "identity", beta=0.9)
        assert_close(y, oy, what="y", **FWD)
        assert_close(dx, odx, what="dx", **BWD)
        assert_close(dw, odw, what="dw", **BWD)


@pytest.mark.parametrize("policy", ["minimal_stats", "recompute_stats"])
def test_softmax_checkpoint_policies(policy):
    """minimal_stats keeps the log2-normaliser from the forward; recompute_stats recomputes it in the
    backward (autograd.py:246-261, 364-377); both give the same gradients."""
    lay = _layer(256, 6000, 4, None, False, seed=2, bias_std=0.1,
                 pooling=dict(type="softmax_weighted", beta=1.1, activation="identity"), policy=policy)
    x = torch.randn(16, 256, generator=torch.Generator().manual_seed(3))
    dy = torch.randn(16, 4, generator=torch.Generator().manual_seed(4))
    y, dx, dw, db = _run(lay, x.numpy(), dy.numpy())
    assert lay.last_info["recomputed_stats"] == (policy == "recompute_stats")
    oy, odx, odw, odb = _oracle(lay, x.numpy(), dy.numpy(), "softmax_weighted", "identity", beta=1.1)
    assert_close(dx, odx, what="dx", **BWD)
    assert_close(dw, odw, what="dw", **BWD)


def test_power_mean_all_zero_group():
    """A group whose activations are all zero pools to 0 and passes no gradient (ops.py:211-217, 254-258)."""
    lay = _layer(64, 1600, 2, None, False, seed=1, bias_std=0.0, pooling=dict(type="power_mean", p=2.0))
    with torch.no_grad():
        lay.bias.view(2, -1)[0] = -1e4       # group 0: every z < 0
    x = torch.randn(5, 64, generator=torch.Generator().manual_seed(1)).numpy()
    dy = np.ones((5, 2), np.float32)
    y, dx, dw, db = _run(lay, x, dy)
    assert float(y[:, 0].abs().max()) == 0.0
    assert float(lay.weight.grad.view(2, -1)[0].abs().max()) == 0.0
    oy, odx, _, _ = _oracle(lay, x, dy, "power_mean", "relu", p=2.0)
    assert_close(y, oy, what="y", **FWD)
    assert_close(dx, odx, what="dx", **BWD)
