"""Pin the CPU oracle to the reference: every golden fixture (made by the
reference's own code, tests/golden/make_golden.py) is reproduced by
oracle/oracle.py on the same seeded inputs."""
import numpy as np
import pytest
import torch

from conftest import (GOLDEN, assert_close, case_names, case_params, load_case, max_case_names, max_case_params,
                      oracle_params, smooth_case_names, topk_case_names,
                      modeb_as_mode_a, modeb_case_names, modeb_case_params)
from oracle import oracle as O


@pytest.mark.parametrize("name", case_names())
def test_oracle_matches_reference(name):
    meta, arr = load_case(name)
    L, idx, w, b = case_params(meta, arr)
    if meta["rule"] != "uniform":
        import hashlib

        assert hashlib.sha256(idx.numpy().tobytes()).hexdigest() == meta["idx_sha"]
        assert hashlib.sha256(w.numpy().tobytes()).hexdigest() == meta["w_sha"]
    counts = L.counts_tensor("cpu").numpy()
    x, dy = arr["x"], arr["dy"]
    pre = O.forward(x, idx.numpy(), w.numpy(), b.numpy(), counts, meta["pool"], meta["act"])
    # fixtures are float64 results rounded to float32: compare at float32 resolution
    assert_close(pre, arr["y"], 2e-6, 1e-7, "y")
    dx, dw, db = O.backward(x, idx.numpy(), w.numpy(), b.numpy(), counts, dy, meta["pool"], meta["act"])
    gs = arr["dw"].shape[0]
    assert_close(dx, arr["dx"], 2e-6, 1e-7, "dx")
    assert_close(dw[:gs], arr["dw"], 2e-6, 1e-7, "dw")
    assert_close(db[:gs], arr["db"], 2e-6, 1e-7, "db")


@pytest.mark.parametrize("tag", ["adam", "adamw"])
def test_oracle_adam_matches_torch(tag):
    d = np.load(GOLDEN / "adam.npz")
    p = d[f"{tag}_p0"].copy()
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    for s in range(5):
        p, m, v = O.adam_step(p, d[f"{tag}_g"][s], m, v, float(d["lr"]), float(d["beta1"]), float(d["beta2"]),
                              float(d["eps"]), float(d[f"{tag}_wd"]), s + 1)
        np.testing.assert_allclose(p, d[f"{tag}_p"][s], rtol=1e-12, atol=1e-14)
        np.testing.assert_allclose(m, d[f"{tag}_m"][s], rtol=1e-12, atol=1e-14)
        np.testing.assert_allclose(v, d[f"{tag}_v"][s], rtol=1e-12, atol=1e-14)


def test_oracle_sum_is_n_times_mean():
    meta, arr = load_case("cfg1_mean_relu")
    L, idx, w, b = case_params(meta, arr)
    c = L.counts_tensor("cpu").numpy()
    m = O.forward(arr["x"], idx.numpy(), w.numpy(), b.numpy(), c, "mean", "relu")
    s = O.forward(arr["x"], idx.numpy(), w.numpy(), b.numpy(), c, "sum", "relu")
    np.testing.assert_allclose(s, m * c[None, :], rtol=1e-12)


@pytest.mark.parametrize("name", modeb_case_names())
def test_oracle_matches_reference_mode_b(name):
    """Mode B (shared index records, canonical and fragment-packed storage): the oracle on the
    equivalent Mode-A tensors reproduces the reference's float64 outputs and gradients."""
    import hashlib

    meta, arr = load_case(name)
    L, idx, w, b = modeb_case_params(meta)
    assert hashlib.sha256(idx.numpy().tobytes()).hexdigest() == meta["idx_sha"]
    assert hashlib.sha256(w.numpy().tobytes()).hexdigest() == meta["w_sha"]
    ia, wa, ba = modeb_as_mode_a(L, idx, w, b)
    counts = L.counts_tensor("cpu").numpy()
    pre = O.forward(arr["x"], ia.numpy(), wa.numpy(), ba.numpy(), counts, meta["pool"], meta["act"])
    assert_close(pre, arr["y"], 2e-6, 1e-7, "y")
    dx, dw, db = O.backward(arr["x"], ia.numpy(), wa.numpy(), ba.numpy(), counts, arr["dy"], meta["pool"],
                            meta["act"])
    assert_close(dx, arr["dx"], 2e-6, 1e-7, "dx")
    # back to the layer's storage layout
    C = L.block
    dwc = torch.from_numpy(dw).reshape(L.groups, L.blocks_per_group, C, 8)
    dbc = torch.from_numpy(db).reshape(L.groups, L.blocks_per_group, C)
    if L.packed:
        dwc, dbc = L.pack_weights(dwc), L.pack_bias(dbc)
    gs = arr["dw"].shape[0]
    assert_close(dwc[:gs], arr["dw"], 2e-6, 1e-7, "dw")
    assert_close(dbc[:gs], arr["db"], 2e-6, 1e-7, "db")


@pytest.mark.parametrize("name", max_case_names())
def test_max_oracle_matches_reference(name):
    """Max pooling: the float64 oracle reproduces the reference's outputs, winners and gradients."""
    from oracle import pool_oracle as P

    meta, arr = load_case(name)
    L, idx, w, b = max_case_params(meta)
    if L.shared_indices:
        ia, wa, ba = modeb_as_mode_a(L, idx, w, b)
    else:
        ia, wa, ba = idx, w, b
    counts = L.counts_tensor("cpu").numpy()
    y, win = P.max_forward(arr["x"], ia.numpy(), wa.numpy(), ba.numpy(), counts, meta["act"])
    assert np.array_equal(win, arr["winner"])
    assert_close(y, arr["y"], 2e-6, 1e-7, "y")
    dx, dw, db = P.max_backward(arr["x"], ia.numpy(), wa.numpy(), ba.numpy(), counts, arr["dy"], meta["act"])
    assert_close(dx, arr["dx"], 2e-6, 1e-7, "dx")
    dwc = torch.from_numpy(dw).reshape(L.groups, L.blocks_per_group, L.block, 8)
    dbc = torch.from_numpy(db).reshape(L.groups, L.blocks_per_group, L.block)
    if L.packed:
        dwc, dbc = L.pack_weights(dwc), L.pack_bias(dbc)
    gs = arr["dw"].shape[0]
    assert_close(dwc[:gs], arr["dw"], 2e-6, 1e-7, "dw")
    assert_close(dbc[:gs], arr["db"], 2e-6, 1e-7, "db")


@pytest.mark.parametrize("name", smooth_case_names())
def test_smooth_oracle_matches_reference(name):
    """LogMeanExp / power mean / softmax-weighted: the float64 oracle reproduces the reference's
    outputs and gradients."""
    from oracle import pool_oracle as P

    meta, arr = load_case(name)
    L, idx, w, b = max_case_params(meta)
    if L.shared_indices:
        ia, wa, ba = modeb_as_mode_a(L, idx, w, b)
    else:
        ia, wa, ba = idx, w, b
    counts = L.counts_tensor("cpu").numpy()
    kw = oracle_params(meta)
    y = P.smooth_forward(arr["x"], ia.numpy(), wa.numpy(), ba.numpy(), counts, meta["pool"], meta["act"], **kw)
    assert_close(y, arr["y"], 2e-6, 1e-7, "y")
    dx, dw, db = P.smooth_backward(arr["x"], ia.numpy(), wa.numpy(), ba.numpy(), counts, arr["dy"], meta["pool"],
                                   meta["act"], **kw)
    assert_close(dx, arr["dx"], 2e-6, 1e-7, "dx")
    dwc = torch.from_numpy(dw).reshape(L.groups, L.blocks_per_group, L.block, 8)
    dbc = torch.from_numpy(db).reshape(L.groups, L.blocks_per_group, L.block)
    if L.packed:
        dwc, dbc = L.pack_weights(dwc), L.pack_bias(dbc)
    gs = arr["dw"].shape[0]
    assert_close(dwc[:gs], arr["dw"], 2e-6, 1e-7, "dw")
    assert_close(dbc[:gs], arr["db"], 2e-6, 1e-7, "db")


@pytest.mark.parametrize("name", topk_case_names())
def test_topk_oracle_matches_reference(name):
    """Top-K mean: the float64 oracle reproduces the reference's outputs, selected slots and
    gradients."""
    from oracle import pool_oracle as P

    meta, arr = load_case(name)
    L, idx, w, b = max_case_params(meta)
    if L.shared_indices:
        ia, wa, ba = modeb_as_mode_a(L, idx, w, b)
    else:
        ia, wa, ba = idx, w, b
    counts = L.counts_tensor("cpu").numpy()
    y, slots = P.topk_forward(arr["x"], ia.numpy(), wa.numpy(), ba.numpy(), counts, meta["k"], meta["act"])
    kk = np.minimum(counts, meta["k"])
    live = np.arange(meta["k"])[None, None, :] < kk[None, :, None]
    assert np.array_equal(np.where(live, slots, -1), np.where(live, arr["topk"], -1))
    assert_close(y, arr["y"], 2e-6, 1e-7, "y")
    dx, dw, db = P.topk_backward(arr["x"], ia.numpy(), wa.numpy(), ba.numpy(), counts, arr["dy"], meta["k"],
                                 meta["act"])
    assert_close(dx, arr["dx"], 2e-6, 1e-7, "dx")
    dwc = torch.from_numpy(dw).reshape(L.groups, L.blocks_per_group, L.block, 8)
    dbc = torch.from_numpy(db).reshape(L.groups, L.blocks_per_group, L.block)
    if L.packed:
        dwc, dbc = L.pack_weights(dwc), L.pack_bias(dbc)
    gs = arr["dw"].shape[0]
    assert_close(dwc[:gs], arr["dw"], 2e-6, 1e-7, "dw")
    assert_close(dbc[:gs], arr["db"], 2e-6, 1e-7, "db")
