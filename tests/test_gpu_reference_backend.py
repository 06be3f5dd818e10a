"""The maintainer-side binding ``granulelayer_b200/reference_backend.py``, plugged into the reference's
own ``SparsePoolingLayer`` / ``Level1Runtime`` at its backend call sites (sparse_pooling/autograd.py:221
forward, :267 backward), reproduces the golden fixtures the reference's float64 model made.

The reference package comes from ``baseline/_ref`` (an unmodified copy of the reference placed there for
the comparator arm of bench.py); the test is skipped where it is absent.  The reference layer is built
with ``backend="triton"`` so that its own native library is not touched; the test then sets
``B200Backend`` as the runtime's backend and makes ``resolve`` report "cuda", which is exactly the
wiring INTEGRATION.md describes.  Tolerances: forward rtol 1e-5 / atol 1e-6; dX, dW, db rtol 1e-4 /
atol 1e-5 (plus the oracle's ReLU-boundary slack)."""
import importlib
import sys
import types

import numpy as np
import pytest
import torch

from conftest import ROOT, assert_close, case_params, load_case, modeb_case_params
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REF = ROOT / "baseline" / "_ref"
FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


@pytest.fixture(scope="module")
def sp():
    if not (REF / "sparse_pooling" / "__init__.py").exists():
        pytest.skip("the reference package is not placed in baseline/_ref on this host")
    sys.path.insert(0, str(REF))
    try:
        return importlib.import_module("sparse_pooling")
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"the reference package does not import here: {type(e).__name__}: {e}")


@pytest.fixture(scope="module")
def backend():
    from granulelayer_b200 import reference_backend
    from granulelayer_b200._native import library_path

    return reference_backend.B200Backend(reference_backend.load_library(library_path()))


def _plug(lay, backend):
    """Route the reference layer's runtime to the B200 backend (the maintainer's wiring)."""
    rt = lay._runtime()
    rt.backend = backend
    cuda = types.SimpleNamespace(fwd={"backend": "cuda"}, bwd={"backend": "cuda"})
    rt.resolve = lambda B, part: cuda
    return rt


def _ref_layer(sp, meta, idx, w, b, C=None, packed=False):
    kw = dict(shared_neurons=C, weight_layout=("packed" if packed else "canonical") if C else "auto")
    lay = sp.SparsePoolingLayer(meta["D"], meta["H"], meta["G"], pooling={"type": "mean", "activation": meta["act"]},
                                dtype=torch.float32, device="cpu", seed=meta["seed"], bias_std=meta["bias_std"],
                                backend="triton", **kw)
    with torch.no_grad():
        lay.indices.copy_(idx)
        lay.weight.copy_(w)
        lay.bias.copy_(b)
    return lay.cuda()


def _step(lay, arr):
    x = torch.as_tensor(arr["x"]).cuda().requires_grad_(True)
    y = lay(x)
    (y * torch.as_tensor(arr["dy"]).cuda()).sum().backward()
    torch.cuda.synchronize()
    return y.detach().cpu(), x.grad.cpu(), lay.weight.grad.cpu(), lay.bias.grad.cpu()


@pytest.mark.parametrize("name", ["cfg1_mean_relu", "gelu_mean", "ragged_b37", "uniform_dup_idx"])
def test_mode_a_through_the_reference_runtime(sp, backend, name):
    meta, arr = load_case(name)
    L, idx, w, b = case_params(meta, arr)
    lay = _ref_layer(sp, meta, idx, w, b)
    rt = _plug(lay, backend)
    y, dx, dw, db = _step(lay, arr)
    assert rt.last_info["forward_backend"] == "cuda" and rt.last_info["backward_backend"] == "cuda"
    gs = arr["dw"].shape[0]
    _, _, _, sdx, sdw, sdb = O.backward(arr["x"], idx.numpy(), w.numpy(), b.numpy(), L.counts_tensor("cpu").numpy(),
                                        arr["dy"], "mean", meta["act"], slack=True)
    assert_close(y, arr["y"], what="y", **FWD)
    assert_close(dx, arr["dx"], what="dx", slack=sdx, **BWD)
    assert_close(dw[:gs], arr["dw"], what="dw", slack=sdw[:gs], **BWD)
    assert_close(db[:gs], arr["db"], what="db", slack=sdb[:gs], **BWD)


@pytest.mark.parametrize("name", ["modeb_c8", "modeb_c64_packed_ragged", "modeb_c16_gelu"])
def test_mode_b_through_the_reference_runtime(sp, backend, name):
    meta, arr = load_case(name)
    L, idx, w, b = modeb_case_params(meta)
    lay = _ref_layer(sp, meta, idx, w, b, C=meta["C"], packed=meta["packed"])
    rt = _plug(lay, backend)
    y, dx, dw, db = _step(lay, arr)
    assert rt.last_info["forward_backend"] == "cuda" and rt.last_info["backward_backend"] == "cuda"
    gs = arr["dw"].shape[0]
    assert_close(y, arr["y"], what="y", **FWD)
    assert_close(dx, arr["dx"], what="dx", **BWD)
    assert_close(dw[:gs], arr["dw"], what="dw", **BWD)
    assert_close(db[:gs], arr["db"], what="db", **BWD)


def test_unserved_layer_raises(sp, backend):
    meta, arr = load_case("cfg1_mean_relu")
    L, idx, w, b = case_params(meta, arr)
    lay = sp.SparsePoolingLayer(meta["D"], meta["H"], meta["G"], shared_neurons=None,
                                pooling={"type": "max", "activation": "relu"}, dtype=torch.float32, device="cpu",
                                seed=meta["seed"], backend="triton").cuda()
    _plug(lay, backend)
    with pytest.raises(NotImplementedError):
        lay(torch.as_tensor(np.asarray(arr["x"])).cuda())
