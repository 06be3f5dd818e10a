import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the sm_100a library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def rel_err(a, b) -> float:
    """Relative L2 error ||a - b|| / ||b|| (the reference's metric, tests/conftest.py:53-55)."""
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / (b.norm() + 1e-30))


def assert_close(actual, expected, rtol, atol, what="", slack=None):
    """Elementwise |a - e| <= atol + rtol |e| (+ slack) — the hot path's parity bar.

    ``slack`` (from ``oracle.backward(..., slack=True)``) admits, element by element,
    exactly the contributions of (token, neuron) pairs sitting on ReLU's jump at 0,
    where fp32 and float64 evaluations of z may take different sides."""
    a = torch.as_tensor(actual).double().cpu()
    e = torch.as_tensor(expected).double().cpu()
    assert a.shape == e.shape, f"{what}: shape {tuple(a.shape)} != {tuple(e.shape)}"
    lim = atol + rtol * e.abs()
    if slack is not None:
        lim = lim + torch.as_tensor(slack).double().cpu() * (1 + 1e-6)
    bad = (a - e).abs() > lim
    if bool(bad.any()):
        i = int(bad.flatten().nonzero()[0])
        raise AssertionError(f"{what}: {int(bad.sum())} of {a.numel()} elements outside rtol={rtol} atol={atol}; "
                             f"first at flat {i}: {a.flatten()[i].item()!r} vs {e.flatten()[i].item()!r}")


def load_case(name):
    d = np.load(GOLDEN / f"fwdbwd_{name}.npz")
    meta = json.loads(str(d["meta"]))
    return meta, {k: d[k] for k in d.files if k != "meta"}


def case_names():
    """Mode-A golden cases."""
    return sorted(p.stem[len("fwdbwd_"):] for p in GOLDEN.glob("fwdbwd_*.npz")
                  if not p.stem.startswith(("fwdbwd_modeb_", "fwdbwd_max_", "fwdbwd_smooth_", "fwdbwd_semantic_",
                                             "fwdbwd_topk_")))


def max_case_names():
    """Max-pooling golden cases (Mode A and Mode B)."""
    return sorted(p.stem[len("fwdbwd_"):] for p in GOLDEN.glob("fwdbwd_max_*.npz"))


def topk_case_names():
    """Top-K mean golden cases (Mode A and Mode B)."""
    return sorted(p.stem[len("fwdbwd_"):] for p in GOLDEN.glob("fwdbwd_topk_*.npz"))


def smooth_case_names():
    """LogMeanExp / power-mean / softmax-weighted golden cases (Mode A and Mode B)."""
    return sorted(p.stem[len("fwdbwd_"):] for p in GOLDEN.glob("fwdbwd_smooth_*.npz"))


def oracle_params(meta):
    """Keyword arguments of oracle/pool_oracle.py for a golden case's pooling parameters."""
    prm = meta.get("params", {})
    return {{"temperature": "tau", "beta": "beta", "p": "p"}[k]: v for k, v in prm.items()}


def max_case_params(meta):
    """(layout, idx, w, b) of a max- or smooth-pooling golden case in the layer's storage layout."""
    from granulelayer_b200.layout import SparseLayout, init_parameters

    C = meta["C"]
    L = SparseLayout(meta["D"], meta["H"], meta["G"], 8, C or 8, C is not None, packed=meta["packed"])
    idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=meta["seed"], bias_std=meta["bias_std"])
    return L, idx, w, b


def modeb_case_names():
    """Mode-B golden cases (shared index records, canonical or fragment-packed storage)."""
    return sorted(p.stem[len("fwdbwd_"):] for p in GOLDEN.glob("fwdbwd_modeb_*.npz"))


def modeb_case_params(meta):
    """(layout, idx, w, b) of a Mode-B golden case in the layer's storage layout, from the seeded init."""
    from granulelayer_b200.layout import SparseLayout, init_parameters

    L = SparseLayout(meta["D"], meta["H"], meta["G"], 8, meta["C"], True, packed=meta["packed"])
    idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=meta["seed"], bias_std=meta["bias_std"])
    return L, idx, w, b


def modeb_as_mode_a(L, idx, w, b):
    """A Mode-B layer written as the equivalent Mode-A tensors (each block's index record repeated
    for its C neurons; C-neuron blocks split into blocks of 8) for the Mode-A oracle."""
    idx, w, b = L.to_canonical(idx, w, b)
    G, NB, C = L.groups, L.blocks_per_group, L.block
    ia = idx[:, :, None, :].expand(G, NB, C, 8).reshape(G, NB * C // 8, 8, 8).contiguous()
    return ia, w.reshape(G, NB * C // 8, 8, 8).contiguous(), b.reshape(G, NB * C // 8, 8).contiguous()


def case_params(meta, arrays):
    """(layout, idx, w, b) of a golden case, regenerated with the product's seeded init."""
    from granulelayer_b200.layout import SparseLayout, init_parameters

    L = SparseLayout(meta["D"], meta["H"], meta["G"], 8, 8, False)
    idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=meta["seed"], bias_std=meta["bias_std"])
    if meta["rule"] == "uniform":
        idx = torch.from_numpy(arrays["idx"])
    return L, idx, w, b


@pytest.fixture
def reference_path():
    """Directory holding the reference's sparse_pooling package, when present
    (GRANULE_REFERENCE); tests that need it are skipped elsewhere."""
    p = os.environ.get("GRANULE_REFERENCE", "")
    cand = [p] if p else []
    cand.append(str(ROOT.parent / "reference"))
    for c in cand:
        if c and (Path(c) / "sparse_pooling" / "__init__.py").exists():
            return c
    pytest.skip("reference package not available on this host")
