"""Two-level (semantic) pooling on the GPU: level-1 shards on the B200 kernels, the transform and
level-2 operator in PyTorch, against the reference's float64 results
(tests/golden/fwdbwd_semantic_*.npz, made by its reference_forward with autograd), including the
gradients of the transform and weighted-sum parameters.  Tolerances: forward rtol 1e-5 /
atol 1e-6; gradients rtol 1e-4 / atol 1e-5."""
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN, assert_close, load_case
from granulelayer_b200 import SparsePoolingLayer

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def _names():
    return sorted(p.stem[len("fwdbwd_"):] for p in GOLDEN.glob("fwdbwd_semantic_*.npz"))


def _layer(meta, arr):
    pooling = {"levels": meta["levels"], "level1_checkpoint": meta["level1_checkpoint"]}
    lay = SparsePoolingLayer(meta["D"], meta["H"], meta["G"], shared_neurons=meta["C"],
                             weight_layout="packed" if meta["packed"] else "canonical", pooling=pooling,
                             dtype=torch.float32, seed=meta["seed"], bias_std=meta["bias_std"])
    with torch.no_grad():
        for n in lay._tnames:
            getattr(lay, "t_" + n).copy_(torch.from_numpy(arr["t_" + n]))
    return lay.cuda()


@pytest.mark.parametrize("name", _names())
def test_matches_reference_golden(name):
    meta, arr = load_case(name)
    lay = _layer(meta, arr)
    xg = torch.from_numpy(arr["x"]).cuda().requires_grad_(True)
    y = lay(xg)
    y.backward(torch.from_numpy(arr["dy"]).cuda())
    torch.cuda.synchronize()
    gs = arr["dw"].shape[0]
    assert_close(y.detach().cpu(), arr["y"], what="y", **FWD)
    assert_close(xg.grad.cpu(), arr["dx"], what="dx", **BWD)
    assert_close(lay.weight.grad.cpu()[:gs], arr["dw"], what="dw", **BWD)
    assert_close(lay.bias.grad.cpu()[:gs], arr["db"], what="db", **BWD)
    for n in lay._tnames:
        assert_close(getattr(lay, "t_" + n).grad.cpu(), arr["dt_" + n], what="d" + n, **BWD)
    assert lay.last_info["recomputed_stats"] == (meta["level1_checkpoint"] == "recompute")


def test_shards_match_single_level_groups():
    """Level 1 of a two-level layer pools the same neurons a single-level layer with S times the
    groups would: mean over 128-neuron shards equals a mean layer whose groups are the shards."""
    D, G, S, nps = 128, 4, 4, 128
    two = SparsePoolingLayer(D, G * S * nps, G, shared_neurons=None, dtype=torch.float32, seed=2, bias_std=0.1,
                             pooling={"levels": [{"type": "mean", "neurons_per_shard": nps},
                                                 {"type": "weighted_sum"}]})
    one = SparsePoolingLayer(D, G * S * nps, G * S, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=2)
    with torch.no_grad():
        one.indices.copy_(two.indices.reshape(one.indices.shape))
        one.weight.copy_(two.weight.reshape(one.weight.shape))
        one.bias.copy_(two.bias.reshape(one.bias.shape))
        two.t_v.zero_()
        two.t_v[:, 1] = 1.0      # y[:, g] = F[:, g, 1]
    two, one = two.cuda(), one.cuda()
    x = torch.randn(9, D, generator=torch.Generator().manual_seed(1)).cuda()
    y1 = one(x).view(9, G, S)[:, :, 1]
    assert torch.equal(two(x), y1)
