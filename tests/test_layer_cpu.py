"""Host-side behaviour of the drop-in layer (no GPU): construction, state dicts,
and loud refusal of anything off the B200 path (no CPU or Triton fallback)."""
import sys

import pytest
import torch

from granulelayer_b200 import FusedAdamW, PhysicalPlan, SparsePoolingLayer
from granulelayer_b200._native import NativeLibraryError
from granulelayer_b200.autograd import UnsupportedOnB200


def _layer(**kw):
    args = dict(shared_neurons=None, pooling="mean", dtype=torch.float32, seed=0)
    args.update(kw)
    return SparsePoolingLayer(64, 3000, 8, **args)


def test_shapes_and_repr():
    lay = _layer()
    assert lay.indices.shape == (8, 48, 8, 8) and lay.indices.dtype == torch.int16
    assert lay.weight.shape == (8, 48, 8, 8) and lay.bias.shape == (8, 48, 8)
    assert "A(independent)" in repr(lay) and "mean[relu]" in repr(lay)
    assert lay.effective_policy == "minimal_stats"


def test_cpu_forward_has_no_fallback():
    lay = _layer()
    with pytest.raises(NativeLibraryError):
        lay(torch.randn(4, 64))


@pytest.mark.parametrize("kw", [dict(shared_neurons=8), dict(shared_neurons=64, weight_layout="canonical")])
def test_mode_b_cpu_forward_has_no_fallback(kw):
    lay = _layer(**kw)
    with pytest.raises(NativeLibraryError):
        lay(torch.randn(2, 64))


@pytest.mark.parametrize("kw", [dict(dtype=torch.float16),
                                # 3 shards of 20 blocks do not tile the 48 stored blocks of a group
                                dict(pooling={"levels": [{"type": "mean", "neurons_per_shard": 160},
                                                         {"type": "weighted_sum"}]})])
def test_unsupported_configurations_raise(kw):
    lay = _layer(**kw)
    with pytest.raises(UnsupportedOnB200):
        lay(torch.randn(2, 64))


def test_main_grad_buffers():
    lay = _layer()
    lay.enable_main_grad()
    assert lay.weight.main_grad.dtype == torch.float32 and lay.weight.main_grad.shape == lay.weight.shape
    lay.weight.main_grad.fill_(1)
    lay.zero_main_grad()
    assert float(lay.weight.main_grad.abs().max()) == 0


def test_state_dict_roundtrip():
    a = _layer(seed=1)
    b = _layer(seed=2)
    assert not torch.equal(a.weight, b.weight)
    b.load_state_dict(a.state_dict())
    assert torch.equal(a.weight, b.weight) and torch.equal(a.indices, b.indices)
    assert set(a.state_dict()) == {"indices", "weight", "bias"}


def test_state_dict_interchanges_with_reference(reference_path):
    sys.path.insert(0, reference_path)
    from sparse_pooling import SparsePoolingLayer as RefLayer

    ref = RefLayer(64, 3000, 8, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=5, bias_std=0.1)
    ours = _layer(seed=5, bias_std=0.1)
    for k, v in ref.state_dict().items():
        assert torch.equal(v, ours.state_dict()[k]), f"{k} differs from the reference's seeded layer"
    ours2 = _layer(seed=9)
    ours2.load_state_dict(ref.state_dict())
    assert torch.equal(ours2.weight, ref.weight)


def test_optimizer_refuses_unsupported_modes():
    p = torch.nn.Parameter(torch.zeros(8, dtype=torch.float16))
    p.main_grad = torch.zeros(8)
    with pytest.raises(UnsupportedOnB200):
        FusedAdamW([p]).step()
    q = torch.nn.Parameter(torch.zeros(8, dtype=torch.bfloat16))   # supported, but only on the GPU
    q.main_grad = torch.zeros(8)
    with pytest.raises(NativeLibraryError):
        FusedAdamW([q], moments="bf16", master_weights=True).step()


def test_explain_on_cpu():
    assert "CPU" in _layer().explain()["backend"]


def test_plan_fields():
    lay = _layer(plan=PhysicalPlan(b200_fwd_tokens=4, b200_dx_tokens=2))
    assert lay.plan.b200_fwd_tokens == 4


def test_connectivity_layer_matches_reference(reference_path):
    """Input-supergroup connectivity (Mode B): the reference's layer and ours hold identical
    buffers (indices from the supergroup generator, sg_feat, sg_buckets, sg_plan) and parameters."""
    sys.path.insert(0, reference_path)
    from sparse_pooling import SparsePoolingLayer as RefLayer
    from sparse_pooling.supergroups import ConnectivityPlan as RefPlan

    from granulelayer_b200.supergroups import ConnectivityPlan

    for C, wl in ((8, "packed"), (64, "canonical")):
        kw = dict(shared_neurons=C, pooling="mean", dtype=torch.float32, seed=3, bias_std=0.1, weight_layout=wl)
        ref = RefLayer(256, 40000, 16, connectivity=RefPlan(64, 2, seed=5), **kw)
        ours = SparsePoolingLayer(256, 40000, 16, connectivity=ConnectivityPlan(64, 2, seed=5), **kw)
        rs, os_ = ref.state_dict(), ours.state_dict()
        assert set(rs) == set(os_) == {"indices", "weight", "bias", "sg_feat", "sg_buckets", "sg_plan"}
        for k in rs:
            assert torch.equal(rs[k], os_[k]), f"{k} differs (C={C}, {wl})"


def test_connectivity_state_dict_checks():
    from granulelayer_b200.supergroups import ConnectivityPlan

    kw = dict(shared_neurons=8, pooling="mean", dtype=torch.float32)
    a = SparsePoolingLayer(256, 20000, 8, connectivity=ConnectivityPlan(64, 2, seed=1), **kw)
    b = SparsePoolingLayer(256, 20000, 8, connectivity=ConnectivityPlan(64, 2, seed=2), **kw)
    plain = SparsePoolingLayer(256, 20000, 8, **kw)
    with pytest.raises(ValueError, match="connectivity"):
        b.load_state_dict(a.state_dict())
    with pytest.raises(ValueError, match="connectivity"):
        plain.load_state_dict(a.state_dict())
    c = SparsePoolingLayer(256, 20000, 8, connectivity=ConnectivityPlan(64, 2, seed=1), seed=9, **kw)
    c.load_state_dict(a.state_dict())
    assert torch.equal(c.weight, a.weight)
    with pytest.raises(ValueError):
        SparsePoolingLayer(256, 20000, 8, shared_neurons=None, connectivity=ConnectivityPlan(64, 2, seed=1))


SEMANTIC = {"levels": [{"type": "max", "neurons_per_shard": 128, "transform": "affine"}, {"type": "weighted_sum"}]}


def test_semantic_layer_parameters():
    """Two-level layers hold the reference's level-1 transform and level-2 weights (layer.py:90-101)."""
    lay = _layer(pooling=SEMANTIC)
    assert lay.num_shards == 3
    assert set(lay.state_dict()) == {"indices", "weight", "bias", "t_alpha", "t_beta", "t_v"}
    assert lay.t_alpha.shape == (8, 3) and float(lay.t_v.detach().sum()) == pytest.approx(8.0)
    with pytest.raises(NativeLibraryError):        # level 1 still runs only on the GPU kernels
        lay(torch.randn(2, 64))


def test_semantic_state_dict_interchanges_with_reference(reference_path):
    sys.path.insert(0, reference_path)
    from sparse_pooling import SparsePoolingLayer as RefLayer

    ref = RefLayer(64, 3000, 8, shared_neurons=None, pooling=SEMANTIC, dtype=torch.float32, seed=3, bias_std=0.1)
    ours = _layer(pooling=SEMANTIC, seed=3, bias_std=0.1)
    assert set(ref.state_dict()) == set(ours.state_dict())
    for k, v in ref.state_dict().items():
        assert torch.equal(v, ours.state_dict()[k]), k
