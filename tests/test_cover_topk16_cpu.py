"""Cover-TopK/16 construction on the CPU: envelope graph, support selection, lowering and persistence
are bit-exact with the reference (sparse_pooling/cover_topk16.py); structural properties of the support
(the reference's tests/test_cover_topk16.py:104-141)."""
import sys

import pytest
import torch

from granulelayer_b200.cover_topk16 import CoverTopK16Layer
from granulelayer_b200.kgen import KLayout, init_envelope_parameters
from granulelayer_b200.supergroups import ConnectivityPlan

SMALL = dict(input_dim=256, hidden_dim=3452, output_dim=8)


def _envelope(D=256, H=3452, G=8, C=256, seed=1):
    L = KLayout(D, H, G, 64, C)
    w, b = init_envelope_parameters(L, "cpu", dtype=torch.bfloat16, seed=seed, bias_std=0.1)
    return w, b


@pytest.mark.parametrize("norm", ["none", "energy"])
@pytest.mark.parametrize("shape", [(256, 3452, 8, 16), (512, 20000, 16, 16), (256, 6000, 4, 8)])
def test_bit_exact_with_reference(reference_path, norm, shape):
    sys.path.insert(0, reference_path)
    from sparse_pooling.cover_topk16 import CoverTopK16Layer as RefLayer
    from sparse_pooling.supergroups import ConnectivityPlan as RefPlan

    D, H, G, R = shape
    w, b = _envelope(D, H, G)
    ref = RefLayer.from_envelope(w, b, input_dim=D, hidden_dim=H, output_dim=G, connectivity=RefPlan(64, R, seed=4),
                                 normalization=norm, device="cpu")
    ours = CoverTopK16Layer.from_envelope(w, b, input_dim=D, hidden_dim=H, output_dim=G,
                                          connectivity=ConnectivityPlan(64, R, seed=4), normalization=norm,
                                          device="cpu")
    rs, os_ = ref.state_dict(), ours.state_dict()
    assert set(rs) == set(os_)
    for k in rs:
        if k in ("weight", "bias"):
            assert torch.equal(rs[k].float(), os_[k]), f"{k} differs"   # BF16 values held exactly in fp32
        else:
            assert torch.equal(rs[k], os_[k]), f"{k} differs"
    assert ref.cover_meta["support_fingerprint"] == ours.cover_meta["support_fingerprint"]
    assert ref.cover_meta["valid_slots"] == ours.cover_meta["valid_slots"] == 16 * H
    assert ref.cover_meta["support_stats"]["repair"]["swaps"] == ours.cover_meta["support_stats"]["repair"]["swaps"]


def test_support_structure():
    w, b = _envelope()
    lay = CoverTopK16Layer.from_envelope(w, b, connectivity=ConnectivityPlan(64, 16, seed=0), device="cpu",
                                         **SMALL)
    L = lay.layout
    assert L.fan_in == 16 and L.block == 16
    idx = lay.indices.view(-1, 16).long()
    assert bool((idx[:, 1:] > idx[:, :-1]).all()), "records are sorted and distinct"
    assert int(idx.max()) < SMALL["input_dim"]
    # every record's inputs lie in its set
    feat = lay.sg_feat.long()
    env = lay.env.long()
    valid = lay.weight.view(-1, 16, 16).abs().sum((1, 2)) > 0
    bk = lay.kg_buckets.long()
    q_of = torch.full((L.groups * L.blocks_per_group,), -1, dtype=torch.long)
    for q, g, j0, n in bk.tolist():
        q_of[g * L.blocks_per_group + j0: g * L.blocks_per_group + j0 + n] = q
    rows = torch.nonzero(valid).squeeze(1)
    assert bool((feat[q_of[rows][:, None], env[rows]] == idx[rows]).all())
    # coverage: every input of each original K64 record is kept by >= 1 of its 16 row groups
    assert lay.cover_meta["support_stats"]["repair"]["swaps"] >= 0
    assert lay.cover_meta["valid_slots"] == 16 * SMALL["hidden_dim"]


def test_save_load_packed_roundtrip(tmp_path):
    w, b = _envelope()
    lay = CoverTopK16Layer.from_envelope(w, b, connectivity=ConnectivityPlan(64, 16, seed=0), device="cpu",
                                         **SMALL)
    info = lay.save_packed(tmp_path / "ct16.pt")
    back = CoverTopK16Layer.load_packed(info["path"], device="cpu")
    for k, v in lay.state_dict().items():
        assert torch.equal(v, back.state_dict()[k])
    assert back.cover_meta["support_fingerprint"] == lay.cover_meta["support_fingerprint"]
    blob = torch.load(info["path"], weights_only=True)
    blob["state"]["indices"][0, 0, 0] += 1
    torch.save(blob, tmp_path / "bad.pt")
    with pytest.raises(ValueError):
        CoverTopK16Layer.load_packed(tmp_path / "bad.pt", device="cpu")


def test_rejects_bad_inputs():
    w, b = _envelope()
    with pytest.raises(ValueError):
        CoverTopK16Layer.from_envelope(w.float(), b.float(), connectivity=ConnectivityPlan(64, 16), device="cpu",
                                       **SMALL)
    with pytest.raises(ValueError):
        CoverTopK16Layer.from_envelope(w, b, connectivity=ConnectivityPlan(32, 16), device="cpu", **SMALL)
    with pytest.raises(ValueError):
        CoverTopK16Layer.from_envelope(w, b, connectivity=ConnectivityPlan(64, 16), normalization="fanin",
                                       device="cpu", **SMALL)


def test_kernel_family_follows_dtype_and_plan():
    """fp32 layers run the split tensor-core entries unless the plan turns them off; bf16 layers always run
    the bf16 tensor-core entries (the routing itself; the kernels are covered by the GPU tests)."""
    from granulelayer_b200 import _native
    from granulelayer_b200.config import PhysicalPlan

    w, b = _envelope()
    kw = dict(connectivity=ConnectivityPlan(64, 16, seed=0), device="cpu", **SMALL)
    f32 = CoverTopK16Layer.from_envelope(w, b, **kw)
    off = CoverTopK16Layer.from_envelope(w, b, plan=PhysicalPlan(b200_f32_tensor_cores="off"), **kw)
    b16 = CoverTopK16Layer.from_envelope(w, b, plan=PhysicalPlan(b200_f32_tensor_cores="off"),
                                         dtype=torch.bfloat16, **kw)
    assert f32.tensor_cores and not off.tensor_cores and b16.tensor_cores
    assert [_native._k16_entry(f32.weight, f32.tensor_cores, bwd) for bwd in (False, True)] == \
        ["gl_k16_fwd_tc_f32", "gl_k16_bwd_tc_f32"]
    assert [_native._k16_entry(off.weight, off.tensor_cores, bwd) for bwd in (False, True)] == \
        ["gl_k16_fwd_f32", "gl_k16_bwd_f32"]
    assert [_native._k16_entry(b16.weight, b16.tensor_cores, bwd) for bwd in (False, True)] == \
        ["gl_k16_fwd_tc", "gl_k16_bwd_tc"]
    # S = 64 sets: the tensor-core layers' forward runs on tcgen05 when the plan asks for it
    assert not f32.tcgen05 and not b16.tcgen05 and not off.tcgen05
    t5 = CoverTopK16Layer.from_envelope(w, b, plan=PhysicalPlan(b200_tcgen05="on"), **kw)
    t5simt = CoverTopK16Layer.from_envelope(w, b, plan=PhysicalPlan(b200_tcgen05="on", b200_f32_tensor_cores="off"),
                                            **kw)
    assert t5.tcgen05 and not t5simt.tcgen05
    assert t5.tcgen05_bwd and not t5simt.tcgen05_bwd and not f32.tcgen05_bwd
    fwd_only = CoverTopK16Layer.from_envelope(w, b, plan=PhysicalPlan(b200_tcgen05="fwd"), **kw)
    bwd_only = CoverTopK16Layer.from_envelope(w, b, plan=PhysicalPlan(b200_tcgen05="bwd"), **kw)
    assert (fwd_only.tcgen05, fwd_only.tcgen05_bwd, bwd_only.tcgen05, bwd_only.tcgen05_bwd) == (True, False, False, True)
    with pytest.raises(ValueError):
        PhysicalPlan(b200_tcgen05="auto")
    with pytest.raises(ValueError):
        PhysicalPlan(b200_f32_tensor_cores="split")
    with pytest.raises(_native.NativeLibraryError):      # no CPU fallback on this path
        f32(torch.randn(2, SMALL["input_dim"]))
