"""Bank-aware processing order (gl_group_order): a permutation of each group's slots that lowers
shared-memory bank conflicts, with forward/backward results unchanged within fp32 tolerance."""
import numpy as np
import pytest
import torch

from conftest import assert_close
from granulelayer_b200 import PhysicalPlan, SparsePoolingLayer, _native
from granulelayer_b200.layout import SparseLayout, init_parameters

pytestmark = pytest.mark.gpu


def _conflicts(idx, order, counts, unit):
    """Mean over units and inputs of the largest bank-group multiplicity (1 = conflict-free)."""
    tot, n = 0.0, 0
    for g in range(idx.shape[0]):
        rec = idx[g].reshape(-1, 8)[order[g][:counts[g]]] % unit
        m = (len(rec) // unit) * unit
        r = rec[:m].reshape(-1, unit, 8)
        for k in range(8):
            c = np.zeros((r.shape[0], unit), int)
            for j in range(unit):
                np.add.at(c, (np.arange(r.shape[0]), r[:, j, k]), 1)
            tot += c.max(1).sum()
            n += r.shape[0]
    return tot / n


@pytest.mark.parametrize("unit", [4, 8])
def test_order_is_a_permutation_and_lowers_conflicts(unit):
    L = SparseLayout(4096, 4 * 24576 + 100, 4, 8, 8, False)   # ragged: padding slots in the last groups
    idx, _, _ = init_parameters(L, "cuda", dtype=torch.float32, seed=7)
    counts = L.counts_tensor("cuda").to(torch.int32)
    slots = L.blocks_per_group * 8
    out = torch.full((L.groups, slots), -1, dtype=torch.int32, device="cuda")
    _native.group_order(idx, counts, L.input_dim, L.blocks_per_group, 0, L.groups, unit, out)
    o = out.cpu().numpy()
    c = counts.cpu().numpy()
    for g in range(L.groups):
        assert np.array_equal(np.sort(o[g][:c[g]]), np.arange(c[g])), "valid slots first, each once"
        assert np.array_equal(o[g][c[g]:], np.arange(c[g], slots)), "padding slots in place"
    ident = np.tile(np.arange(slots), (L.groups, 1))
    ic = idx.cpu().numpy().astype(np.int64)
    before, after = _conflicts(ic, ident, c, unit), _conflicts(ic, o, c, unit)
    assert after < 0.7 * before, (before, after)
    # deterministic
    out2 = torch.empty_like(out)
    _native.group_order(idx, counts, L.input_dim, L.blocks_per_group, 0, L.groups, unit, out2)
    assert torch.equal(out, out2)


def test_order_subrange_matches_full():
    L = SparseLayout(1024, 8 * 3000, 8, 8, 8, False)
    idx, _, _ = init_parameters(L, "cuda", dtype=torch.float32, seed=3)
    counts = L.counts_tensor("cuda").to(torch.int32)
    slots = L.blocks_per_group * 8
    full = torch.empty((8, slots), dtype=torch.int32, device="cuda")
    part = torch.empty((3, slots), dtype=torch.int32, device="cuda")
    _native.group_order(idx, counts, 1024, L.blocks_per_group, 0, 8, 8, full)
    _native.group_order(idx, counts, 1024, L.blocks_per_group, 2, 5, 8, part)
    assert torch.equal(full[2:5], part)


@pytest.mark.parametrize("accum", ["fixed", "fp32"])
def test_ordered_and_slot_order_agree(accum):
    D, H, G, B = 4096, 3 * 24576, 3, 40
    outs = []
    for mode in ("auto", "identity"):   # "auto" = the bank-aware order
        lay = SparsePoolingLayer(D, H, G, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=11,
                                 bias_std=0.1, plan=PhysicalPlan(b200_neuron_order=mode, b200_dx_accum=accum)).cuda()
        x = torch.randn(B, D, generator=torch.Generator().manual_seed(1)).cuda().requires_grad_(True)
        dy = torch.randn(B, G, generator=torch.Generator().manual_seed(2)).cuda()
        y = lay(x)
        y.backward(dy)
        outs.append((y.detach().cpu(), x.grad.cpu(), lay.weight.grad.cpu(), lay.bias.grad.cpu()))
    (ya, dxa, dwa, dba), (yb, dxb, dwb, dbb) = outs
    assert_close(ya, yb, rtol=1e-5, atol=1e-6, what="y")
    assert_close(dxa, dxb, rtol=1e-4, atol=1e-5, what="dx")
    assert_close(dwa, dwb, rtol=1e-4, atol=1e-5, what="dw")
    assert_close(dba, dbb, rtol=1e-4, atol=1e-5, what="db")


def test_order_rejects_bad_unit():
    L = SparseLayout(256, 1000, 2, 8, 8, False)
    idx, _, _ = init_parameters(L, "cuda", dtype=torch.float32, seed=1)
    counts = L.counts_tensor("cuda").to(torch.int32)
    out = torch.empty((2, L.blocks_per_group * 8), dtype=torch.int32, device="cuda")
    with pytest.raises(_native.NativeLibraryError):
        _native.group_order(idx, counts, 256, L.blocks_per_group, 0, 2, 16, out)


def _single_rank_group():
    import socket

    import torch.distributed as dist

    if not dist.is_initialized():
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        dist.init_process_group("gloo", rank=0, world_size=1, init_method=f"tcp://127.0.0.1:{port}")
    return dist


def test_bank_ordered_shard_matches_layer():
    """A GPU shard stores its neurons in bank-aware order; outputs, dX and the slot-order dW/db
    equal the drop-in layer's, and the stored parameters are a per-group permutation."""
    from granulelayer_b200.distributed import GroupShardedLayer

    dist = _single_rank_group()
    try:
        D, H, G, B = 4096, 3 * 24576 + 100, 3, 24
        full = SparsePoolingLayer(D, H, G, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=5,
                                  bias_std=0.1).cuda()
        shard = GroupShardedLayer.from_full(full)
        assert shard.neuron_order is not None, "shards built from GPU tensors are stored in bank order"
        ci, cw, cb = shard.canonical_shard()
        assert torch.equal(ci, full.indices) and torch.equal(cw, full.weight) and torch.equal(cb, full.bias)
        assert not torch.equal(shard.indices, full.indices)
        sd = shard.full_state_dict()
        for k, v in full.state_dict().items():
            assert torch.equal(sd[k], v), f"{k}: gathered shard state differs from the single-GPU layer"
        x = torch.randn(B, D, generator=torch.Generator().manual_seed(1)).cuda()
        dy = torch.randn(B, G, generator=torch.Generator().manual_seed(2)).cuda()
        outs = []
        for lay in (full, shard):
            xr = x.clone().requires_grad_(True)
            y = lay(xr)
            y.backward(dy)
            gw = lay.weight.grad if lay is full else shard.canonical(lay.weight.grad)
            gb = lay.bias.grad if lay is full else shard.canonical(lay.bias.grad)
            outs.append((y.detach(), xr.grad, gw, gb))
        for what, a, b, tol in zip(("y", "dx", "dw", "db"), outs[1], outs[0],
                                   (dict(rtol=1e-5, atol=1e-6),) + (dict(rtol=1e-4, atol=1e-5),) * 3):
            assert_close(a, b, what=what, **tol)
    finally:
        dist.destroy_process_group()
