"""Layout partition and seeded initialisation: bit-exact with the reference.

Pins: tests/golden/init_hashes.json (sha256 of the reference's init_parameters
output, layout.py:204-251) and the reference's own partition tests
(tests/test_sparse_projection.py:13-51, 54-65).
"""
import hashlib
import json

import pytest
import torch

from conftest import GOLDEN
from granulelayer_b200.layout import SparseLayout, init_parameters

HASHES = json.loads((GOLDEN / "init_hashes.json").read_text())


def _sha(t):
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("case", HASHES, ids=lambda c: f"{c['layout']}-s{c['seed']}-{c['dtype']}")
def test_init_parameters_bit_exact(case):
    D, H, G, K, C, shared, packed = case["layout"]
    L = SparseLayout(D, H, G, K, C, shared, packed=packed)
    assert list(L.index_shape) == case["index_shape"]
    assert list(L.weight_shape) == case["weight_shape"]
    assert list(L.bias_shape) == case["bias_shape"]
    dtype = torch.float32 if case["dtype"] == "float32" else torch.bfloat16
    i, w, b = init_parameters(L, "cpu", dtype=dtype, seed=case["seed"], bias_std=case["bias_std"],
                              chunk_records=case["chunk_records"])
    if dtype == torch.bfloat16:
        w, b = w.view(torch.int16), b.view(torch.int16)
    assert _sha(i) == case["idx"], "indices differ from the reference"
    assert _sha(w) == case["w"], "weights differ from the reference"
    assert _sha(b) == case["b"], "bias differs from the reference"


@pytest.mark.parametrize("H,G,C", [(100_000_000, 1024, 8), (100_663_296, 4096, 8), (5000, 16, 8), (1000, 7, 16)])
def test_partition_enumerates_exactly_H(H, G, C):
    L = SparseLayout(1024, H, G, 8, C, False)
    counts = L.counts_tensor("cpu").long()
    offs = L.offsets_tensor("cpu")
    assert int(counts.sum()) == H
    assert int(offs[0]) == 0
    assert torch.equal(offs[1:], offs[:-1] + counts[:-1])
    assert int(counts.max() - counts.min()) <= 1
    assert L.slots_per_group >= L.max_group
    assert L.blocks_per_group % 4 == 0
    if H < 10**6:
        ids = L.global_ids("cpu")
        assert torch.equal(torch.sort(ids[ids >= 0]).values, torch.arange(H))


def test_baseline_layout_shapes():
    # the 100M-neuron layer of the measured configs: G = 4096 groups of 24,576 neurons, no padding
    L = SparseLayout(4096, 100_663_296, 4096, 8, 8, False)
    assert L.index_shape == (4096, 3072, 8, 8)
    assert L.weight_shape == (4096, 3072, 8, 8)
    assert L.bias_shape == (4096, 3072, 8)
    assert L.padding_fraction() == 0.0


@pytest.mark.parametrize("shared", [True, False])
def test_indices_distinct_sorted_and_padding_zero(shared):
    L = SparseLayout(64, 3001, 8, 8, 16, shared)
    idx, w, b = init_parameters(L, "cpu", seed=1, bias_std=0.5)
    flat = idx.reshape(-1, 8).long()
    inval = ~L.valid_mask("cpu")
    if not shared:
        flat = flat[~inval.reshape(-1)]
    assert int(flat.min()) >= 0 and int(flat.max()) < 64
    assert bool((flat[:, 1:] > flat[:, :-1]).all())
    assert bool((w.reshape(8, -1, 8)[inval] == 0).all())
    assert bool((b.reshape(8, -1)[inval] == 0).all())


@pytest.mark.parametrize("C", [8, 16, 32, 64])
def test_pack_unpack_roundtrip(C):
    Lp = SparseLayout(64, 7000, 8, 8, C, True, packed=True)
    L = Lp.canonical
    i, w, b = init_parameters(L, "cpu", seed=2, bias_std=0.1)
    ip, wp, bp = init_parameters(Lp, "cpu", seed=2, bias_std=0.1)
    assert torch.equal(Lp.unpack_weights(wp), w)
    assert torch.equal(Lp.unpack_bias(bp), b)
    assert torch.equal(Lp.unpack_indices(ip), i)
    assert torch.equal(Lp.pack_weights(w), wp)


def test_layout_validation():
    with pytest.raises(ValueError):
        SparseLayout(64, 100, 8, 7, 8, False)
    with pytest.raises(ValueError):
        SparseLayout(40000, 100, 8, 8, 8, False)
    with pytest.raises(ValueError):
        SparseLayout(64, 4, 8, 8, 8, False)
    with pytest.raises(ValueError):
        SparseLayout(64, 100, 8, 8, 8, False, packed=True)


def test_windowed_indices_rule():
    """Config-5 locality rule: sorted distinct records inside one window per supergroup; seeded."""
    from granulelayer_b200.layout import SparseLayout, windowed_indices

    L = SparseLayout(2048, 5000, 7, 8, 8, False)      # ragged groups: padding slots exist
    idx = windowed_indices(L, "cpu", window=128, supergroup=512, seed=4)
    assert idx.shape == L.index_shape and idx.dtype == torch.int16
    assert torch.equal(idx, windowed_indices(L, "cpu", window=128, supergroup=512, seed=4))
    assert not torch.equal(idx, windowed_indices(L, "cpu", window=128, supergroup=512, seed=5))
    counts = L.counts_tensor("cpu")
    valid = (torch.arange(L.blocks_per_group * 8)[None, :] < counts[:, None]).view(L.groups, L.blocks_per_group, 8)
    rec = idx[valid].long()
    assert rec.shape == (5000, 8)
    assert bool((rec[:, 1:] > rec[:, :-1]).all())
    assert int(idx[~valid].abs().max()) == 0
    sg = torch.arange(5000) // 512
    for s in range(int(sg.max()) + 1):
        r = rec[sg == s]
        assert int(r.max()) - int(r.min()) < 128 and int(r.min()) >= 0 and int(r.max()) < 2048
