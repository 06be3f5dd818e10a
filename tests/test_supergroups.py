"""Input-supergroup generator: bit-exact with the reference (tests/golden/graph_hashes.json, made by
sparse_pooling.supergroups.generate_indices and experimental/kgen_graph.generate) and structurally valid."""
import hashlib
import json

import pytest
import torch

from conftest import GOLDEN
from granulelayer_b200.layout import SparseLayout
from granulelayer_b200.supergroups import (ConnectivityPlan, generate_indices, generate_records, interleaved_order,
                                           unit_to_block_buckets, validate_records)

CASES = json.loads((GOLDEN / "graph_hashes.json").read_text())


def _sha(t):
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def _klayout_counts(D, H, G, K, C):
    base, rem = divmod(H, G)
    counts = (base + (torch.arange(G) < rem).to(torch.int64)).to(torch.int32)
    NB = -(-(base + (1 if rem else 0)) // C)
    return counts, NB


@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "mode_b"], ids=lambda c: str(c["layout"]))
def test_mode_b_indices_bit_exact(case):
    D, H, G, K, C, shared = case["layout"]
    L = SparseLayout(D, H, G, K, C, shared)
    plan = ConnectivityPlan(**case["plan"])
    idx, graph, _ = generate_indices(L, plan, "cpu")
    assert [list(idx.shape), list(graph.feat.shape), list(graph.buckets.shape)] == case["shapes"]
    assert _sha(idx) == case["idx"]
    assert _sha(graph.feat) == case["feat"]
    assert _sha(graph.buckets) == case["buckets"]


@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "kgen"], ids=lambda c: str(c["layout"]))
def test_generalized_graph_bit_exact_and_valid(case):
    D, H, G, K, C = case["layout"]
    plan = ConnectivityPlan(**case["plan"])
    counts, NB = _klayout_counts(D, H, G, K, C)
    rec, feat, ubk, _ = generate_records(D, counts, C, K, NB, 1, plan, "cpu")
    bk = unit_to_block_buckets(ubk, counts, C, 1)
    assert _sha(rec) == case["idx"] and _sha(feat) == case["feat"]
    assert _sha(ubk) == case["buckets"] and _sha(bk) == case["block_buckets"]
    rep = validate_records(D, counts, C, K, rec, feat, bk, plan.partition_rounds)
    assert rep["H"] == H


def test_plan_validation_and_json():
    p = ConnectivityPlan(64, 4, seed=3)
    assert ConnectivityPlan.from_json(p.to_json()) == p
    assert p.num_supergroups(1024) == 64
    with pytest.raises(ValueError):
        ConnectivityPlan(60, 1)
    with pytest.raises(ValueError):
        ConnectivityPlan(64, 0)
    with pytest.raises(ValueError):
        p.num_supergroups(1000)


def test_interleaved_order_is_a_permutation():
    o = interleaved_order(12, 3)
    assert sorted(o.tolist()) == list(range(12))
    assert o[:3].tolist() == [0, 4, 8]  # position p -> round p % R, set p // R


def test_against_live_reference(reference_path):
    """Same draws as the importable reference on a configuration not in the fixtures."""
    import sys

    sys.path.insert(0, reference_path)
    from sparse_pooling.layout import SparseLayout as RL
    from sparse_pooling.supergroups import ConnectivityPlan as RP, generate_indices as rgen

    for C, S, R, gen in ((16, 32, 2, "balanced_permutation"), (8, 16, 3, "independent_subsets")):
        ri, rg, _ = rgen(RL(128, 5000, 8, 8, C, True), RP(S, R, gen, 9), "cpu")
        mi, mg, _ = generate_indices(SparseLayout(128, 5000, 8, 8, C, True), ConnectivityPlan(S, R, gen, 9), "cpu")
        assert torch.equal(ri, mi) and torch.equal(rg.feat, mg.feat) and torch.equal(rg.buckets, mg.buckets)
