"""Configuration surface behaves like the reference's (sparse_pooling/config.py)."""
import sys

import pytest
import torch

from granulelayer_b200.config import LevelSpec, PhysicalPlan, PoolingConfig, resolve_reduction


def test_defaults_and_aliases():
    assert LevelSpec("mean").activation == "relu"          # config.py:45
    assert LevelSpec("mean").out_activation == "identity"
    assert LevelSpec("max").out_activation == "relu"        # config.py:52
    s = LevelSpec("mean_relu")
    assert (s.type, s.activation) == ("mean", "relu")
    assert LevelSpec("sum").activation == "relu"
    assert LevelSpec("lme").type == "logmeanexp"


def test_validation_errors():
    with pytest.raises(ValueError):
        LevelSpec("nope")
    with pytest.raises(ValueError):
        LevelSpec("mean", activation="tanh")
    with pytest.raises(ValueError):
        LevelSpec("topk_mean", k=3)
    with pytest.raises(ValueError):
        LevelSpec("power_mean", activation="identity")
    with pytest.raises(ValueError):
        PoolingConfig([LevelSpec("mean", neurons_per_shard=64)])
    with pytest.raises(ValueError):
        PoolingConfig([LevelSpec("weighted_sum")])
    with pytest.raises(ValueError):
        PhysicalPlan(reduction="nope")
    with pytest.raises(ValueError):
        PhysicalPlan(b200_fwd_tokens=3)


def test_parse_forms():
    assert PoolingConfig.parse("mean").levels[0].type == "mean"
    assert PoolingConfig.parse({"type": "sum", "activation": "identity"}).levels[0].activation == "identity"
    c = PoolingConfig.parse({"levels": [{"type": "mean", "neurons_per_shard": 256}, {"type": "weighted_sum"}]})
    assert c.is_semantic_hierarchy
    assert c.describe() == "mean[relu] -> weighted_sum"


def test_reduction_policy():
    assert resolve_reduction(PhysicalPlan())[0] == "fast"
    assert resolve_reduction(PhysicalPlan(reduction="deterministic"))[0] == "deterministic"


def test_reference_plan_fields_are_accepted():
    # every field of the reference's PhysicalPlan constructs here (drop-in)
    p = PhysicalPlan(block_m=32, cuda_block_m=16, cuda_warps=8, grad_precision="bf16", cuda_dx_warps=16,
                     cuda_grouped_dx_plan="private_t32", reduction="fast")
    assert p.block_m == 32


def test_same_fields_as_reference(reference_path):
    import dataclasses

    sys.path.insert(0, reference_path)
    from sparse_pooling.config import PhysicalPlan as RefPlan

    ours = {f.name for f in dataclasses.fields(PhysicalPlan)}
    theirs = {f.name for f in dataclasses.fields(RefPlan)}
    assert theirs <= ours
