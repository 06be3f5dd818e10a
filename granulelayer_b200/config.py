"""Pooling semantics and execution plan: the reference's configuration surface.

Drop-in mirror of ``sparse_pooling/config.py`` (reference file:line cited per
object).  The dataclasses keep the reference's names, fields, defaults and
validation so that code constructing them for the reference constructs them
here unchanged.  Fields that only steer the reference's RTX 3090 tuning tables
are accepted and recorded but do not change what the B200 kernels do.

B200 execution covers fan-in-8 layers in Mode A (independent indices) and Mode B
(shared index records) with every single-level operator of the reference (mean,
max, top-K mean, LogMeanExp, power mean, softmax-weighted), the ``sum``
extension (``sum = n_g * mean``; the reference has no sum operator) and two-level
(semantic) hierarchies whose level-1 shards tile the stored blocks.  Anything
else parses (so configs round-trip) and is refused at run time with a clear
error.
"""
from __future__ import annotations

import warnings
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Union

# sparse_pooling/config.py:22-29, plus "sum" (extension: y_g = sum of act(z) over the group)
POOL_TYPES = ("max", "topk_mean", "mean", "logmeanexp", "power_mean", "softmax_weighted", "sum")
LEVEL2_ONLY_TYPES = ("weighted_sum",)  # config.py:31
ACTIVATIONS = ("identity", "relu", "gelu")  # config.py:33
TRANSFORMS = ("none", "activation", "affine", "gate")  # config.py:34
CHECKPOINT_POLICIES = ("minimal_stats", "recompute_stats", "save_winners", "auto")  # config.py:35

POOL_ID = {name: i for i, name in enumerate(POOL_TYPES)}
ACT_ID = {name: i for i, name in enumerate(ACTIVATIONS)}

# Operators the B200 kernels execute (the hot path); the rest are parsed only.
B200_POOLS = ("mean", "sum", "max", "logmeanexp", "power_mean", "softmax_weighted", "topk_mean")

# per-neuron activation used when the spec leaves it empty (config.py:42-49)
DEFAULT_ACTIVATION = {
    "max": "identity",
    "topk_mean": "identity",
    "mean": "relu",
    "logmeanexp": "identity",
    "power_mean": "relu",
    "softmax_weighted": "identity",
    "sum": "relu",
}
# activation of the pooled value when left empty (config.py:51-58)
DEFAULT_OUT_ACTIVATION = {
    "max": "relu",
    "topk_mean": "identity",
    "mean": "identity",
    "logmeanexp": "identity",
    "power_mean": "identity",
    "softmax_weighted": "identity",
    "sum": "identity",
}
# shorthand names (config.py:60-66)
ALIASES = {
    "mean_relu": ("mean", {"activation": "relu"}),
    "sum_relu": ("sum", {"activation": "relu"}),
    "lme": ("logmeanexp", {}),
    "softmax": ("softmax_weighted", {}),
    "power": ("power_mean", {}),
    "topk": ("topk_mean", {}),
}


@dataclass
class LevelSpec:
    """One pooling level (sparse_pooling/config.py:69-161).

    ``type`` names the operator; ``activation`` is applied per neuron before
    pooling and ``out_activation`` to the pooled value; ``k``, ``temperature``,
    ``beta`` and ``p`` parameterise Top-K, LogMeanExp, softmax-weighted and power
    mean; ``neurons_per_shard``/``transform`` describe a two-level hierarchy.
    """

    type: str
    activation: str = ""
    out_activation: str = ""
    k: int = 8
    temperature: float = 1.0
    beta: float = 1.0
    p: float = 2.0
    neurons_per_shard: Optional[int] = None
    transform: str = "none"
    transform_activation: str = "relu"

    def __post_init__(self):
        if self.type in ALIASES:
            name, extra = ALIASES[self.type]
            self.type = name
            for key, val in extra.items():
                if not getattr(self, key):
                    setattr(self, key, val)
        if self.type not in POOL_TYPES + LEVEL2_ONLY_TYPES:
            raise ValueError(f"unknown pooling type {self.type!r}")
        self.activation = self.activation or DEFAULT_ACTIVATION.get(self.type, "identity")
        self.out_activation = self.out_activation or DEFAULT_OUT_ACTIVATION.get(self.type, "identity")
        for a in (self.activation, self.out_activation):
            if a not in ACTIVATIONS:
                raise ValueError(f"unknown activation {a!r}")
        if self.transform not in TRANSFORMS:
            raise ValueError(f"unknown transform {self.transform!r}")
        if self.type == "topk_mean" and (self.k < 1 or self.k > 64 or self.k & (self.k - 1)):
            raise ValueError("topk_mean k must be a power of two in [1, 64]")
        if self.type == "logmeanexp" and not self.temperature > 0:
            raise ValueError("temperature must be > 0")
        if self.type == "softmax_weighted" and not self.beta > 0:
            raise ValueError("beta must be > 0")
        if self.type == "power_mean":
            if not self.p >= 1:
                raise ValueError("power_mean requires p >= 1")
            if self.activation != "relu":
                raise ValueError("power_mean is defined on relu activations")

    @property
    def pool_id(self) -> int:
        return POOL_ID[self.type]

    @property
    def act_id(self) -> int:
        return ACT_ID[self.activation]

    @property
    def out_act_id(self) -> int:
        return ACT_ID[self.out_activation]

    @property
    def scalar_param(self) -> float:
        return {"logmeanexp": self.temperature, "softmax_weighted": self.beta,
                "power_mean": self.p}.get(self.type, 0.0)

    def describe(self) -> str:
        s = self.type
        if self.type == "topk_mean":
            s += f"(k={self.k})"
        elif self.type == "logmeanexp":
            s += f"(tau={self.temperature:g})"
        elif self.type == "softmax_weighted":
            s += f"(beta={self.beta:g})"
        elif self.type == "power_mean":
            s += f"(p={self.p:g})"
        if self.activation != "identity":
            s = f"{s}[{self.activation}]"
        if self.out_activation != "identity":
            s = f"{self.out_activation}({s})"
        return s


@dataclass
class PoolingConfig:
    """One or two pooling levels plus the checkpoint policy (config.py:164-227)."""

    levels: List[LevelSpec]
    checkpoint_policy: str = "auto"
    level1_checkpoint: str = "save"

    def __post_init__(self):
        if not 1 <= len(self.levels) <= 2:
            raise ValueError("1 or 2 pooling levels are supported")
        if self.levels[0].type in LEVEL2_ONLY_TYPES:
            raise ValueError(f"{self.levels[0].type} cannot be a level-1 operator")
        if len(self.levels) == 2 and self.levels[0].neurons_per_shard is None:
            raise ValueError("a two-level config needs level-1 neurons_per_shard")
        if len(self.levels) == 1 and self.levels[0].neurons_per_shard is not None:
            raise ValueError("neurons_per_shard on a single level would change the model; "
                             "use PhysicalPlan for execution-only sharding")
        if self.checkpoint_policy not in CHECKPOINT_POLICIES:
            raise ValueError(f"unknown checkpoint policy {self.checkpoint_policy!r}")
        if self.level1_checkpoint not in ("save", "recompute"):
            raise ValueError("level1_checkpoint must be 'save' or 'recompute'")
        if len(self.levels) == 2:
            l1, l2 = self.levels
            monotone = ("identity", "relu")
            if (l1.type == l2.type == "max" and l1.transform == "none"
                    and l1.out_activation in monotone and l2.activation in monotone):
                warnings.warn("Max -> Max without a non-monotone transform between the levels is "
                              "exactly global Max; it adds no expressiveness")

    @property
    def is_semantic_hierarchy(self) -> bool:
        return len(self.levels) == 2

    @staticmethod
    def parse(spec: Union[str, Dict[str, Any], "PoolingConfig"], checkpoint_policy: str = "auto"):
        if isinstance(spec, PoolingConfig):
            return spec
        if isinstance(spec, str):
            return PoolingConfig([LevelSpec(type=spec)], checkpoint_policy=checkpoint_policy)
        if isinstance(spec, dict):
            if "levels" in spec:
                return PoolingConfig([LevelSpec(**lv) for lv in spec["levels"]],
                                     checkpoint_policy=spec.get("checkpoint_policy", checkpoint_policy),
                                     level1_checkpoint=spec.get("level1_checkpoint", "save"))
            return PoolingConfig([LevelSpec(**spec)], checkpoint_policy=checkpoint_policy)
        raise TypeError(f"cannot parse pooling spec {spec!r}")

    def describe(self) -> str:
        return " -> ".join(lv.describe() for lv in self.levels)


REDUCTIONS = ("auto", "fast", "deterministic")  # config.py:393


@dataclass
class PhysicalPlan:
    """Execution-only plan (config.py:240-391).  Never changes the function.

    The reference's fields are all accepted with their defaults.  On B200 the
    ones that matter are ``reduction`` (see ``resolve_reduction``) and the
    ``b200_*`` fields below; the Triton and RTX 3090 fields (``block_m``,
    ``num_warps``, ``cuda_*`` ...) are recorded for compatibility only.
    """

    phys_splits: int = 0
    block_m: int = 64
    num_warps: int = 4
    num_stages: int = 2
    token_tiles_per_program: int = 1
    input_layout: str = "feature_major"
    backend: str = "auto"
    tuning_profile: str = "auto"
    cuda_block_m: int = 32
    cuda_warps: int = 16
    grad_precision: str = "split"
    cuda_dx_epilogue: str = "auto"
    cuda_dw_epilogue: str = "auto"
    cuda_dx_warps: int = 0
    cuda_dw_cfg: int = -1
    cuda_dw_staging: str = "auto"
    cuda_input_supergroup_backend: str = "auto"
    cuda_grouped_fwd: str = ""
    cuda_grouped_dx: str = ""
    cuda_grouped_dw: str = ""
    cuda_grouped_fwd_tokens: int = 0
    cuda_grouped_fwd_warps: int = 0
    cuda_grouped_fwd_chunk_units: int = 0
    cuda_grouped_dx_tokens: int = 0
    cuda_grouped_dx_warps: int = 0
    cuda_grouped_dx_reduction: int = 0
    cuda_grouped_dx_chunk_units: int = 0
    cuda_grouped_dx_scatter: str = "auto"
    cuda_grouped_dx_plan: str = "auto"
    cuda_grouped_backward: str = "auto"
    cuda_grouped_fused_cfg: int = 0
    cuda_grouped_dw_cfg: int = -1
    cuda_grouped_dw_projection: str = "auto"
    cuda_grouped_merge: str = "atomic"
    reduction: str = "auto"
    deterministic_workspace_bytes: int = 0
    # ---- B200 fields (0 = automatic) ----
    b200_fwd_tokens: int = 0       # tokens per forward tile (power of two, bounded by shared memory)
    b200_dx_tokens: int = 0        # tokens per dX tile
    b200_dx_splits: int = 0        # neuron-range splits of the dX kernel (global red flushes)
    # block-private dX accumulation of the backward: "fixed" = int32 fixed point (faster; rounding
    # well inside the dX tolerance), "fp32" = fp32 shared-memory atomics, "auto" = "fixed"
    b200_dx_accum: str = "auto"
    # processing order of each group's neurons: "identity" = slot order (default); "auto" = the
    # bank-aware order of gl_group_order (computed once per index tensor) where the token tile allows
    # it.  The bank-aware order halves shared-memory bank conflicts but scatters the parameter-record
    # loads of a warp step over ~6x more cache lines on the same L1 data path; measured at the
    # 100M-neuron config it is slower (backward 835 ms vs 755 ms), so it is off by default.
    b200_neuron_order: str = "identity"
    # input locality: "auto" = when every group reads at most a quarter of the input features, the
    # kernels stage only each group's features (gl_group_feature_map, once per index tensor);
    # "off" = always stage the whole input row
    b200_locality: str = "auto"
    # bf16 Mode-B layers (fragment-packed storage; mean, sum and max pools): "auto" = the tensor-core
    # kernels; "off" = the fp32 kernels, which widen the bf16 parameters.  Either way a bf16 layer
    # computes on x rounded to bf16, the reference's compute dtype
    b200_bf16_tensor_cores: str = "auto"
    # fp32 Cover-TopK16 layers: "auto" = the tensor-core kernels on three-term bf16 splits of x, w and dz
    # (gl_k16_*_tc_f32, fp32-level results); "off" = the fp32 SIMT kernels (gl_k16_*_f32)
    b200_f32_tensor_cores: str = "auto"
    # Cover-TopK16 layers on the tensor cores with S = 64 sets: which passes run on tcgen05 with TMEM
    # accumulators (gl_k16_fwd_t5* / gl_k16_bwd_t5*): "on" (both), "fwd", "bwd", or "off" (the mma.sync kernels)
    b200_tcgen05: str = "off"

    def __post_init__(self):
        if self.input_layout not in ("feature_major", "token_major"):
            raise ValueError("input_layout must be 'feature_major' or 'token_major'")
        if self.backend not in ("triton", "cuda", "auto"):
            raise ValueError("backend must be 'triton', 'cuda' or 'auto'")
        if not isinstance(self.tuning_profile, str) or not self.tuning_profile:
            raise ValueError("tuning_profile must be 'auto' or a registered profile name")
        if self.grad_precision not in ("split", "bf16"):
            raise ValueError("grad_precision must be 'split' or 'bf16'")
        if self.reduction not in REDUCTIONS:
            raise ValueError(f"reduction must be one of {REDUCTIONS} (got {self.reduction!r})")
        if self.deterministic_workspace_bytes < 0:
            raise ValueError("deterministic_workspace_bytes must be >= 0")
        for f in ("b200_fwd_tokens", "b200_dx_tokens"):
            v = getattr(self, f)
            if v and (v & (v - 1) or v > 128):
                raise ValueError(f"{f} must be 0 or a power of two <= 128 (each kernel documents its own range)")
        if self.b200_dx_splits < 0:
            raise ValueError("b200_dx_splits must be >= 0")
        if self.b200_dx_accum not in ("auto", "fixed", "fp32"):
            raise ValueError("b200_dx_accum must be 'auto', 'fixed' or 'fp32'")
        if self.b200_neuron_order not in ("auto", "identity"):
            raise ValueError("b200_neuron_order must be 'auto' or 'identity'")
        if self.b200_locality not in ("auto", "off"):
            raise ValueError("b200_locality must be 'auto' or 'off'")
        if self.b200_bf16_tensor_cores not in ("auto", "off"):
            raise ValueError("b200_bf16_tensor_cores must be 'auto' or 'off'")
        if self.b200_f32_tensor_cores not in ("auto", "off"):
            raise ValueError("b200_f32_tensor_cores must be 'auto' or 'off'")
        if self.b200_tcgen05 not in ("on", "off", "fwd", "bwd"):
            raise ValueError("b200_tcgen05 must be 'on', 'off', 'fwd' or 'bwd'")


def resolve_reduction(plan: PhysicalPlan):
    """(mode, reason, strict) of the plan's reduction policy (config.py:397-421).

    "fast" uses FP32 atomics in the backward's reductions; "deterministic" runs
    the bitwise-repeatable backward where the layer has one (Mode B, mean / sum;
    ``Level1Runtime.deterministic_reason``), and elsewhere an explicit request
    raises and the PyTorch global deterministic setting raises unless warn_only
    is set (then it warns).
    """
    import torch

    glob = torch.are_deterministic_algorithms_enabled()
    warn_only = glob and torch.is_deterministic_algorithms_warn_only_enabled()
    if plan.reduction == "deterministic":
        return "deterministic", "explicit reduction='deterministic'", True
    if plan.reduction == "fast":
        if glob and not warn_only:
            raise RuntimeError("PhysicalPlan(reduction='fast') uses FP32 atomics, but "
                               "torch.use_deterministic_algorithms(True) is set: use reduction='deterministic' "
                               "or 'auto', or enable warn_only")
        if glob:
            warnings.warn("reduction='fast' under torch.use_deterministic_algorithms(warn_only=True): "
                          "GranuleLayer reductions use FP32 atomics", stacklevel=3)
            return "fast", "explicit reduction='fast' (global deterministic warn_only)", False
        return "fast", "explicit reduction='fast'", False
    if glob:
        return "deterministic", "torch.use_deterministic_algorithms(True)", not warn_only
    return "fast", "default (torch deterministic algorithms off)", False


DEFAULT_WORKSPACE_BUDGET = 512 * 2**20  # config.py:448


def human_bytes(n: float) -> str:
    for unit in ("B", "KiB", "MiB", "GiB", "TiB"):
        if abs(n) < 1024 or unit == "TiB":
            return f"{n:.1f} {unit}" if unit != "B" else f"{int(n)} B"
        n /= 1024
    return f"{n:.1f} TiB"
