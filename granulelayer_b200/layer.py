"""PyTorch-facing module (mirror of sparse_pooling/layer.py).

``SparsePoolingLayer`` keeps the reference's constructor (layer.py:40-58),
parameter/buffer names and shapes (``indices``, ``weight``, ``bias``),
``forward`` (layer.py:186-197), ``explain``, ``last_info``,
``enable_main_grad``/``zero_main_grad`` and ``effective_policy``, so that
model code and state dicts move between the two unchanged.

``weight_layout="octet"`` (a B200 extension, Mode A) stores the parameters in
octet order (``octet_storage``) once they are on a GPU and the lane-per-neuron
kernels can run the layer (``octet_storage.unsupported``), which lets those
kernels run it without shared-memory bank conflicts.  The
state dict stays the reference's (slot order, converted on save and load), and
``canonical_parameters()`` returns slot-order tensors; ``layer.weight`` itself
then holds the permuted storage.

Execution is the B200 path only: Mode A (``shared_neurons=None``) and Mode B
(``shared_neurons=C``, canonical or fragment-packed storage, with or without
input-supergroup ``connectivity``), fp32, single-level ``mean`` or ``sum``
pooling with identity/ReLU/GELU neuron activation.  Any other configuration
still constructs (so checkpoints load) but ``forward`` raises
``UnsupportedOnB200`` instead of falling back.
"""
from __future__ import annotations

import math
from typing import Optional, Union

import torch
from torch import nn

from .autograd import Level1Runtime, SparsePoolFunction, check_supported, resolve_policy
from .config import DEFAULT_WORKSPACE_BUDGET, PhysicalPlan, PoolingConfig
from .layout import SparseLayout, init_parameters


class SparsePoolingLayer(nn.Module):
    """Weight-sparse projection to ``hidden_dim`` logical neurons (fan-in 8)
    fused with pooling into ``output_dim`` contiguous groups.

    Args mirror the reference (layer.py:16-58): ``shared_neurons=None`` selects
    Mode A (independent indices per neuron, the B200 path); ``pooling`` is an
    operator name, a level dict or a ``PoolingConfig``; ``plan`` is an
    execution-only ``PhysicalPlan``; ``seed`` and ``bias_std`` drive the
    bit-exact seeded initialisation of ``layout.init_parameters``.
    ``backend`` and ``workspace_budget`` are accepted for compatibility;
    ``weight_layout`` takes the reference's values and ``"octet"`` (Mode A:
    octet storage, the module docstring).  ``connectivity`` (a ``ConnectivityPlan``, Mode B only) draws
    the indices from input supergroups with the reference's generator
    (supergroups.py:200-271, bit-exact) and registers its ``sg_feat``,
    ``sg_buckets`` and ``sg_plan`` buffers (layer.py:78-84); the kernels run such
    layers as ordinary Mode-B layers.
    """

    def __init__(self, input_dim: int = 1024, hidden_dim: int = 100_000_000, output_dim: int = 1024,
                 fan_in: int = 8, shared_neurons: Optional[int] = 8,
                 pooling: Union[str, dict, PoolingConfig] = "max", checkpoint_policy: str = "auto",
                 dtype: torch.dtype = torch.bfloat16, plan: Optional[PhysicalPlan] = None,
                 workspace_budget: int = DEFAULT_WORKSPACE_BUDGET, device=None, seed: int = 0,
                 bias_std: float = 0.0, backend: str = "auto", weight_layout: str = "auto", connectivity=None):
        super().__init__()
        self.cfg = PoolingConfig.parse(pooling, checkpoint_policy)
        if isinstance(pooling, (str, PoolingConfig)) or "checkpoint_policy" not in (pooling or {}):
            self.cfg.checkpoint_policy = checkpoint_policy
        mode_b = shared_neurons is not None
        if weight_layout == "auto":
            weight_layout = "packed" if (mode_b and backend != "triton") else "canonical"
        if weight_layout not in ("packed", "canonical", "octet"):
            raise ValueError("weight_layout must be 'auto', 'packed', 'canonical' or 'octet'")
        if weight_layout == "octet" and (mode_b or self.cfg.is_semantic_hierarchy):
            raise ValueError("weight_layout='octet' is defined for single-level Mode-A layers")
        self.octet = weight_layout == "octet"
        self._order = self._kperm = None   # the octet arrangement, once applied
        self.layout = SparseLayout(input_dim, hidden_dim, output_dim, fan_in, shared_neurons if mode_b else 8,
                                   mode_b, packed=(weight_layout == "packed"))
        self.compute_dtype = dtype
        self.plan = plan or PhysicalPlan()
        self.backend_name = backend
        self.workspace_budget = workspace_budget
        self.connectivity = connectivity
        self.graph_stats = None
        idx, w, b = init_parameters(self.layout, device or "cpu", dtype=dtype, seed=seed, bias_std=bias_std)
        if connectivity is not None:
            from .supergroups import generate_indices

            idx_c, graph, self.graph_stats = generate_indices(self.layout.canonical, connectivity, device or "cpu")
            idx = self.layout.pack_indices(idx_c) if self.layout.packed else idx_c
            self.register_buffer("sg_feat", graph.feat)
            self.register_buffer("sg_buckets", graph.buckets)
            self.register_buffer("sg_plan", torch.frombuffer(bytearray(connectivity.to_json().encode()),
                                                             dtype=torch.uint8).clone())
        self.register_buffer("indices", idx)
        self.weight = nn.Parameter(w)
        self.bias = nn.Parameter(b)
        self._tnames = []
        if self.cfg.is_semantic_hierarchy:   # layer.py:90-101: level-1 transform / level-2 weights
            l1, l2 = self.cfg.levels
            S = math.ceil(self.layout.max_group / l1.neurons_per_shard)
            self.num_shards = S
            G = output_dim
            if l1.transform in ("affine", "gate"):
                self.t_alpha = nn.Parameter(torch.ones(G, S, device=device))
                self.t_beta = nn.Parameter(torch.zeros(G, S, device=device))
                self._tnames += ["alpha", "beta"]
            if l2.type == "weighted_sum":
                self.t_v = nn.Parameter(torch.full((G, S), 1.0 / S, device=device))
                self._tnames += ["v"]
        self._rt = None
        self._rt_key = None
        self._units = None

    @torch.no_grad()
    def arrange_storage(self):
        """Octet layouts: store the records in octet order now (a no-op for other layouts, on the CPU, when
        already arranged, or when the lane-per-neuron kernels cannot run the layer: ``octet_storage.
        unsupported`` says why, and the layer then keeps slot order).  The first forward on a GPU does
        this; call it earlier if optimizer state is created before that forward (parameters and
        ``main_grad`` are permuted in place)."""
        if not self.octet or self._order is not None or not self.indices.is_cuda:
            return
        from . import octet_storage

        if octet_storage.unsupported(self.layout, self.cfg.levels[0].type, self.weight.dtype, self.indices.device,
                                     self.plan) is not None:
            return

        L = self.layout
        order, kperm = octet_storage.arrange(self.indices, L.counts_tensor(self.indices.device), L.input_dim,
                                             L.blocks_per_group)
        for t in (self.indices, self.weight.data, self.bias.data, getattr(self.weight, "main_grad", None),
                  getattr(self.bias, "main_grad", None)):
            if t is not None:
                octet_storage.apply_(t, order, kperm)
        self._order, self._kperm = order, kperm
        self._rt = None

    def canonical(self, t: torch.Tensor) -> torch.Tensor:
        """An index-, weight- or bias-shaped tensor of this layer's storage (a parameter, its gradient,
        ``main_grad`` or an optimizer moment) in slot order, the reference's storage; ``t`` itself when the
        layer stores slot order."""
        from . import octet_storage

        return octet_storage.canonical(t, self._order, self._kperm)

    def canonical_parameters(self):
        """(indices, weight, bias) in slot order (the reference's storage), whatever the layout."""
        return tuple(self.canonical(t) for t in (self.indices, self.weight.detach(), self.bias.detach()))

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        super()._save_to_state_dict(destination, prefix, keep_vars)
        if self._order is not None:   # octet storage: checkpoints hold the reference's slot order
            from . import octet_storage

            for name in ("indices", "weight", "bias"):
                destination[prefix + name] = octet_storage.canonical(destination[prefix + name].detach(),
                                                                     self._order, self._kperm)

    def _runtime(self) -> Level1Runtime:
        if self.octet and self._order is None and self.indices.is_cuda:
            self.arrange_storage()
        key = (self.indices.device, self.indices.data_ptr(), id(self.plan))
        if self._rt is None or self._rt_key != key:
            check_supported(self.layout, self.cfg.levels[0], self.compute_dtype,
                            semantic=self.cfg.is_semantic_hierarchy)
            if self.cfg.is_semantic_hierarchy:
                from .semantic import UnitLayout

                units = UnitLayout(self.layout, self.cfg.levels[0].neurons_per_shard)
                self._rt = Level1Runtime(units, units.view(self.indices), self.cfg.levels[0], self.plan,
                                         counts=units.counts_tensor(self.indices.device))
                self._units = units
            else:
                self._rt = Level1Runtime(self.layout, self.indices, self.cfg.levels[0], self.plan)
                self._rt.octets = self._order is not None
            self._rt_key = key
        self._rt.param_dtype = self.weight.dtype
        if self.connectivity is not None and not self.cfg.is_semantic_hierarchy:
            self._rt.sets = (self.sg_feat, self.sg_buckets)
        return self._rt

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        """Connectivity must agree between checkpoint and layer (layer.py:133-142)."""
        plan = state_dict.get(prefix + "sg_plan")
        if self.connectivity is not None and plan is not None:
            from .supergroups import ConnectivityPlan

            got = ConnectivityPlan.from_json(bytes(plan.cpu().tolist()).decode())
            if got != self.connectivity:
                raise ValueError(f"checkpoint connectivity {got} != layer connectivity {self.connectivity}")
        if (self.connectivity is None) != (plan is None):
            raise ValueError("checkpoint and layer disagree on input-supergroup connectivity")
        if self._order is not None:   # octet storage: back to slot order; arranged again at the next forward
            from . import octet_storage

            with torch.no_grad():
                for t in (getattr(self.weight, "main_grad", None), getattr(self.bias, "main_grad", None)):
                    if t is not None:
                        t.copy_(octet_storage.canonical(t, self._order, self._kperm))
            self._order = self._kperm = None
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)
        self._rt = None

    @property
    def last_info(self):
        return {} if self._rt is None else dict(self._rt.last_info)

    def explain(self, batch: int = 8192) -> dict:
        """The execution the layer would use for ``batch`` tokens, without running it."""
        out = dict(backend_requested=self.backend_name)
        if not self.indices.is_cuda:
            out["backend"] = "none (CPU parameters; the B200 path needs CUDA tensors)"
            return out
        rt = self._runtime()
        out.update(rt.describe_execution(batch))
        return out

    @property
    def effective_policy(self) -> str:
        return resolve_policy(self.cfg.levels[0], self.cfg.checkpoint_policy)

    def enable_main_grad(self):
        """Accumulate W/b gradients into persistent FP32 ``main_grad`` buffers
        (autograd then returns None for them; layer.py:174-179)."""
        for p in (self.weight, self.bias):
            if getattr(p, "main_grad", None) is None:
                p.main_grad = torch.zeros(p.shape, device=p.device, dtype=torch.float32)

    def zero_main_grad(self):
        for p in (self.weight, self.bias):
            if getattr(p, "main_grad", None) is not None:
                p.main_grad.zero_()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        rt = self._runtime()
        if self.cfg.is_semantic_hierarchy:   # layer.py:186-195
            from .semantic import SemanticPoolFunction

            tparams = [getattr(self, "t_" + n) for n in self._tnames]
            y = SemanticPoolFunction.apply(x2, self.weight, self.bias, rt, self._units, self.cfg, self.effective_policy,
                                           self._tnames, *tparams)
        else:
            y = SparsePoolFunction.apply(x2, self.weight, self.bias, rt, self.effective_policy, self.compute_dtype)
        return y.reshape(*lead, y.shape[-1])

    def extra_repr(self) -> str:
        L = self.layout
        mode = f"B(C={L.block})" if L.shared_indices else "A(independent)"
        return (f"in={L.input_dim}, hidden={L.hidden_dim:,}, out={L.groups}, fan_in={L.fan_in}, "
                f"mode={mode}, pooling={self.cfg.describe()}, policy={self.effective_policy}")
