"""Two-level (semantic) pooling: level 1 pools neuron shards on the B200 kernels, level 2 pools the
compact ``[B, G, S]`` features in PyTorch.

Mirror of the reference's semantic hierarchy: ``PoolingConfig`` with two levels, level 1 carrying
``neurons_per_shard`` (config.py:164-227), the pooling units (kernels/ops.py:31-56: unit
``u = g * S + s`` covers blocks ``[s * BPS, (s + 1) * BPS)`` of group ``g``, ``S = ceil(max_group /
neurons_per_shard)``), the level-1 transform and level-2 operator
(reference/pytorch_reference.py:51-139) and ``SemanticPoolFunction`` (autograd.py:417-476).

Level 1 runs on the same kernels as a single-level layer: the unit view of the parameters
(``[G, NB, ...]`` read as ``[G * S, BPS, ...]``) is a reshape when ``S * BPS`` equals the
layer's blocks per group, which the layer checks.  Level 2 touches only ``B * G * S`` values and
stays in PyTorch, as in the reference.
"""
from __future__ import annotations

import math
from typing import Dict, List

import torch

from .autograd import (Level1Runtime, UnsupportedOnB200, _compute_operands, _grad_buffers, act_torch, dact_torch)
from .config import LevelSpec, PoolingConfig
from .layout import SparseLayout


class UnitLayout:
    """The layout attributes the level-1 runtime reads, for the shard units of a layout."""

    def __init__(self, layout: SparseLayout, nps: int):
        S, BPS = shard_geometry(layout, nps)
        self.parent = layout
        self.shards = S
        self.block = layout.block
        self.blocks_per_group = BPS
        self.input_dim = layout.input_dim
        self.packed = layout.packed
        self.shared_indices = layout.shared_indices
        self.groups = layout.groups * S
        self.nps = nps

    def counts_tensor(self, device) -> torch.Tensor:
        """Valid neurons of each unit (kernels/ops.py:51-56)."""
        n_g = self.parent.counts_tensor(device).to(torch.int64)
        s = torch.arange(self.shards, device=device, dtype=torch.int64)
        return torch.clamp(n_g[:, None] - s[None, :] * self.nps, min=0, max=self.nps).reshape(-1).to(torch.int32)

    def view(self, t: torch.Tensor) -> torch.Tensor:
        """A [G, ...] parameter / index / gradient tensor read as [G * S, ...]."""
        return t.reshape(self.groups, t.shape[1] // self.shards, *t.shape[2:])


def shard_geometry(layout: SparseLayout, nps: int):
    """(S, BPS) of a level-1 sharding (kernels/ops.py:45-56), with the B200 condition that the shards
    tile the stored blocks of a group exactly."""
    if nps % (4 * layout.block) != 0:
        raise ValueError(f"neurons_per_shard must be a multiple of 4*C = {4 * layout.block}")
    S = math.ceil(layout.max_group / nps)
    if layout.base <= (S - 1) * nps:   # the smallest group's last shard
        raise ValueError("a semantic shard would be empty; choose a different neurons_per_shard")
    BPS = nps // layout.block
    if S * BPS != layout.blocks_per_group:
        raise UnsupportedOnB200(f"neurons_per_shard={nps} does not tile the {layout.blocks_per_group} stored "
                                f"blocks per group ({S} shards of {BPS})")
    return S, BPS


def apply_transform(f: torch.Tensor, level1: LevelSpec, tp: Dict[str, torch.Tensor]) -> torch.Tensor:
    """Level-1 feature transform (pytorch_reference.py:104-115)."""
    tr = level1.transform
    if tr == "none":
        return f
    if tr == "activation":
        return act_torch(f, level1.transform_activation)
    if tr == "affine":
        return act_torch(tp["alpha"] * f + tp["beta"], level1.transform_activation)
    if tr == "gate":
        return f * torch.sigmoid(tp["alpha"] * f + tp["beta"])
    raise ValueError(tr)


def pool_dense(h: torch.Tensor, level: LevelSpec) -> torch.Tensor:
    """A pooling operator over the last dimension with every element valid, followed by its
    out-activation (pytorch_reference.py:51-98 with an all-true mask)."""
    a = act_torch(h, level.activation)
    n = h.shape[-1]
    t = level.type
    if t == "max":
        pooled = a.amax(-1)
    elif t == "topk_mean":
        k = min(level.k, n)
        order = torch.sort(h.detach(), dim=-1, descending=True, stable=True).indices[..., :k]
        pooled = a.gather(-1, order).sum(-1) / k
    elif t == "mean":
        pooled = a.mean(-1)
    elif t == "sum":
        pooled = a.sum(-1)
    elif t == "logmeanexp":
        tau = level.temperature
        pooled = tau * (torch.logsumexp(a / tau, dim=-1) - math.log(n))
    elif t == "power_mean":
        m = a.amax(-1, keepdim=True)
        safe = torch.where(m > 0, m, torch.ones_like(m))
        s = ((a / safe) ** level.p).mean(-1)
        pooled = torch.where(m.squeeze(-1) > 0, safe.squeeze(-1) * s ** (1.0 / level.p), torch.zeros_like(s))
    elif t == "softmax_weighted":
        pooled = (torch.softmax(level.beta * a, dim=-1) * a).sum(-1)
    else:
        raise ValueError(t)
    return act_torch(pooled, level.out_activation)


def level2_forward(f: torch.Tensor, cfg: PoolingConfig, tp: Dict[str, torch.Tensor]) -> torch.Tensor:
    """f [B, G, S] level-1 features -> y [B, G] (pytorch_reference.py:118-127)."""
    l1, l2 = cfg.levels
    h = apply_transform(f, l1, tp)
    if l2.type == "weighted_sum":
        return act_torch((h * tp["v"]).sum(-1), l2.out_activation)
    return pool_dense(h, l2)


class SemanticPoolFunction(torch.autograd.Function):
    """y = level2(transform(F)), F [B, G, S] = out_act(level-1 pooled shards) (autograd.py:417-476).

    ``cfg.level1_checkpoint == "save"`` keeps the level-1 pre-activations (and statistics) from the
    forward; ``"recompute"`` keeps only x, W, b and re-runs level 1 in the backward."""

    @staticmethod
    def forward(ctx, x, w, b, rt: Level1Runtime, units: UnitLayout, cfg: PoolingConfig, policy: str, tnames: List[str],
                *tparams):
        xc, wc, bc = _compute_operands(x, w, b)
        l1 = rt.level
        out = rt.forward(xc, units.view(wc), units.view(bc), track_ids=(policy == "save_winners"))
        B, G, S = x.shape[0], units.parent.groups, units.shards
        pre = out["pre"]
        with torch.no_grad():
            y = level2_forward(act_torch(pre, l1.out_activation).reshape(B, G, S), cfg, dict(zip(tnames, tparams)))
        saved = {}
        if cfg.level1_checkpoint == "save":
            saved["pre"] = pre
            if policy == "save_winners" and "winner" in out:
                saved["winner"] = out["winner"]
            if "L2" in out and policy != "recompute_stats":
                saved["L2"] = out["L2"]
        ctx.rt, ctx.units, ctx.cfg, ctx.policy, ctx.tnames = rt, units, cfg, policy, tnames
        ctx.saved_keys = list(saved)
        ctx.n_t = len(tparams)
        ctx.save_for_backward(x, w, b, *tparams, *saved.values())
        rt.last_info["checkpoint_bytes"] = sum(t.numel() * t.element_size() for t in saved.values())
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, b, *rest = ctx.saved_tensors
        tparams = rest[:ctx.n_t]
        saved = dict(zip(ctx.saved_keys, rest[ctx.n_t:]))
        rt: Level1Runtime = ctx.rt
        units: UnitLayout = ctx.units
        l1 = rt.level
        xc, wc, bc = _compute_operands(x, w, b)
        wu, bu = units.view(wc), units.view(bc)
        recomputed = "pre" not in saved
        if recomputed:  # rebuild the level-1 features
            saved.update(rt.forward(xc, wu, bu, track_ids=(ctx.policy == "save_winners")))
        B, G, S = x.shape[0], units.parent.groups, units.shards
        pre = saved["pre"]
        with torch.enable_grad():
            fv = act_torch(pre, l1.out_activation).reshape(B, G, S).detach().requires_grad_(True)
            tp = [p.detach().requires_grad_(True) for p in tparams]
            y = level2_forward(fv, ctx.cfg, dict(zip(ctx.tnames, tp)))
            grads = torch.autograd.grad(y, [fv] + tp, dy, allow_unused=True)
        g_pre = (grads[0].reshape(B, G * S).float() * dact_torch(pre, l1.out_activation)).contiguous()
        policy = ctx.policy if ctx.policy != "recompute_stats" else "minimal_stats"
        dw_buf, db_buf, use_main = _grad_buffers(w, b)
        dx = rt.backward(xc, wu, bu, g_pre, saved, policy, units.view(dw_buf), units.view(db_buf), recomputed)
        gw = None if use_main else dw_buf.to(w.dtype)
        gb = None if use_main else db_buf.to(b.dtype)
        return (dx.to(x.dtype, memory_format=torch.contiguous_format), gw, gb, None, None, None, None, None,
                *grads[1:])
