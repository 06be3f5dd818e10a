"""Group sharding of the sparse-pooling layer across the GPUs of one node.

The reference is single-GPU.  Here rank r of P owns the contiguous pooling
groups ``[g0, g1) = shard_range(G, r, P)``, i.e. contiguous slices of the
``indices``/``weight``/``bias`` tensors (and of their gradients and Adam
moments).  Groups are independent in the forward pass, in dW/db and in the
optimizer; the two exchanges are

    forward : pre_r [B, g1-g0]  --all_gather-->  pre [B, G]   (replicated)
    backward: dX_r  [B, D]      --all_reduce(SUM)-->  dX       (replicated)

both NCCL collectives over NVLink (any torch.distributed backend works; the
CPU tests use gloo).  ``ShardedTrainStep`` issues the all-gather right after
the forward kernel and lets the backward kernel run under it, and issues the
dX all-reduce before the optimizer kernels so that they overlap it.

Nothing here touches another GPU's memory directly: remote data arrives only
through the collectives into local buffers.

Storage order.  A shard on a GPU stores its neurons, by default, in octet order (``gl_group_octets``):
within each group the records are permuted so that every 8 consecutive records ("octet") cover the
residues d mod 8 of their inputs evenly, and each record's 8 (index, weight) pairs are permuted so that at
every input position the octet's records read 8 distinct residues; the lane-per-neuron kernels
(``gl_fwd_octet_f32`` / ``gl_bwd_octet_f32``) then gather and scatter without shared-memory bank
conflicts.  Octet storage also interleaves each 32-record block's weights (``octet_storage``), which only
those kernels read, so a shard they cannot run (``octet_storage.unsupported``: e.g. an input_dim too wide
for their shared-memory tiles) gets the bank-aware order instead.  ``neuron_order="bank"`` keeps the
earlier bank-aware processing order of ``gl_group_order`` (unit 48, neurons only) with the generic
kernels, ``"slot"`` the reference's order.  The permutations are
within groups and within records, so pooled outputs and dX are unchanged; ``neuron_order[g][p]`` is the
slot stored at position p, ``input_order[g][p]`` (octet order) the record's input permutation (bits
3c .. 3c+2: the original input placed at position c), and ``canonical`` / ``canonical_shard`` return
tensors in slot order (the layout of ``SparsePoolingLayer``).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist
from torch import nn

from . import octet_storage
from .autograd import Level1Runtime, _compute_operands, _grad_buffers, act_torch, check_supported, dact_torch
from .config import PhysicalPlan, PoolingConfig
from .layout import SparseLayout, init_parameters


def _default_runtime(lay):
    rt = Level1Runtime(lay.layout, lay.indices, lay.cfg.levels[0], lay.plan, counts=lay.counts)
    rt.octets = lay.input_order is not None
    return rt


def shard_range(G: int, rank: int, world: int):
    """Contiguous near-equal split of G groups: rank r gets [g0, g1)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, rem = divmod(G, world)
    g0 = rank * base + min(rank, rem)
    return g0, g0 + base + (1 if rank < rem else 0)


def gather_columns(local: torch.Tensor, G: int, group=None) -> torch.Tensor:
    """All-gather per-rank column blocks [B, g1-g0] into [B, G] (uneven shards padded)."""
    world = dist.get_world_size(group)
    B = local.shape[0]
    width = -(-G // world)
    buf = local.new_zeros((B, width))
    buf[:, :local.shape[1]] = local
    out = local.new_empty((world * B, width))
    dist.all_gather_into_tensor(out, buf, group=group)
    out = out.view(world, B, width)
    cols = [out[r, :, :shard_range(G, r, world)[1] - shard_range(G, r, world)[0]] for r in range(world)]
    return torch.cat(cols, dim=1)


class _ShardedPoolFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, rt, G, g0, g1, group):
        xc, wc, bc = _compute_operands(x, w, b)
        out = rt.forward(xc, wc, bc)
        pre_l = out["pre"]
        pre = gather_columns(pre_l, G, group)
        ctx.rt, ctx.g0, ctx.g1, ctx.group = rt, g0, g1, group
        ctx.has_wmax = "wabsmax" in out
        ctx.save_for_backward(x, w, b, pre_l, *([out["wabsmax"]] if ctx.has_wmax else []))
        return act_torch(pre, rt.level.out_activation)

    @staticmethod
    def backward(ctx, dy):
        x, w, b, pre_l, *rest = ctx.saved_tensors
        rt = ctx.rt
        xc, wc, bc = _compute_operands(x, w, b)
        g_pre = (dy[:, ctx.g0:ctx.g1].float() * dact_torch(pre_l, rt.level.out_activation)).contiguous()
        dw_buf, db_buf, use_main = _grad_buffers(w, b)
        saved = {"pre": pre_l}
        if ctx.has_wmax:
            saved["wabsmax"] = rest[0]
        dx = rt.backward(xc, wc, bc, g_pre, saved, "minimal_stats", dw_buf, db_buf)
        dist.all_reduce(dx, group=ctx.group)
        gw = None if use_main else dw_buf.to(w.dtype)
        gb = None if use_main else db_buf.to(b.dtype)
        return dx.to(x.dtype), gw, gb, None, None, None, None, None


class GroupShardedLayer(nn.Module):
    """The groups ``[g0, g1)`` of a Mode-A ``SparsePoolingLayer`` on this rank.

    ``forward(x)`` returns the full pooled output [.., G] on every rank (all-gather);
    the input gradient is all-reduced so every rank sees the full dX.  Parameters
    are the local slices; ``from_full`` cuts them from a full layer (bit-identical
    to the single-GPU layer), the constructor draws them locally with
    ``seed + rank`` (statistically identical, for benchmarks at full scale).
    ``runtime_factory`` lets tests substitute the launch backend.
    """

    def __init__(self, input_dim: int, hidden_dim: int, output_dim: int, pooling="mean",
                 plan: Optional[PhysicalPlan] = None, device=None, seed: int = 0, bias_std: float = 0.0,
                 group=None, runtime_factory: Optional[Callable] = None, _params=None, neuron_order: str = "octet"):
        super().__init__()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.cfg = PoolingConfig.parse(pooling)
        self.layout = SparseLayout(input_dim, hidden_dim, output_dim, 8, 8, False)
        self.plan = plan or PhysicalPlan()
        self.g0, self.g1 = shard_range(output_dim, self.rank, self.world)
        check_supported(self.layout, self.cfg.levels[0], torch.float32)
        counts = self.layout.counts_tensor("cpu")[self.g0:self.g1]
        if _params is None:
            G_l = self.g1 - self.g0
            NB = self.layout.blocks_per_group
            # local draw: a layout of G_l groups with this shard's slot count per group
            loc = SparseLayout(input_dim, int(counts.sum()), G_l, 8, 8, False)
            if loc.blocks_per_group != NB or not torch.equal(loc.counts_tensor("cpu"), counts):
                raise ValueError("local initialisation needs equal group sizes; use GroupShardedLayer.from_full")
            idx, w, b = init_parameters(loc, device or "cpu", dtype=torch.float32, seed=seed + self.rank,
                                        bias_std=bias_std)
        else:
            idx, w, b = _params
        self.register_buffer("indices", idx)
        self.weight = nn.Parameter(w)
        self.bias = nn.Parameter(b)
        self.register_buffer("counts", counts.to(idx.device))
        factory = runtime_factory or _default_runtime
        self._factory = factory
        self._rt = None
        if neuron_order not in ("octet", "bank", "slot"):
            raise ValueError("neuron_order must be 'octet', 'bank' or 'slot'")
        self.order_kind = neuron_order
        self.register_buffer("neuron_order", None)
        self.register_buffer("input_order", None)
        if neuron_order != "slot":
            self.reorder_neurons()

    @torch.no_grad()
    def reorder_neurons(self):
        """Store this shard's records in octet (or bank-aware) order (module docstring).  Needs CUDA
        tensors (a no-op otherwise) and must run before optimizer state exists: parameters and any
        ``main_grad`` buffers are permuted in place."""
        if (self.order_kind == "slot" or self.neuron_order is not None or not self.indices.is_cuda
                or self.indices.shape[0] == 0):
            return
        from . import _native

        G_l, NB = self.indices.shape[0], self.layout.blocks_per_group
        slots = NB * 8
        counts = self.counts.to(torch.int32).contiguous()
        kp = None
        if self.order_kind == "octet" and octet_storage.unsupported(
                self.layout, self.cfg.levels[0].type, self.weight.dtype, self.indices.device, self.plan) is None:
            o, kp = octet_storage.arrange(self.indices, counts, self.layout.input_dim, NB)
        else:
            o = torch.empty((G_l, slots), dtype=torch.int32, device=self.indices.device)
            _native.group_order(self.indices, counts, self.layout.input_dim, NB, 0, G_l, 48, o)
        for t in (self.indices, self.weight.data, self.bias.data, getattr(self.weight, "main_grad", None),
                  getattr(self.bias, "main_grad", None)):
            if t is not None:
                octet_storage.apply_(t, o, kp)
        self.neuron_order = o
        self.input_order = kp
        self._rt = None

    def canonical(self, t: torch.Tensor) -> torch.Tensor:
        """``t`` (indices-, weight- or bias-shaped, in this shard's storage order) in slot order."""
        return octet_storage.canonical(t, self.neuron_order, self.input_order)

    def canonical_shard(self):
        """(indices, weight, bias) of this shard in slot order."""
        return self.canonical(self.indices), self.canonical(self.weight.detach()), self.canonical(self.bias.detach())

    @torch.no_grad()
    def full_state_dict(self) -> dict:
        """{"indices", "weight", "bias"} of the whole layer in slot order, gathered from every rank:
        bit for bit the state dict of the equivalent single-GPU ``SparsePoolingLayer`` (its keys,
        shapes and storage order), so checkpoints written here load into the drop-in layer and into
        the reference's.  Collective: every rank calls it and receives the full tensors."""
        G, world = self.layout.groups, self.world
        width = -(-G // world)
        out = {}
        for name, t in zip(("indices", "weight", "bias"), self.canonical_shard()):
            dtype = t.dtype
            if dtype == torch.int16:   # not every backend gathers int16 (gloo does not): widen exactly
                t = t.to(torch.int32)
            pad = t.new_zeros((width,) + tuple(t.shape[1:]))
            pad[:t.shape[0]] = t
            parts = [torch.empty_like(pad) for _ in range(world)]
            dist.all_gather(parts, pad.contiguous(), group=self.group)
            out[name] = torch.cat([parts[r][:shard_range(G, r, world)[1] - shard_range(G, r, world)[0]]
                                   for r in range(world)], dim=0).to(dtype)
        return out

    @torch.no_grad()
    def load_full_state_dict(self, sd: dict):
        """Load this rank's groups from a full (single-GPU layout) state dict, e.g. one written by
        ``SparsePoolingLayer.state_dict()``, ``full_state_dict()`` or the reference's layer."""
        for name, dst in (("indices", self.indices), ("weight", self.weight.data), ("bias", self.bias.data)):
            src = sd[name]
            if tuple(src.shape[1:]) != tuple(dst.shape[1:]) or src.shape[0] != self.layout.groups:
                raise ValueError(f"{name}: full shape {tuple(src.shape)} does not match this layer")
            dst.copy_(src[self.g0:self.g1])
        order, self.neuron_order, self.input_order = self.neuron_order, None, None
        self._rt = None
        if order is not None:
            self.reorder_neurons()

    @classmethod
    def from_full(cls, layer, group=None, runtime_factory=None, neuron_order: str = "octet"):
        """Shard an existing (full) ``SparsePoolingLayer``: slices of its tensors (reordered into the
        octet storage order when they are on a GPU; ``reorder_neurons`` after moving otherwise)."""
        L = layer.layout
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        g0, g1 = shard_range(L.groups, rank, world)
        params = (layer.indices[g0:g1].clone(), layer.weight.detach()[g0:g1].clone(),
                  layer.bias.detach()[g0:g1].clone())
        return cls(L.input_dim, L.hidden_dim, L.groups, pooling=layer.cfg, plan=layer.plan, group=group,
                   runtime_factory=runtime_factory, _params=params, neuron_order=neuron_order)

    def runtime(self):
        if self._rt is None or self._rt.idx is not self.indices:
            self._rt = self._factory(self)
        return self._rt

    def enable_main_grad(self):
        for p in (self.weight, self.bias):
            if getattr(p, "main_grad", None) is None:
                p.main_grad = torch.zeros(p.shape, device=p.device, dtype=torch.float32)

    def forward(self, x):
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        y = _ShardedPoolFunction.apply(x2, self.weight, self.bias, self.runtime(), self.layout.groups, self.g0,
                                       self.g1, self.group)
        return y.reshape(*lead, y.shape[-1])


class ShardedTrainStep:
    """One training step of a ``GroupShardedLayer`` with the collectives overlapped.

    step(x, dy): forward kernel -> async all-gather of pre -> backward kernel
    (dW/db into main_grad, partial dX) -> async all-reduce of dX -> optimizer
    kernels -> wait.  Returns (y [B, G], dx [B, D]).
    """

    def __init__(self, layer: GroupShardedLayer, optimizer):
        self.layer = layer
        self.opt = optimizer
        layer.enable_main_grad()

    def step(self, x: torch.Tensor, dy: torch.Tensor):
        lay = self.layer
        rt = lay.runtime()
        G = lay.layout.groups
        w, b = lay.weight.detach(), lay.bias.detach()
        fout = rt.forward(x, w, b)
        pre_l = fout["pre"]
        world = lay.world
        width = -(-G // world)
        if world > 1:
            buf = pre_l.new_zeros((x.shape[0], width)) if pre_l.shape[1] != width else pre_l
            if buf is not pre_l:
                buf[:, :pre_l.shape[1]] = pre_l
            gathered = pre_l.new_empty((world * x.shape[0], width))
            ag = dist.all_gather_into_tensor(gathered, buf, group=lay.group, async_op=True)
            gathered = gathered.view(world, x.shape[0], width)
        out_act = lay.cfg.levels[0].out_activation
        g_pre = dy[:, lay.g0:lay.g1]
        if out_act != "identity":
            g_pre = g_pre * dact_torch(pre_l, out_act)
        g_pre = g_pre.contiguous()
        dx = rt.backward(x, w, b, g_pre, fout, "minimal_stats", lay.weight.main_grad, lay.bias.main_grad)
        if world > 1:
            ar = dist.all_reduce(dx, group=lay.group, async_op=True)
        self.opt.step()
        if world > 1:
            ag.wait()
            ar.wait()
            cols = [gathered[r, :, :shard_range(G, r, world)[1] - shard_range(G, r, world)[0]]
                    for r in range(world)]
            pre = torch.cat(cols, dim=1)
        else:
            pre = pre_l
        return act_torch(pre, out_act), dx
