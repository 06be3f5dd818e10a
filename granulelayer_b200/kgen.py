"""Generalized fan-in layout, the K64 envelope and its compact K16/C16 lowering
(mirror of sparse_pooling/experimental/kgen_layout.py and kgen_lowered.py).

``KLayout`` (kgen_layout.py:29-100): fan-in K in {8, 16, 32, 64}, logical block
C (multiple of 8, <= 2048); output g owns n_g = H // G + (g < H % G) neurons;
storage ``indices [G, NB, K] int16`` (one record shared by the C neurons of a
block), ``weights [G, NB, C, K]``, ``bias [G, NB, C]``, NB = ceil(max n_g / C)
(no padding to a multiple of 4).

``Envelope`` (kgen_lowered.py:46-104): the K64 / C-logical graph of the
generalized generator (quantum 1) over given pre-pruning BF16 values.

``lower_env`` (kgen_lowered.py:147-201): every valid 16-neuron row group
u = (g, j, c // 16) of the envelope becomes one compact record of 16 neurons
sharing the k inputs ``feat[q(g, j)][env[u]]``; its neurons keep their weights at
those coordinates and their own bias; padded 16-blocks copy the output's first
record and hold zeros.  The result is the K16/C16 layer's storage.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch

from .supergroups import GENERATOR, GENERATOR_VERSION, ConnectivityPlan, GraphSpec, generate_records, \
    unit_to_block_buckets


@dataclass(frozen=True)
class KLayout:
    input_dim: int
    hidden_dim: int
    groups: int
    fan_in: int
    block: int

    def __post_init__(self):
        if self.fan_in not in (8, 16, 32, 64):
            raise ValueError(f"fan_in must be 8, 16, 32 or 64 (got {self.fan_in})")
        if self.block % 8 or not 8 <= self.block <= 2048:
            raise ValueError(f"C must be a multiple of 8 in [8, 2048] (got {self.block})")
        if self.input_dim > 32767:
            raise ValueError("int16 indices require input_dim <= 32767")
        if self.fan_in > self.input_dim:
            raise ValueError("fan_in > input_dim")
        if self.hidden_dim < self.groups:
            raise ValueError("need at least one neuron per group")

    @property
    def base(self) -> int:
        return self.hidden_dim // self.groups

    @property
    def rem(self) -> int:
        return self.hidden_dim % self.groups

    @property
    def max_group(self) -> int:
        return self.base + (1 if self.rem else 0)

    @property
    def blocks_per_group(self) -> int:
        return -(-self.max_group // self.block)

    @property
    def slots_per_group(self) -> int:
        return self.blocks_per_group * self.block

    def counts_tensor(self, device) -> torch.Tensor:
        g = torch.arange(self.groups, device=device)
        return (self.base + (g < self.rem).to(torch.int64)).to(torch.int32)

    def valid_blocks(self, device="cpu") -> torch.Tensor:
        return (self.counts_tensor(device).to(torch.int64) + self.block - 1) // self.block

    @property
    def index_shape(self):
        return (self.groups, self.blocks_per_group, self.fan_in)

    @property
    def weight_shape(self):
        return (self.groups, self.blocks_per_group, self.block, self.fan_in)

    @property
    def bias_shape(self):
        return (self.groups, self.blocks_per_group, self.block)

    def valid_mask(self, device) -> torch.Tensor:
        """[G, NB, C] bool valid neurons."""
        s = torch.arange(self.slots_per_group, device=device)
        return (s[None, :] < self.counts_tensor(device)[:, None]).view(self.bias_shape)

    def padding_fraction(self) -> float:
        return 1.0 - self.hidden_dim / (self.groups * self.slots_per_group)


@torch.no_grad()
def init_envelope_parameters(layout: KLayout, device, dtype=torch.bfloat16, seed: int = 0, weight_std=None,
                             bias_std: float = 0.0, chunk: int = 1 << 25):
    """(weights, bias) N(0, weight_std^2) (default 1/sqrt(K)) in flat canonical order from one seeded
    generator, then bias N(0, bias_std^2) when bias_std > 0, padding zeroed (kgen_layout.py:103-132)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    std = 1.0 / math.sqrt(layout.fan_in) if weight_std is None else weight_std
    w = torch.empty(layout.weight_shape, dtype=dtype, device=device)
    flat = w.view(-1)
    for lo in range(0, flat.numel(), chunk):
        hi = min(lo + chunk, flat.numel())
        flat[lo:hi] = (torch.randn(hi - lo, generator=gen, device=device) * std).to(dtype)
    b = torch.zeros(layout.bias_shape, dtype=dtype, device=device)
    if bias_std > 0:
        b.copy_((torch.randn(b.shape, generator=gen, device=device) * bias_std).to(dtype))
    pad = ~layout.valid_mask(device)
    w.masked_fill_(pad[..., None], 0)
    b.masked_fill_(pad, 0)
    return w, b


@dataclass
class Envelope:
    """The K64 envelope: layout, pre-pruning values, set table ``sg_feat [Q, 64]``, logical-block
    buckets ``kg_buckets [n, 4]`` (q, g, first block, blocks), graph spec, connectivity; ``mask``
    [G, NB, C, 64] the selected support once known."""

    layout: KLayout
    weight: torch.Tensor
    bias: torch.Tensor
    sg_feat: torch.Tensor
    kg_buckets: torch.Tensor
    spec: GraphSpec
    connectivity: ConnectivityPlan
    indices: Optional[torch.Tensor] = None
    mask: Optional[torch.Tensor] = None
    graph_stats: dict = field(default_factory=dict)

    @classmethod
    @torch.no_grad()
    def generate(cls, input_dim: int, hidden_dim: int, output_dim: int, shared_neurons: int,
                 connectivity: ConnectivityPlan, weight, bias, device=None, keep_indices: bool = False):
        L = KLayout(input_dim, hidden_dim, output_dim, 64, shared_neurons)
        device = torch.device(device or weight.device)
        if tuple(weight.shape) != L.weight_shape or tuple(bias.shape) != L.bias_shape:
            raise ValueError(f"envelope values: weight {tuple(weight.shape)} / bias {tuple(bias.shape)}, expected "
                             f"{L.weight_shape} / {L.bias_shape} ([G, NB, C, 64] order)")
        if weight.dtype != torch.bfloat16 or bias.dtype != torch.bfloat16:
            raise ValueError("envelope values must be BF16 (the parameter dtype of the envelope recipe)")
        counts = L.counts_tensor(device)
        idx, feat, ubk, st = generate_records(input_dim, counts, L.block, 64, L.blocks_per_group, 1, connectivity,
                                              device)
        bk = unit_to_block_buckets(ubk, counts, L.block, 1)
        spec = GraphSpec(64, L.block, connectivity.input_supergroup_dim, connectivity.partition_rounds,
                         connectivity.seed, 1, connectivity.generation)
        return cls(L, weight.to(device), bias.to(device), feat.contiguous(), bk.contiguous(), spec, connectivity,
                   idx.contiguous() if keep_indices else None,
                   graph_stats=dict(st, generator=GENERATOR, generator_version=GENERATOR_VERSION, quantum=1))


@dataclass
class Lowered:
    """Compact K16/C16 storage: indices [G, NB16, k] int16, weight [G, NB16, 16, k], bias [G, NB16, 16],
    block buckets [n, 4] (q, g, first 16-block, 16-blocks), env [G*NB16, k] uint8 local positions, spec."""

    layout: KLayout
    indices: torch.Tensor
    weight: torch.Tensor
    bias: torch.Tensor
    kg_buckets: torch.Tensor
    env: torch.Tensor
    spec: GraphSpec
    records_16: int


@torch.no_grad()
def lower_env(env_obj: Envelope, env_u: torch.Tensor, source: str = "lowered-local-of-K64") -> Lowered:
    """Compact lowering of ``env_u`` [n16, k] (sorted distinct local positions 0..63 of every K64 row group)."""
    L = env_obj.layout
    C = L.block
    k = env_u.shape[1]
    dev = env_obj.weight.device
    env_u = env_u.to(dev).to(torch.int64)
    G, NB = L.groups, L.blocks_per_group
    gpb = C // 16
    counts = L.counts_tensor(dev).to(torch.int64)
    nb16 = (int(counts.max()) + 15) // 16
    nvb16 = (counts + 15) // 16
    b = env_obj.kg_buckets.to(dev).to(torch.int64)
    # set of every K64 block
    rb = torch.repeat_interleave(torch.arange(len(b), device=dev), b[:, 3])
    kb = torch.arange(len(rb), device=dev) - torch.repeat_interleave(torch.cumsum(b[:, 3], 0) - b[:, 3], b[:, 3])
    bq = torch.full((G * NB,), -1, dtype=torch.int64, device=dev)
    bq[b[rb, 1] * NB + b[rb, 2] + kb] = b[rb, 0]
    g_ = torch.arange(G, device=dev)[:, None].expand(G, nb16)
    j16 = torch.arange(nb16, device=dev)[None, :].expand(G, nb16)
    live = j16 < nvb16[:, None]
    u = torch.where(live, g_ * (NB * gpb) + j16, g_ * (NB * gpb))   # padded 16-blocks: the output's first group
    q = bq[u // gpb]
    if bool((q[live] < 0).any()):
        raise AssertionError("a valid K64 block is in no bucket")
    env = env_u[u.reshape(-1)]
    if bool((env[:, 1:] <= env[:, :-1]).any()):
        raise ValueError("local positions of a record must be sorted and distinct")
    feat = env_obj.sg_feat.to(dev).to(torch.int64)
    idx = feat[q.reshape(-1)[:, None], env].reshape(G, nb16, k).to(torch.int16)
    wv = env_obj.weight.detach().reshape(-1, 16, 64)
    w = torch.gather(wv[u.reshape(-1)], 2, env[:, None, :].expand(-1, 16, k)).reshape(G, nb16, 16, k)
    bias = env_obj.bias.detach().reshape(-1, 16)[u.reshape(-1)].reshape(G, nb16, 16)
    valid16 = (torch.arange(nb16 * 16, device=dev)[None, :] < counts[:, None]).view(G, nb16, 16)
    w = w * (live[:, :, None, None] & valid16[..., None])
    bias = bias * (live[:, :, None] & valid16)
    first = b[:, 2] * gpb
    end = torch.minimum((b[:, 2] + b[:, 3]) * gpb, nvb16[b[:, 1]])
    bk = torch.stack([b[:, 0], b[:, 1], first, end - first], 1)
    bk = bk[bk[:, 3] > 0].to(torch.int32).contiguous()
    sp = env_obj.spec
    spec = GraphSpec(k, 16, sp.S, sp.R, sp.seed, 1, sp.generation, source=source)
    KL = KLayout(L.input_dim, L.hidden_dim, G, k, 16)
    if KL.blocks_per_group != nb16:
        raise AssertionError("lowered block count differs from the K16/C16 layout")
    return Lowered(KL, idx.contiguous(), w.contiguous(), bias.contiguous(), bk, env.to(torch.uint8).contiguous(),
                   spec, int(live.sum()))
