"""Neuron layout and seeded parameter generation (mirror of sparse_pooling/layout.py).

Partition (layout.py:10-14, 66-120): H logical neurons are split into G
contiguous pooling groups; group g owns ``n_g = H // G + (g < H % G)`` neurons
whose global ids are ``offset_g + slot`` with
``offset_g = g * (H // G) + min(g, H % G)``.  Each group is stored in
``NB`` blocks of ``C`` neuron slots, NB padded to a multiple of 4
(layout.py:80-83); slots ``>= n_g`` are padding with zero weight, bias and
(Mode A) index.

Storage (layout.py:123-140), fan-in K = 8:

    Mode A (independent indices, the B200 hot path)
        indices [G, NB, C, 8] int16, weights [G, NB, C, 8], bias [G, NB, C]
    Mode B (C neurons share one index record)
        indices [G, NB, 8], weights [G, NB, C, 8], bias [G, NB, C]
    Mode B fragment-packed (``packed=True``): pure permutations of the above
        (layout.py:20-33, 146-179).

In Mode A with C = 8 the flat neuron slot ``s = g * NB * 8 + blk * 8 + c`` owns
the 16-byte index record ``indices.view(-1, 8)[s]``, the 32-byte fp32 weight
row ``weights.view(-1, 8)[s]`` and ``bias.view(-1)[s]``: the B200 kernels read
these tensors in place, with no repacking.

``init_parameters`` reproduces layout.py:191-251 draw for draw (same torch
generator, same call order and chunking) so that a layer built here with a
given seed holds bit-identical indices, weights and bias to one built by the
reference on the same device and torch version.
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass

import torch

FAN_IN = 8


@dataclass(frozen=True)
class SparseLayout:
    input_dim: int
    hidden_dim: int
    groups: int
    fan_in: int
    block: int            # C: neurons per stored block
    shared_indices: bool  # True: Mode B, False: Mode A
    packed: bool = False  # fragment-packed storage (Mode B only)

    def __post_init__(self):
        if self.fan_in != FAN_IN:
            raise ValueError("kernels are specialised for fan-in 8")
        if self.input_dim > 32767:
            raise ValueError("int16 indices require input_dim <= 32767")
        if self.block not in (8, 16, 32, 64):
            raise ValueError("block (shared_neurons) must be 8, 16, 32 or 64")
        if self.hidden_dim < self.groups:
            raise ValueError("need at least one neuron per group")
        if self.packed and not self.shared_indices:
            raise ValueError("fragment-packed storage is only defined for Mode B")

    # ---- partition (layout.py:66-120) ------------------------------------
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
        nb = -(-self.max_group // self.block)
        return -(-nb // 4) * 4

    @property
    def n_tiles8(self) -> int:
        return self.block // 8

    @property
    def unit_blocks(self) -> int:
        return max(1, 4 // self.n_tiles8)

    @property
    def slots_per_group(self) -> int:
        return self.blocks_per_group * self.block

    def group_count(self, g: int) -> int:
        return self.base + (1 if g < self.rem else 0)

    def group_offset(self, g: int) -> int:
        return g * self.base + min(g, self.rem)

    def counts_tensor(self, device) -> torch.Tensor:
        g = torch.arange(self.groups, device=device)
        return (self.base + (g < self.rem).to(torch.int64)).to(torch.int32)

    def offsets_tensor(self, device) -> torch.Tensor:
        g = torch.arange(self.groups, device=device, dtype=torch.int64)
        return g * self.base + torch.clamp(g, max=self.rem)

    def global_ids(self, device) -> torch.Tensor:
        """[G, slots] int64 global neuron id of every slot, -1 for padding."""
        s = torch.arange(self.slots_per_group, device=device, dtype=torch.int64)
        ids = self.offsets_tensor(device)[:, None] + s[None, :]
        valid = s[None, :] < self.counts_tensor(device)[:, None].to(torch.int64)
        return torch.where(valid, ids, torch.full_like(ids, -1))

    def valid_mask(self, device) -> torch.Tensor:
        s = torch.arange(self.slots_per_group, device=device)
        return s[None, :] < self.counts_tensor(device)[:, None]

    # ---- shapes (layout.py:122-144) ----------------------------------------
    @property
    def index_shape(self):
        G, NB, C, K = self.groups, self.blocks_per_group, self.block, self.fan_in
        if self.packed:
            return (G, NB // self.unit_blocks, K, self.unit_blocks)
        return (G, NB, K) if self.shared_indices else (G, NB, C, K)

    @property
    def weight_shape(self):
        if self.packed:
            return (self.groups, self.blocks_per_group * self.n_tiles8 // 4, 32, 4, 2)
        return (self.groups, self.blocks_per_group, self.block, self.fan_in)

    @property
    def bias_shape(self):
        if self.packed:
            return (self.groups, self.blocks_per_group * self.n_tiles8 // 4, 4, 4, 2)
        return (self.groups, self.blocks_per_group, self.block)

    @property
    def canonical(self) -> "SparseLayout":
        return dataclasses.replace(self, packed=False)

    # ---- Mode B fragment packing: permutations (layout.py:146-179) ---------
    # Canonical weight element (g, blk, c, k) with fragment f = blk*NT + c//8,
    # quad = f // 4, fi = f % 4, n = c % 8, k = 2*kh + e sits at packed
    # [g, quad, n*4 + kh, fi, e]; bias (g, blk, c) with c%8 = 2*l4 + e at
    # [g, quad, l4, fi, e]; indices (g, blk, k) at [g, blk // UB, k, blk % UB].
    def pack_weights(self, w):
        G, Q = self.groups, self.blocks_per_group * self.n_tiles8 // 4
        v = w.reshape(G, Q, 4, 8, 4, 2)            # g, quad, fi, n, kh, e
        return v.permute(0, 1, 3, 4, 2, 5).reshape(self.weight_shape).contiguous()

    def unpack_weights(self, wp):
        G, Q = self.groups, self.blocks_per_group * self.n_tiles8 // 4
        v = wp.reshape(G, Q, 8, 4, 4, 2)           # g, quad, n, kh, fi, e
        return v.permute(0, 1, 4, 2, 3, 5).reshape(G, self.blocks_per_group, self.block, 8).contiguous()

    def pack_bias(self, b):
        G, Q = self.groups, self.blocks_per_group * self.n_tiles8 // 4
        v = b.reshape(G, Q, 4, 4, 2)               # g, quad, fi, l4, e
        return v.permute(0, 1, 3, 2, 4).reshape(self.bias_shape).contiguous()

    def unpack_bias(self, bp):
        G, Q = self.groups, self.blocks_per_group * self.n_tiles8 // 4
        v = bp.reshape(G, Q, 4, 4, 2)              # g, quad, l4, fi, e
        return v.permute(0, 1, 3, 2, 4).reshape(G, self.blocks_per_group, self.block).contiguous()

    def pack_indices(self, idx):
        G, NB, UB = self.groups, self.blocks_per_group, self.unit_blocks
        return idx.reshape(G, NB // UB, UB, 8).permute(0, 1, 3, 2).contiguous()

    def unpack_indices(self, ip):
        G, NB, UB = self.groups, self.blocks_per_group, self.unit_blocks
        return ip.permute(0, 1, 3, 2).reshape(G, NB, 8).contiguous()

    def to_canonical(self, idx, w, b):
        if not self.packed:
            return idx, w, b
        return self.unpack_indices(idx), self.unpack_weights(w), self.unpack_bias(b)

    def param_bytes(self, dtype_bytes: int = 2) -> dict:
        return {"weights": math.prod(self.weight_shape) * dtype_bytes,
                "bias": math.prod(self.bias_shape) * dtype_bytes,
                "indices": math.prod(self.index_shape) * 2}

    def padding_fraction(self) -> float:
        return 1.0 - self.hidden_dim / (self.groups * self.slots_per_group)


def _distinct_sorted_records(n_rec: int, d: int, k: int, gen: torch.Generator, device) -> torch.Tensor:
    """``n_rec`` records of ``k`` distinct indices in [0, d), each sorted.

    Same draws as layout.py:191-201: one int64 ``randint`` block, then every
    record holding a repeat is redrawn whole (new ``randint`` of just those
    rows) until no repeats remain; sorting happens before each repeat check.
    """
    rec = torch.randint(0, d, (n_rec, k), generator=gen, device=device, dtype=torch.int64)
    while True:
        rec = torch.sort(rec, dim=1).values
        bad = (rec[:, 1:] == rec[:, :-1]).any(dim=1)
        n_bad = int(bad.sum())
        if n_bad == 0:
            return rec
        rec[bad] = torch.randint(0, d, (n_bad, k), generator=gen, device=device, dtype=torch.int64)


@torch.no_grad()
def init_parameters(layout: SparseLayout, device, dtype=torch.bfloat16, seed: int = 0,
                    weight_std: float | None = None, bias_std: float = 0.0,
                    chunk_records: int = 1 << 22):
    """(indices, weights, bias) for ``layout`` with padding zeroed (layout.py:204-251).

    Draw order on one ``torch.Generator(device)`` seeded with ``seed``: all index
    records (chunks of ``chunk_records``), then all weights ``N(0, weight_std^2)``
    (default ``1/sqrt(8)``, chunks of ``chunk_records * 8`` values), then the bias
    ``N(0, bias_std^2)`` in one draw when ``bias_std > 0``.
    """
    if layout.packed:
        idx, w, b = init_parameters(layout.canonical, device, dtype, seed, weight_std, bias_std, chunk_records)
        return layout.pack_indices(idx), layout.pack_weights(w), layout.pack_bias(b)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    K = layout.fan_in
    std = 1.0 / math.sqrt(K) if weight_std is None else weight_std

    idx = torch.empty(layout.index_shape, dtype=torch.int16, device=device)
    recs = idx.view(-1, K)
    for lo in range(0, recs.shape[0], chunk_records):
        hi = min(lo + chunk_records, recs.shape[0])
        recs[lo:hi] = _distinct_sorted_records(hi - lo, layout.input_dim, K, gen, device).to(torch.int16)

    w = torch.empty(layout.weight_shape, dtype=dtype, device=device)
    wf = w.view(-1)
    step = chunk_records * K
    for lo in range(0, wf.numel(), step):
        hi = min(lo + step, wf.numel())
        wf[lo:hi] = (torch.randn(hi - lo, generator=gen, device=device) * std).to(dtype)

    b = torch.empty(layout.bias_shape, dtype=dtype, device=device)
    if bias_std > 0:
        b.copy_((torch.randn(b.shape, generator=gen, device=device) * bias_std).to(dtype))
    else:
        b.zero_()
    zero_padding_(layout, weights=w, bias=b, indices=idx)
    return idx, w, b


@torch.no_grad()
def windowed_indices(layout: SparseLayout, device, window: int = 512, supergroup: int = 4096, seed: int = 4,
                     chunk_records: int = 1 << 22) -> torch.Tensor:
    """Mode-A indices with input locality: the valid neurons, numbered group-major (global id
    ``offset_g + slot``), form supergroups of ``supergroup`` consecutive neurons; supergroup s draws
    every neuron's ``fan_in`` distinct sorted indices uniformly from its own window
    ``[o_s, o_s + window)``.  Padded slots hold 0.

    The reference has no Mode-A locality rule (its input supergroups are random feature subsets of
    Mode-B layers, supergroups.py:58-482); this is the benchmark's own seeded rule: one
    ``torch.Generator(device)`` seeded with ``seed`` draws all window offsets o_s ~ U{0 .. D - window}
    first, then the records in chunks with the same distinct-and-sorted redraw rule as
    ``init_parameters``.
    """
    if layout.shared_indices or layout.packed:
        raise ValueError("windowed_indices builds canonical Mode-A index tensors")
    D, K = layout.input_dim, layout.fan_in
    window = min(window, D)
    if window < K:
        raise ValueError(f"window {window} < fan_in {K}")
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    n_valid = layout.hidden_dim
    n_sg = -(-n_valid // supergroup)
    offs = torch.randint(0, D - window + 1, (n_sg,), generator=gen, device=device, dtype=torch.int64)
    recs = torch.empty((n_valid, K), dtype=torch.int16, device=device)
    for lo in range(0, n_valid, chunk_records):
        hi = min(lo + chunk_records, n_valid)
        r = _distinct_sorted_records(hi - lo, window, K, gen, device)
        sg = torch.arange(lo, hi, device=device) // supergroup
        recs[lo:hi] = (r + offs[sg][:, None]).to(torch.int16)
    idx = torch.zeros(layout.index_shape, dtype=torch.int16, device=device)
    G, NB, C = layout.groups, layout.blocks_per_group, layout.block
    counts = layout.counts_tensor(device).to(torch.int64)
    slots = torch.arange(NB * C, device=device)
    valid = (slots[None, :] < counts[:, None]).view(G, NB, C)
    idx[valid] = recs
    return idx


@torch.no_grad()
def zero_padding_(layout: SparseLayout, weights=None, bias=None, indices=None):
    """Zero the padded slots of weights, bias and Mode-A indices (layout.py:254-277).

    Mode-B index records are shared by valid and padded neurons of a block and
    stay untouched.
    """
    ref = next(t for t in (weights, bias, indices) if t is not None)
    G, NB, C = layout.groups, layout.blocks_per_group, layout.block
    counts = layout.counts_tensor(ref.device).to(torch.int64)
    slots = torch.arange(NB * C, device=ref.device)
    pad = (slots[None, :] >= counts[:, None]).view(G, NB, C)
    if layout.packed:
        if weights is not None:
            weights.masked_fill_(layout.pack_weights(pad[..., None].expand(G, NB, C, 8)), 0)
        if bias is not None:
            bias.masked_fill_(layout.pack_bias(pad), 0)
        return
    if weights is not None:
        weights.masked_fill_(pad[..., None], 0)
    if bias is not None:
        bias.masked_fill_(pad, 0)
    if indices is not None and not layout.shared_indices:
        indices.masked_fill_(pad[..., None], 0)
