"""Octet storage of Mode-A parameters (no counterpart in the reference).

``gl_group_octets`` (csrc/octets.cu) returns, per group, ``order[p]`` = the slot stored at position p and
``kperm[p]`` = that record's input order (bits 3c .. 3c+2: the original input index placed at column c).
Storing a layer's records that way lets the lane-per-neuron kernels (gl_fwd_octet_f32 / gl_bwd_octet_f32)
gather and scatter without shared-memory bank conflicts.  These helpers compute the arrangement, apply it
to index-, weight- and bias-shaped tensors in place, and undo it (``canonical``) for checkpoints and for
callers that address neurons by slot.
"""
from __future__ import annotations

import torch

from . import _native


def arrange(indices: torch.Tensor, counts: torch.Tensor, input_dim: int, blocks_per_group: int):
    """(order, kperm) [G, NB*8] int32 of Mode-A ``indices`` [G, NB, 8, 8] (CUDA tensors)."""
    G, slots = indices.shape[0], blocks_per_group * 8
    order = torch.empty((G, slots), dtype=torch.int32, device=indices.device)
    kperm = torch.empty_like(order)
    _native.group_octets(indices, counts.to(torch.int32).contiguous(), input_dim, blocks_per_group, 0, G, order,
                         kperm)
    return order, kperm


def input_index(kperm: torch.Tensor) -> torch.Tensor:
    """[G, slots, 8] int64: the original input index placed at each column (bits 3c .. 3c+2 of kperm)."""
    sh = torch.arange(0, 24, 3, device=kperm.device, dtype=torch.int32)
    return ((kperm[:, :, None] >> sh) & 7).long()


@torch.no_grad()
def apply_(t: torch.Tensor, order: torch.Tensor, kperm=None) -> None:
    """Permute an index-, weight- or bias-shaped tensor (slot order) into storage order, in place: records by
    ``order`` and, for the 8-value records (indices, weights), their inputs by ``kperm``."""
    G, slots = order.shape
    per = t.numel() // (G * slots)
    v = t.view(G, slots, per)
    r = torch.gather(v, 1, order.long().to(t.device)[:, :, None].expand(G, slots, per))
    if kperm is not None and per == 8:
        r = torch.gather(r, 2, input_index(kperm.to(t.device)))
    v.copy_(r)


def canonical(t: torch.Tensor, order, kperm=None) -> torch.Tensor:
    """``t`` (index-, weight- or bias-shaped, in storage order) in slot order, as a new tensor."""
    if order is None:
        return t
    G, slots = order.shape
    per = t.numel() // (G * slots)
    src = t.reshape(G, slots, per)
    if kperm is not None and per == 8:
        rec = torch.empty_like(src)
        rec.scatter_(2, input_index(kperm.to(t.device)), src)
        src = rec
    out = torch.empty_like(t)
    out.view(G, slots, per).scatter_(1, order.long().to(t.device)[:, :, None].expand(G, slots, per), src)
    return out
