"""Octet storage of Mode-A parameters (no counterpart in the reference).

``gl_group_octets`` (csrc/octets.cu) returns, per group, ``order[p]`` = the slot stored at position p and
``kperm[p]`` = that record's input order (bits 3c .. 3c+2: the original input index placed at column c).
Storing a layer's records that way lets the lane-per-neuron kernels (gl_fwd_octet_f32 / gl_bwd_octet_f32)
gather and scatter without shared-memory bank conflicts.  In octet storage the weights (and any
weight-shaped floating-point tensor: gradients, optimizer moments) are also interleaved per block of 32
consecutive records: the block stores the records' inputs 0-3 (16 bytes each, record j at 16 j), then their
inputs 4-7, so a warp's 16-byte weight loads and dW reductions cover whole 32-byte sectors.  These helpers
compute the arrangement, apply it to index-, weight- and bias-shaped tensors in place, and undo it
(``canonical``) for checkpoints and for callers that address neurons by slot.
"""
from __future__ import annotations

import torch

from . import _native


def unsupported(layout, pool: str, dtype: torch.dtype, device, plan=None):
    """Why the lane-per-neuron kernels cannot run a layer (None when they can).  Octet storage, with its
    interleaved weights, is read by those kernels only, so it is applied only when this returns None: Mode A,
    mean or sum pooling, fp32 parameters, int32 fixed-point dX (``b200_dx_accum`` not ``"fp32"``), and two
    16-byte-per-feature token tiles (32 D + 1024 bytes) within the GPU's opt-in shared memory per block."""
    if layout.shared_indices:
        return "Mode B layers keep their block storage"
    if pool not in ("mean", "sum"):
        return f"pool {pool!r} (mean and sum only)"
    if dtype != torch.float32:
        return f"{dtype} parameters (fp32 only)"
    if plan is not None and getattr(plan, "b200_dx_accum", "auto") == "fp32":
        return "b200_dx_accum='fp32' (the octet backward accumulates dX in int32 fixed point)"
    device = torch.device(device)
    if device.type != "cuda":
        return "parameters not on a GPU"
    optin = torch.cuda.get_device_properties(device).shared_memory_per_block_optin
    if 32 * layout.input_dim + 1024 > optin:
        return f"input_dim {layout.input_dim}: two 4-token tiles need {32 * layout.input_dim + 1024} bytes of " \
               f"shared memory, the GPU allows {optin}"
    return None


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


def _interleaved(t: torch.Tensor, kperm, per: int) -> bool:
    """Weight-shaped floating-point tensors of octet storage are interleaved per 32-record block."""
    return kperm is not None and per == 8 and t.is_floating_point()


@torch.no_grad()
def apply_(t: torch.Tensor, order: torch.Tensor, kperm=None) -> None:
    """Permute an index-, weight- or bias-shaped tensor (slot order) into storage order, in place: records by
    ``order`` and, for the 8-value records (indices, weights), their inputs by ``kperm``; with ``kperm``,
    weight-shaped floating-point tensors are then interleaved per 32-record block (module docstring)."""
    G, slots = order.shape
    per = t.numel() // (G * slots)
    v = t.view(G, slots, per)
    r = torch.gather(v, 1, order.long().to(t.device)[:, :, None].expand(G, slots, per))
    if kperm is not None and per == 8:
        r = torch.gather(r, 2, input_index(kperm.to(t.device)))
    if _interleaved(t, kperm, per):
        r = r.reshape(G, slots // 32, 32, 2, 4).transpose(2, 3)
    v.copy_(r.reshape(G, slots, per))


def canonical(t: torch.Tensor, order, kperm=None) -> torch.Tensor:
    """``t`` (index-, weight- or bias-shaped, in storage order) in slot order, as a new tensor."""
    if order is None:
        return t
    G, slots = order.shape
    per = t.numel() // (G * slots)
    src = t.reshape(G, slots, per)
    if _interleaved(t, kperm, per):
        src = src.reshape(G, slots // 32, 2, 32, 4).transpose(2, 3).reshape(G, slots, per)
    if kperm is not None and per == 8:
        rec = torch.empty_like(src)
        rec.scatter_(2, input_index(kperm.to(t.device)), src)
        src = rec
    out = torch.empty_like(t)
    out.view(G, slots, per).scatter_(1, order.long().to(t.device)[:, :, None].expand(G, slots, per), src)
    return out
