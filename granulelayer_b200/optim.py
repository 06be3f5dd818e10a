"""Fused Adam(W) over FP32 ``main_grad`` (mirror of sparse_pooling/optim.py).

``FusedAdamW.step`` reads each parameter's FP32 ``main_grad`` (or ``.grad``),
updates the parameter and its moments in place and zeroes the gradient, all
in one pass of the sm_100a kernel ``gl_adam_f32`` (the reference's
``_adamw_kernel``, optim.py:26-64).  The constructor, defaults and state layout
match optim.py:67-126 (``state[p] = {"step", "m", "v"[, "master"]}``): moments
in bf16 (default) or fp32, fp32 or bf16 parameters, for bf16 parameters an
optional fp32 master copy (``master_weights``) or stochastic rounding
(``stochastic_rounding``, default on).  Memory per element beyond the
parameter and its fp32 gradient: 4 B (bf16 moments), 8 B (fp32 moments),
+4 B with a master copy (optim.py:1-14).
"""
from __future__ import annotations

from typing import Iterable

import torch

from . import _native
from .autograd import UnsupportedOnB200


class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params: Iterable[torch.nn.Parameter], lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                 weight_decay=0.0, moments: str = "bf16", master_weights: bool = False,
                 stochastic_rounding: bool = True):
        if moments not in ("bf16", "fp32"):
            raise ValueError("moments must be 'bf16' or 'fp32'")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.moments = moments
        self.master_weights = master_weights
        self.stochastic_rounding = stochastic_rounding
        self._seed = 0

    def state_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for st in self.state.values() for t in st.values()
                   if torch.is_tensor(t))

    @torch.no_grad()
    def step(self, closure=None):
        mdt = torch.bfloat16 if self.moments == "bf16" else torch.float32
        for group in self.param_groups:
            b1, b2 = group["betas"]
            for p in group["params"]:
                g = getattr(p, "main_grad", None)
                if g is None:
                    if p.grad is None:
                        continue
                    g = p.grad.float().contiguous()
                if p.dtype not in (torch.float32, torch.bfloat16):
                    raise UnsupportedOnB200(f"the B200 optimizer updates fp32 or bf16 parameters (got {p.dtype})")
                if not p.is_contiguous() or not g.is_contiguous():
                    raise ValueError("FusedAdamW needs contiguous parameters and gradients")
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["m"] = torch.zeros(p.shape, device=p.device, dtype=mdt)
                    st["v"] = torch.zeros(p.shape, device=p.device, dtype=mdt)
                    if self.master_weights and p.dtype != torch.float32:
                        st["master"] = p.detach().float().clone()
                st["step"] += 1
                t = st["step"]
                self._seed += 1
                _native.adam(p, g, st["m"], st["v"], group["lr"], b1, b2, group["eps"], group["weight_decay"],
                             1 - b1 ** t, 1 - b2 ** t, zero_grad=True, master=st.get("master"),
                             stochastic=self.stochastic_rounding and p.dtype == torch.bfloat16, seed=self._seed)
                if getattr(p, "main_grad", None) is None:
                    p.grad = None
        return None
