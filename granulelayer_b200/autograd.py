"""Autograd contract and launch orchestration (mirror of sparse_pooling/autograd.py).

``SparsePoolFunction`` keeps the reference's contract (autograd.py:380-414):
forward saves ``(x, w, b, pre)`` and nothing of size [B, H]; backward forms
``g_pre = dy * out_act'(pre)``, accumulates dW/db into the FP32 ``main_grad``
buffers when present (returning None for them), else into temporary FP32
buffers returned in the parameter dtype, and returns dX in ``x.dtype``.

``Level1Runtime`` replaces the reference's runtime (autograd.py:68-300) for
the B200 path.  Its ``forward`` returns ``{"pre": [B, G] fp32}`` and its
``backward`` returns dX [B, D] fp32 after accumulating dW/db, the same
protocol the reference's backends implement (autograd.py:220-223, 265-267).
Both call the sm_100a library through its C ABI; there is no Triton, no
backend dispatch and no CPU fallback: an unsupported layer or a CPU tensor
raises.
"""
from __future__ import annotations

from typing import Dict, Optional

import math

import torch

from . import _native
from .config import B200_POOLS, LevelSpec, PhysicalPlan, resolve_reduction
from .layout import SparseLayout

# checkpoint policy per operator when "auto" (autograd.py:31-38)
AUTO_POLICY = {"max": "save_winners", "topk_mean": "save_winners", "mean": "minimal_stats",
               "logmeanexp": "minimal_stats", "power_mean": "minimal_stats", "softmax_weighted": "minimal_stats",
               "sum": "minimal_stats"}


def resolve_policy(level: LevelSpec, requested: str) -> str:
    """autograd.py:60-65: "auto" maps per operator; save_winners needs winners."""
    if requested == "auto":
        return AUTO_POLICY[level.type]
    if requested == "save_winners" and level.type not in ("max", "topk_mean"):
        return "minimal_stats"
    return requested


def act_torch(x: torch.Tensor, name: str) -> torch.Tensor:
    """Activation of the pooled value (kernels/ops.py:165-170)."""
    if name == "identity":
        return x
    if name == "relu":
        return torch.relu(x)
    return torch.nn.functional.gelu(x)


def dact_torch(x: torch.Tensor, name: str) -> torch.Tensor:
    """Derivative of ``act_torch`` (kernels/ops.py:173-179)."""
    if name == "identity":
        return torch.ones_like(x)
    if name == "relu":
        return (x > 0).to(x.dtype)
    cdf = 0.5 * (1 + torch.erf(x * 0.7071067811865476))
    return cdf + x * 0.3989422804014327 * torch.exp(-0.5 * x * x)


def kernel_param(level: LevelSpec) -> float:
    """The kernels' pool parameter: log2(e)/tau (LogMeanExp), log2(e)*beta (softmax-weighted), p (power
    mean); kernels/ops.py:74-79."""
    if level.type == "logmeanexp":
        return LOG2E / level.temperature
    if level.type == "softmax_weighted":
        return LOG2E * level.beta
    if level.type == "power_mean":
        return float(level.p)
    return 0.0


LOG2E = 1.0 / math.log(2.0)


class UnsupportedOnB200(NotImplementedError):
    """The layer configuration is outside the sm_100a hot path."""


def check_supported(layout: SparseLayout, level: LevelSpec, dtype: torch.dtype, semantic: bool = False):
    """Raise UnsupportedOnB200 for a level-1 configuration the kernels do not run."""
    if not layout.shared_indices and layout.block != 8:
        raise UnsupportedOnB200("Mode A layers store blocks of 8 neurons")
    if level.type not in B200_POOLS:
        raise UnsupportedOnB200(f"pooling {level.type!r} is not on the B200 path (supported: {B200_POOLS})")
    if level.neurons_per_shard is not None and not semantic:
        raise UnsupportedOnB200("neurons_per_shard belongs to a two-level configuration")
    if dtype not in (torch.float32, torch.bfloat16):
        raise UnsupportedOnB200(f"the B200 kernels read float32 or bfloat16 parameters (layer dtype {dtype})")


class Level1Runtime:
    """Launches the B200 kernels for one single-level layer (or one group shard).

    ``counts`` holds the valid-neuron count of each local group; ``g0:g1`` of the
    parameter tensors are processed (the whole tensor by default).
    """

    def __init__(self, layout: SparseLayout, idx: torch.Tensor, level: LevelSpec, plan: PhysicalPlan,
                 counts: Optional[torch.Tensor] = None):
        self.layout = layout
        self.idx = idx
        self.level = level
        self.plan = plan
        G = idx.shape[0]
        self.counts_i32 = (counts if counts is not None else layout.counts_tensor(idx.device)).to(
            device=idx.device, dtype=torch.int32).contiguous()
        if self.counts_i32.numel() != G:
            raise ValueError(f"counts has {self.counts_i32.numel()} entries for {G} groups")
        self.counts_f32 = self.counts_i32.to(torch.float32)
        self.pool = {"mean": _native.POOL_MEAN, "sum": _native.POOL_SUM, "max": _native.POOL_MAX,
                     "logmeanexp": _native.POOL_LME, "power_mean": _native.POOL_POWER,
                     "softmax_weighted": _native.POOL_SOFTMAX, "topk_mean": _native.POOL_TOPK}.get(
                         level.type, _native.POOL_MEAN)
        self.k = level.k if level.type == "topk_mean" else 1   # slots per (token, group) of the event pools
        self.param = kernel_param(level)
        self.param_dtype = torch.float32   # storage type of w and b (set by the layer)
        self.act = _native.ACT_IDS[level.activation]
        self.last_info: Dict = {}
        self.det = False
        self._rowmax = None
        self._rowmax_key = None
        self._orders: Dict = {}
        self.sets = None   # (feat [Q, S], buckets [n, 4]) of a layer with input-supergroup connectivity
        self.octets = False   # storage in octet order (gl_group_octets): the lane-per-neuron kernels
        self._local = None

    def set_plan(self):
        """(chunks [m, 3] int32, largest chunk, bucket bounds [n] int32) of the input-set backward, once per
        graph: each chunk holds consecutive buckets of one set, at most SET_MAX_CHUNK of them and about
        TARGET quads; a bucket's bound is the largest number of its record inputs on one feature."""
        feat, buckets = self.sets
        key = (self.idx.data_ptr(), buckets.data_ptr(), buckets.shape[0])
        if getattr(self, "_set_plan_key", None) == key:
            return self._set_plan
        L = self.layout
        C, UB, D = L.block, L.unit_blocks, L.input_dim
        nt = C // 8
        qpu = nt // 4 if nt >= 4 else 1
        bk = buckets.to("cpu", torch.int64)
        quads = (bk[:, 3] * qpu).tolist()
        qs = bk[:, 0].tolist()
        target, chunks, start, acc = 4096, [], 0, 0   # per-CTA staging and flush amortised over ~4k quads
        for i in range(len(qs)):
            if i > start and (qs[i] != qs[start] or i - start >= _native.SET_MAX_CHUNK or acc >= target):
                chunks.append((qs[start], start, i))
                start, acc = i, 0
            acc += quads[i]
        if qs:
            chunks.append((qs[start], start, len(qs)))
        largest = max((e - a for _, a, e in chunks), default=1)
        ch = torch.tensor(chunks, dtype=torch.int32).reshape(-1, 3).to(self.idx.device)
        # per-bucket bound: counts of (record, input) per feature over the bucket's blocks
        idx = self.idx.permute(0, 1, 3, 2).reshape(self.idx.shape[0], -1, 8) if L.packed else self.idx
        dev = idx.device
        bkd = bk.to(dev)
        nblk = bkd[:, 3] * UB
        bid = torch.repeat_interleave(torch.arange(bkd.shape[0], device=dev), nblk)
        first = torch.repeat_interleave(bkd[:, 2] * UB, nblk)
        within = torch.arange(int(nblk.sum()), device=dev) - torch.repeat_interleave(torch.cumsum(nblk, 0) - nblk, nblk)
        blk = first + within
        g = bkd[bid, 1]
        f = idx[g, blk].long().clamp_(0, D - 1)                     # [nblocks, 8]
        Q, S = feat.shape
        lmap = torch.zeros(Q, D, dtype=torch.int64, device=dev)
        lmap.scatter_(1, feat.long().clamp(0, D - 1), torch.arange(S, device=dev).expand(Q, S).contiguous())
        local = lmap[bkd[bid, 0][:, None], f]                       # positions in the bucket's set
        cnt = torch.bincount((bid[:, None] * S + local).reshape(-1), minlength=bkd.shape[0] * S)
        rowmax = cnt.reshape(-1, S).amax(1).to(torch.int32).contiguous()
        self._set_plan, self._set_plan_key = (ch, largest, rowmax), key
        return self._set_plan

    def record_rowmax(self) -> torch.Tensor:
        """[G] int32: for each group, the largest number of inputs of its valid Mode-B records (blocks
        holding a valid slot) on one feature, the bound of the fixed-point dX tile.  Depends only on the
        indices; computed once per index tensor."""
        key = (self.idx.data_ptr(), self.idx.shape, self.counts_i32.data_ptr())
        if getattr(self, "_rec_rowmax_key", None) != key:
            idx = self.idx
            if self.layout.packed:   # [G, NB/UB, 8, UB] -> [G, NB, 8]
                idx = idx.permute(0, 1, 3, 2)
            G, D, C = idx.shape[0], self.layout.input_dim, self.layout.block
            idx = idx.reshape(G, -1, 8)
            NB = idx.shape[1]
            valid = (torch.arange(NB, device=idx.device) * C)[None, :] < self.counts_i32[:, None]
            out = torch.zeros(G, device=idx.device, dtype=torch.int32)
            step = max(1, (1 << 24) // max(1, NB * 8))
            for a in range(0, G, step):
                e = min(G, a + step)
                sub = idx[a:e].long().clamp_(0, D - 1).reshape(e - a, -1)
                wts = valid[a:e, :, None].expand(e - a, NB, 8).reshape(e - a, -1).to(torch.int32)
                cnt = torch.zeros(e - a, D, device=idx.device, dtype=torch.int32)
                cnt.scatter_add_(1, sub, wts)
                out[a:e] = cnt.amax(1)
            self._rec_rowmax, self._rec_rowmax_key = out.contiguous(), key
        return self._rec_rowmax

    @property
    def tensor_cores(self) -> bool:
        """bf16 fragment-packed Mode-B mean / sum / max layers run the tensor-core kernels, with x rounded
        to bf16 (the reference's compute dtype for a bf16 layer, autograd.py:349-354)."""
        return (self.plan.b200_bf16_tensor_cores == "auto" and self.param_dtype == torch.bfloat16
                and self.layout.shared_indices and self.layout.packed
                and self.pool in (_native.POOL_MEAN, _native.POOL_SUM, _native.POOL_MAX)
                and self.idx.is_cuda and _native.shared_tc_tokens(self.layout.input_dim, False) > 0)

    def input_sets(self) -> bool:
        """Layers with input-supergroup connectivity: the input-set kernels (forward for mean / sum,
        backward) run when requested (cuda_input_supergroup_backend = "grouped") or, under "auto", when
        the generic tensor-core backward's full-row tiles do not fit in shared memory (large D); at
        D = 1024 the two backwards measure the same (C = 64) or the generic one is 4% faster (C = 8)."""
        mode = self.plan.cuda_input_supergroup_backend
        if self.sets is None or mode == "generic":
            return False
        return mode == "grouped" or _native.shared_tc_tokens(self.layout.input_dim, True) < 0

    @property
    def fixed_point(self) -> bool:
        return self.plan.b200_dx_accum in ("auto", "fixed")

    def rowmax(self) -> torch.Tensor:
        """Per-group max number of records sharing one input feature (depends only on
        the indices; recomputed when the index tensor changes)."""
        key = (self.idx.data_ptr(), self.idx._version)
        if self._rowmax is None or self._rowmax_key != key:
            out = torch.empty(self.groups, device=self.idx.device, dtype=torch.int32)
            _native.group_index_maxcount(self.idx, self.counts_i32, self.layout.input_dim,
                                         self.layout.blocks_per_group, 0, self.groups, out)
            self._rowmax, self._rowmax_key = out, key
        return self._rowmax

    def feature_prefix(self) -> torch.Tensor:
        """Record inputs per feature cumulated over the groups ((G+1) x D int32, gl_group_feature_prefix), which
        the lane-per-neuron backward subtracts its rounding offsets by; depends only on the indices and counts,
        recomputed when the index tensor changes."""
        key = (self.idx.data_ptr(), self.idx._version, self.counts_i32.data_ptr())
        if getattr(self, "_fprefix_key", None) != key:
            D = self.layout.input_dim
            out = torch.empty((self.groups + 1) * D, device=self.idx.device, dtype=torch.int32)
            _native.group_feature_prefix(self.idx, self.counts_i32, D, self.layout.blocks_per_group, 0, self.groups,
                                         out)
            self._fprefix, self._fprefix_key = out, key
        return self._fprefix

    def order(self, tokens: int) -> Optional[torch.Tensor]:
        """Bank-aware processing order for a kernel running token tiles of ``tokens`` (one wavefront
        serves 32 / tokens neurons; orders are built for 4 and 8), or None for slot order.  Depends
        only on the indices; recomputed when the index tensor changes."""
        unit = 32 // tokens if tokens > 0 else 0
        if self.plan.b200_neuron_order == "identity" or unit not in (4, 8) or self.groups == 0:
            return None
        key = (self.idx.data_ptr(), self.idx._version, unit)
        out = self._orders.get(unit)
        if out is None or out[0] != key:
            o = torch.empty((self.groups, self.layout.blocks_per_group * 8), device=self.idx.device,
                            dtype=torch.int32)
            _native.group_order(self.idx, self.counts_i32, self.layout.input_dim, self.layout.blocks_per_group, 0,
                                self.groups, unit, o)
            out = (key, o)
            self._orders[unit] = out
        return out[1]

    def locality(self):
        """(lidx, fmap, nfeat) when every group reads at most a quarter of the input features (the
        kernels then stage only each group's features), else None.  Built once per index tensor.
        The smooth pools (LogMeanExp, power mean, softmax-weighted), top-K and bf16 storage run on the
        full-row staging."""
        if (self.plan.b200_locality == "off" or self.layout.shared_indices or not self.idx.is_cuda
                or self.smooth or self.pool == _native.POOL_TOPK or self.param_dtype != torch.float32):
            return None
        G, D, NB = self.groups, self.layout.input_dim, self.layout.blocks_per_group
        if G == 0 or G > 65535 or D < 256:
            return None
        key = (self.idx.data_ptr(), self.idx._version)
        if self._local is not None and self._local[0] == key:
            return self._local[1]
        nf = torch.empty(G, device=self.idx.device, dtype=torch.int32)
        _native.group_feature_map(self.idx, self.counts_i32, D, NB, 0, G, nf)
        fmax = int(nf.max())
        maps = None
        if fmax <= D // 4:
            cap = -(-fmax // 8) * 8
            fmap = torch.zeros((G, cap), device=self.idx.device, dtype=torch.int16)
            lidx = torch.empty_like(self.idx)
            _native.group_feature_map(self.idx, self.counts_i32, D, NB, 0, G, nf, fmap, lidx)
            maps = (lidx, fmap, nf)
        self._local = (key, maps)
        return maps

    def octet_kernels(self, B: int, D: int) -> bool:
        """Whether this call runs the lane-per-neuron kernels (gl_fwd_octet_f32 / gl_bwd_octet_f32): every
        non-empty call on octet storage does, since no other kernel reads its interleaved weights; a layer
        changed after its storage was arranged (parameter dtype, pool, plan) raises instead of running
        another kernel on that storage."""
        if not self.octets or B == 0:
            return False
        from . import octet_storage

        why = octet_storage.unsupported(self.layout, self.level.type, self.param_dtype, self.idx.device, self.plan)
        if why is not None:
            raise RuntimeError(f"octet storage cannot run this call: {why}")
        return True

    def tokens(self, backward: bool) -> int:
        lib = _native.load()
        D = self.layout.input_dim
        if backward:
            return self.plan.b200_dx_tokens or lib.gl_bwd_auto_tokens(D)
        return self.plan.b200_fwd_tokens or lib.gl_fwd_auto_tokens(D)

    @property
    def groups(self) -> int:
        return self.idx.shape[0]

    def check_devices(self, *tensors):
        dev = self.idx.device
        for t in tensors:
            if t is not None and t.device != dev:
                raise ValueError(f"tensor on {t.device} but the layer's parameters are on {dev} "
                                 "(move the input or the layer)")

    def deterministic_reason(self) -> Optional[str]:
        """Why reduction='deterministic' is unavailable for this layer, or None.  The deterministic
        backward covers Mode-B layers with the mean / sum pools (the reference's deterministic path
        covers packed Mode-B Mean layers, README "Deterministic execution").  The forwards and Adam
        already sum in a fixed order; the Mode-A, event (max / top-K) and smooth-pool backwards use
        FP32 atomics."""
        if not self.layout.shared_indices:
            return "Mode-A layers accumulate dX with FP32 atomics"
        if self.pool not in (_native.POOL_MEAN, _native.POOL_SUM):
            return f"the deterministic backward covers the mean / sum pools, not {self.level.type}"
        return None

    def resolve_reduction(self, B: int) -> bool:
        mode, why, strict = resolve_reduction(self.plan)
        if mode == "deterministic":
            reason = self.deterministic_reason()
            if reason is not None:
                msg = f"reduction='deterministic' ({why}) is unsupported for this layer: {reason}"
                if strict:
                    raise ValueError(msg)
                import warnings

                warnings.warn(msg + "; running reduction='fast'", stacklevel=4)
                mode, why = "fast", why + f"; unsupported ({reason}) -> fast (warn_only)"
        self.det = mode == "deterministic"
        self.last_info["reduction"] = {"mode": mode, "reason": why}
        return self.det

    def det_scales(self, w: torch.Tensor, g_pre: torch.Tensor):
        """(qscale, qinv) [B]: the per-token power-of-two scales of the deterministic dX accumulation,
        2^e with sum_d |dx[t, d]| 2^e <= 2^60 by the bound sum_g |c1[t, g]| n_g 8 max|w|_g max|act'|."""
        G = self.groups
        wmax = w.reshape(G, -1).abs().amax(1).float()
        n = self.counts_f32
        per = 8.0 * wmax * (1.0 if self.pool == _native.POOL_MEAN else n)   # |c1| n_g = |g_pre| for mean
        dmax = 1.13 if self.level.activation == "gelu" else 1.0
        bound = (g_pre.abs() * per[None, :]).sum(1) * dmax
        e = torch.clamp(torch.floor(60.0 - torch.log2(bound)), min=-126.0, max=126.0)
        finite = torch.isfinite(bound)
        e = torch.where(finite, e, torch.zeros_like(e))
        qscale = torch.where(finite, torch.exp2(e), torch.zeros_like(e)).contiguous()
        qinv = torch.where(finite, torch.exp2(-e), torch.full_like(e, float("nan"))).contiguous()
        return qscale, qinv

    def describe_execution(self, B: int) -> Dict:
        lib = _native.load()
        D = self.layout.input_dim
        if self.layout.shared_indices:
            return {
                "backend": "b200",
                "library": str(_native.library_path()),
                "mode": f"B (C={self.layout.block}, {'packed' if self.layout.packed else 'canonical'})",
                "forward": {"kernel": "gl_fwd_shared_f32",
                            "tokens": self.plan.b200_fwd_tokens or lib.gl_shared_auto_tokens(D, 0)},
                "backward": {"kernel": "gl_bwd_shared_f32",
                             "tokens": self.plan.b200_dx_tokens or lib.gl_shared_auto_tokens(D, 1)},
                "optimizer": {"kernel": "gl_adam_f32"},
                "batch": B,
            }
        return {
            "backend": "b200",
            "library": str(_native.library_path()),
            "forward": {"kernel": "gl_fwd_f32", "tokens": self.plan.b200_fwd_tokens or lib.gl_fwd_auto_tokens(D)},
            "backward": {"kernel": "gl_bwd_f32", "tokens": self.plan.b200_dx_tokens or lib.gl_bwd_auto_tokens(D)},
            "optimizer": {"kernel": "gl_adam_f32"},
            "batch": B,
        }

    @property
    def is_max(self) -> bool:
        """Max or top-K: winner slots in the forward, the winner-event backward."""
        return self.pool in (_native.POOL_MAX, _native.POOL_TOPK)

    @property
    def smooth(self) -> bool:
        """LogMeanExp, power mean or softmax-weighted: dense backward from per-(token, group)
        coefficients (kernels/ops.py:242-262)."""
        return self.pool in (_native.POOL_LME, _native.POOL_POWER, _native.POOL_SOFTMAX)

    def coefficients(self, g_pre: torch.Tensor, stats: Dict):
        """(c1, c2, c3) of the smooth pools (kernels/ops.py:242-262); L2 comes from the forward (softmax)
        or from pre (LogMeanExp)."""
        n = self.counts_f32[None, :]
        pre = stats["pre"]
        if self.pool == _native.POOL_LME:
            L2 = stats.get("L2")
            if L2 is None:
                L2 = pre * self.param + torch.log2(n)
            return g_pre, L2.contiguous(), None
        if self.pool == _native.POOL_POWER:
            pos = pre > 0
            zero = torch.zeros_like(g_pre)
            c1 = torch.where(pos, g_pre / n, zero)
            c2 = torch.where(pos, 1.0 / torch.where(pos, pre, torch.ones_like(pre)), zero)
            return c1.contiguous(), c2.contiguous(), None
        return g_pre, stats["L2"].contiguous(), pre.contiguous()

    def forward(self, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, track_ids: bool = False):
        """{"pre": [B, G] pooled values, "wabsmax": [G] max |w| per group (Mode A mean/sum, for the
        backward), "winner": [B, G] int32 winning slots (max pooling, when ``track_ids``)}."""
        B = x.shape[0]
        self.check_devices(x, w, b)
        self.resolve_reduction(B)
        pre = torch.empty((B, self.groups), device=x.device, dtype=torch.float32)
        winners = (torch.empty((B, self.groups * self.k), device=x.device, dtype=torch.int32)
                   if self.is_max and track_ids else None)
        stat = (torch.empty((B, self.groups), device=x.device, dtype=torch.float32)
                if self.pool in (_native.POOL_LME, _native.POOL_SOFTMAX) else None)
        out = {"pre": pre}
        if winners is not None:
            out["winner"] = winners
        if stat is not None:
            out["L2"] = stat
        if self.tensor_cores and B > 0 and self.pool in (_native.POOL_MEAN, _native.POOL_SUM) and self.input_sets():
            chunks, largest, _ = self.set_plan()
            _native.fwd_shared_tc_sets(x, self.idx, w, b, self.counts_i32, pre, self.layout.blocks_per_group,
                                       self.layout.block, 0, self.groups, self.pool, self.act, self.sets[0],
                                       self.sets[1], chunks, largest, tokens=self.plan.b200_fwd_tokens)
            self.last_info.update(forward_backend="b200", forward_kernel="gl_fwd_shared_tc_sets", workspace_bytes=0)
            return out
        if self.tensor_cores:
            _native.fwd_shared_tc(x, self.idx, w, b, self.counts_i32, pre, self.layout.blocks_per_group,
                                  self.layout.block, 0, self.groups, self.pool, self.act, winners=winners)
            self.last_info.update(forward_backend="b200", forward_kernel="gl_fwd_shared_tc", workspace_bytes=0)
            return out
        if self.layout.shared_indices:
            _native.fwd_shared(x, self.idx, w, b, self.counts_i32, pre, self.layout.blocks_per_group,
                               self.layout.block, 0, self.groups, self.pool, self.act, self.layout.packed,
                               tokens=self.plan.b200_fwd_tokens, winners=winners, stat=stat, param=self.param,
                               k=self.k)
            self.last_info.update(forward_backend="b200", forward_kernel="gl_fwd_shared_f32", workspace_bytes=0)
            return out
        wabsmax = (torch.empty(self.groups, device=x.device, dtype=torch.float32)
                   if B > 0 and not self.is_max and not self.smooth else None)
        if self.octet_kernels(B, x.shape[1]):
            _native.fwd_octet(x, self.idx, w, b, self.counts_i32, pre, self.layout.blocks_per_group, 0, self.groups,
                              self.pool, self.act, wabsmax=wabsmax)
            self.last_info.update(forward_backend="b200", forward_kernel="gl_fwd_octet_f32", workspace_bytes=0)
            out["wabsmax"] = wabsmax
            return out
        _native.fwd(x, self.idx, w, b, self.counts_i32, pre, self.layout.blocks_per_group, 0, self.groups,
                    self.pool, self.act, tokens=self.plan.b200_fwd_tokens, wabsmax=wabsmax,
                    order=self.order(self.tokens(False)) if B > 0 else None,
                    local=self.locality() if B > 0 else None, winners=winners, stat=stat, param=self.param,
                    k=self.k)
        self.last_info.update(forward_backend="b200", workspace_bytes=0)
        if wabsmax is not None:
            out["wabsmax"] = wabsmax
        return out

    def _event_backward(self, x, w, b, g_pre, saved, dw_buf, db_buf) -> torch.Tensor:
        """Max / top-K pooling: one event per chosen slot of each (token, group), coefficient
        dL/dpre (divided by min(k, n) for top-K) (autograd.py:280-290); the slots come from the forward
        (save_winners) or are recomputed here (minimal_stats)."""
        winners = saved.get("winner")
        recomputed = winners is None
        if recomputed:
            winners = self.forward(x, w, b, track_ids=True)["winner"]
        self.last_info["recomputed_stats"] = recomputed
        coef = g_pre
        if self.pool == _native.POOL_TOPK:
            coef = (g_pre / torch.clamp(self.counts_f32, max=float(self.k))[None, :]).contiguous()
        dx = torch.zeros(x.shape, device=x.device, dtype=torch.float32)
        L = self.layout
        _native.bwd_events(x, self.idx, w, b, winners, coef, dx, dw_buf, db_buf, L.blocks_per_group, L.block,
                           L.shared_indices, L.packed, 0, self.groups, self.act, kev=self.k)
        self.last_info["backward_backend"] = "b200"
        self.last_info["backward_kernel"] = "gl_bwd_events_f32"
        return dx

    def backward(self, x, w, b, g_pre: torch.Tensor, saved: Dict, policy: str, dw_buf: torch.Tensor,
                 db_buf: torch.Tensor, recomputed: bool = False) -> torch.Tensor:
        B, D = x.shape
        self.last_info["policy"] = policy
        self.last_info["recomputed_stats"] = recomputed
        self.check_devices(x, w, b, g_pre, dw_buf, db_buf)
        self.resolve_reduction(B)
        if self.is_max:
            return self._event_backward(x, w, b, g_pre, saved, dw_buf, db_buf)
        c1, c2, c3 = g_pre, None, None
        if self.smooth:
            stats = dict(saved)
            if self.pool == _native.POOL_SOFTMAX and "L2" not in stats:   # autograd.py:246-261
                stats.update(self.forward(x, w, b))
                self.last_info["recomputed_stats"] = True
            c1, c2, c3 = self.coefficients(g_pre, stats)
        dx = torch.zeros((B, D), device=x.device, dtype=torch.float32)
        if self.layout.shared_indices and self.det and B > 0:
            qscale, qinv = self.det_scales(w, g_pre)
            dxq = torch.zeros((B, D), device=x.device, dtype=torch.int64)
            _native.bwd_shared_det(x, self.idx, w, b, self.counts_i32, g_pre, dx, dw_buf, db_buf,
                                   self.layout.blocks_per_group, self.layout.block, 0, self.groups, self.pool,
                                   self.act, self.layout.packed, dxq, qscale, qinv)
            self.last_info["backward_backend"] = "b200"
            self.last_info["backward_kernel"] = "gl_bwd_shared_det_f32"
            self.last_info["dx_accumulation"] = "int64 fixed point per token (deterministic)"
            return dx
        if self.tensor_cores and not self.is_max and B > 0 and self.input_sets():
            chunks, largest, brow = self.set_plan()
            wabsmax = rowmax = None
            if self.fixed_point:
                wabsmax = w.reshape(self.groups, -1).abs().amax(1).float().contiguous()
                rowmax = brow
            _native.bwd_shared_tc_sets(x, self.idx, w, b, self.counts_i32, c1, dx, dw_buf, db_buf,
                                       self.layout.blocks_per_group, self.layout.block, 0, self.groups, self.pool,
                                       self.act, self.sets[0], self.sets[1], chunks, largest, rowmax=rowmax,
                                       wabsmax=wabsmax, tokens=self.plan.b200_dx_tokens)
            self.last_info["backward_backend"] = "b200"
            self.last_info["backward_kernel"] = "gl_bwd_shared_tc_sets"
            self.last_info["dx_accumulation"] = ("int32 fixed point" if wabsmax is not None else "fp32 atomics") + \
                " of tensor-core partials over input sets (Mode B)"
            return dx
        if (self.tensor_cores and not self.is_max and B > 0
                and _native.shared_tc_tokens(self.layout.input_dim, True) > 0):
            wabsmax = rowmax = None
            if self.fixed_point:
                wabsmax = w.reshape(self.groups, -1).abs().amax(1).float().contiguous()
                rowmax = self.record_rowmax()
            _native.bwd_shared_tc(x, self.idx, w, b, self.counts_i32, c1, dx, dw_buf, db_buf,
                                  self.layout.blocks_per_group, self.layout.block, 0, self.groups, self.pool, self.act,
                                  wabsmax=wabsmax, rowmax=rowmax)
            self.last_info["backward_backend"] = "b200"
            self.last_info["backward_kernel"] = "gl_bwd_shared_tc"
            self.last_info["dx_accumulation"] = ("int32 fixed point" if wabsmax is not None else "fp32 atomics") + \
                " of tensor-core partials (Mode B)"
            return dx
        if self.layout.shared_indices:
            _native.bwd_shared(x, self.idx, w, b, self.counts_i32, c1, dx, dw_buf, db_buf,
                               self.layout.blocks_per_group, self.layout.block, 0, self.groups, self.pool, self.act,
                               self.layout.packed, tokens=self.plan.b200_dx_tokens, c2=c2, c3=c3, param=self.param)
            self.last_info["backward_backend"] = "b200"
            self.last_info["backward_kernel"] = "gl_bwd_shared_f32"
            self.last_info["dx_accumulation"] = "fp32 shared-memory reductions (Mode B)"
            return dx
        wabsmax = rowmax = None
        if self.fixed_point and B > 0 and not self.smooth:
            wabsmax = saved.get("wabsmax")
            if wabsmax is None and (w.dtype != torch.float32 or self.octets):   # padding slots hold zeros
                wabsmax = w.reshape(self.groups, -1).abs().amax(1).float().contiguous()
            elif wabsmax is None:
                wabsmax = torch.empty(self.groups, device=x.device, dtype=torch.float32)
                _native.group_absmax(w, self.counts_i32, self.layout.blocks_per_group, 0, self.groups, wabsmax)
            rowmax = self.rowmax()
            if self.octet_kernels(B, D):
                _native.bwd_octet(x, self.idx, w, b, self.counts_i32, c1, dx, dw_buf, db_buf,
                                  self.layout.blocks_per_group, 0, self.groups, self.pool, self.act, wabsmax, rowmax,
                                  feat_prefix=self.feature_prefix())
                self.last_info["backward_backend"] = "b200"
                self.last_info["backward_kernel"] = "gl_bwd_octet_prefix_f32"
                self.last_info["dx_accumulation"] = "int32 fixed point"
                return dx
        _native.bwd(x, self.idx, w, b, self.counts_i32, c1, dx, dw_buf, db_buf, self.layout.blocks_per_group,
                    0, self.groups, self.pool, self.act, tokens=self.plan.b200_dx_tokens, wabsmax=wabsmax,
                    rowmax=rowmax, order=self.order(self.tokens(True)) if B > 0 else None,
                    local=self.locality() if B > 0 else None, c2=c2, c3=c3, param=self.param)
        self.last_info["backward_backend"] = "b200"
        self.last_info["dx_accumulation"] = "int32 fixed point" if wabsmax is not None else "fp32 atomics"
        return dx


def _compute_operands(x, w, b):
    """x in the layer's compute dtype, as autograd.py:349-354 casts it (a bf16 layer computes on x rounded
    to bf16), held as the fp32 unit-stride rows the kernels read (bf16 values widen exactly)."""
    xc = x.to(w.dtype).to(torch.float32) if w.dtype == torch.bfloat16 else x.to(torch.float32)
    if xc.dim() != 2 or xc.stride(1) != 1:
        xc = xc.contiguous()
    return xc, w.contiguous(), b.contiguous()


def _grad_buffers(w, b):
    """main_grad when both exist (accumulate), else zeroed temporaries (autograd.py:357-363)."""
    mg_w = getattr(w, "main_grad", None)
    mg_b = getattr(b, "main_grad", None)
    if mg_w is not None and mg_b is not None:
        return mg_w, mg_b, True
    return (torch.zeros(w.shape, device=w.device, dtype=torch.float32),
            torch.zeros(b.shape, device=b.device, dtype=torch.float32), False)


class SparsePoolFunction(torch.autograd.Function):
    """y [B, G] = out_act(pool(act(sparse_projection(x)))) (autograd.py:380-414)."""

    @staticmethod
    def forward(ctx, x, w, b, rt: Level1Runtime, policy: str, compute_dtype):
        xc, wc, bc = _compute_operands(x, w, b)
        out = rt.forward(xc, wc, bc, track_ids=(policy == "save_winners"))
        pre = out["pre"]
        y = act_torch(pre, rt.level.out_activation)
        ctx.rt, ctx.policy = rt, policy
        # softmax-weighted keeps its log2-normaliser under minimal_stats (autograd.py:364-377)
        keep = ("wabsmax", "winner", "L2") if policy != "recompute_stats" else ("wabsmax",)
        ctx.extra = [k for k in keep if k in out and (k != "L2" or rt.pool == _native.POOL_SOFTMAX)]
        ctx.save_for_backward(x, w, b, pre, *[out[k] for k in ctx.extra])
        rt.last_info["checkpoint_bytes"] = sum(t.numel() * t.element_size() for t in [pre] + [out[k] for k in ctx.extra
                                                                                           if k in ("winner", "L2")])
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, b, pre, *rest = ctx.saved_tensors
        rt: Level1Runtime = ctx.rt
        xc, wc, bc = _compute_operands(x, w, b)
        g_pre = (dy.float() * dact_torch(pre, rt.level.out_activation)).contiguous()
        dw_buf, db_buf, use_main = _grad_buffers(w, b)
        saved = {"pre": pre}
        saved.update(zip(ctx.extra, rest))
        dx = rt.backward(xc, wc, bc, g_pre, saved, ctx.policy, dw_buf, db_buf)
        gw = None if use_main else dw_buf.to(w.dtype)
        gb = None if use_main else db_buf.to(b.dtype)
        return dx.to(x.dtype, memory_format=torch.contiguous_format), gw, gb, None, None, None
