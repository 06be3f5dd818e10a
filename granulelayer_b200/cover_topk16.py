"""Cover-TopK/16 opt-in layer (mirror of sparse_pooling/cover_topk16.py).

A frozen 16-input support per 16-neuron row group is selected once from a K64
envelope (``local_supports.build_cover_topk``) and the layer then runs compactly
at K = 16, C = 16: 16 neurons share each 16-index record (their row group's
inputs), each with its own 16 weights and bias, pooled by Mean(ReLU) into the
envelope's outputs with the ORIGINAL per-output valid-neuron counts
(cover_topk16.py:1-36).

Construction (``from_envelope`` / ``from_checkpoint``) and persistence
(``save_packed`` / ``load_packed``) follow cover_topk16.py:80-233 and are
bit-exact with the reference (indices, weights, bias, buckets, env map and the
support fingerprint; pinned by tests).  Execution differs by design: the
reference runs BF16 tensor-core kgen kernels (RTX 3090); here the K16/C16
forward and backward are fp32 sm_100a kernels (``csrc/k16.cu``) called through
the C ABI, with the BF16 envelope values held as fp32 parameters.
"""
from __future__ import annotations

import hashlib
import json
import time
from pathlib import Path
from typing import Optional

import torch
from torch import nn

from . import _native
from .config import PhysicalPlan
from .kgen import Envelope, KLayout, Lowered, lower_env
from .local_supports import RNG_SCHEMA, SCHEMA as LS_SCHEMA, build_cover_topk, normalize_energy
from .supergroups import ConnectivityPlan, GraphSpec

POLICY = "Cover-TopK"
FAN_IN = 16
SCHEMA = "granule.cover_topk16/1"
PACKED_SCHEMA = "granule.cover_topk16_packed/1"
CKPT_SCHEMA = "granule.k64_checkpoint/1"
NORMALIZATIONS = ("none", "energy")


def tensor_sha256(t: torch.Tensor) -> str:
    h = hashlib.sha256()
    v = t.detach().contiguous().view(-1)
    for i in range(0, v.numel(), 1 << 28):
        h.update(v[i:i + (1 << 28)].cpu().numpy().tobytes())
    return h.hexdigest()


def _fp_tensor(t: torch.Tensor):
    """(sha256 of the raw bytes, shape, dtype) (kgen_lowered.py:36-43)."""
    c = t.detach().contiguous()
    h = hashlib.sha256()
    v = c.view(-1).view(torch.uint8) if c.numel() else c.view(-1)
    for i in range(0, v.numel(), 1 << 28):
        h.update(v[i:i + (1 << 28)].cpu().numpy().tobytes())
    return h.hexdigest(), list(c.shape), str(c.dtype)


def _operand(x, w):
    """x in the layer's compute dtype (a bf16 layer computes on x rounded to bf16, as the reference's
    kgen path does), as the fp32 rows the kernels read."""
    return x.to(torch.bfloat16).to(torch.float32) if w.dtype == torch.bfloat16 else x.to(torch.float32)


class _K16Function(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, layer: "CoverTopK16Layer"):
        xc = _operand(x, w)
        if xc.stride(-1) != 1:
            xc = xc.contiguous()
        B = xc.shape[0]
        pre = torch.zeros((B, layer.layout.groups), device=x.device, dtype=torch.float32)
        if layer.tcgen05:
            name = _native.k16_fwd_t5(xc, layer._work(), w, b, layer.counts, pre, layer.layout.blocks_per_group)
        else:
            name = _native.k16_fwd(xc, layer._work(), w, b, layer.counts, pre, layer.layout.blocks_per_group,
                                   tensor_cores=layer.tensor_cores)
        ctx.layer = layer
        ctx.save_for_backward(x, w, b)
        layer.last_info.update(forward_backend="b200-k16", checkpoint_bytes=0, forward_kernel=name)
        return pre

    @staticmethod
    def backward(ctx, dy):
        layer: CoverTopK16Layer = ctx.layer
        x, w, b = ctx.saved_tensors
        xc = _operand(x, w).contiguous()
        c1t = (dy.float() / layer.counts_f[None, :]).t().contiguous()     # Mean: dL/dpre / n_g, [G, B]
        mg_w, mg_b = getattr(w, "main_grad", None), getattr(b, "main_grad", None)
        use_main = mg_w is not None and mg_b is not None
        dw = mg_w if use_main else torch.zeros(w.shape, device=w.device, dtype=torch.float32)
        db = mg_b if use_main else torch.zeros(b.shape, device=b.device, dtype=torch.float32)
        dx = torch.zeros_like(xc)
        if layer.tcgen05_bwd:
            name = _native.k16_bwd_t5(xc, layer._work(), w, b, layer.counts, c1t, dx, dw, db,
                                      layer.layout.blocks_per_group)
            layer.last_info["dx_accumulation"] = "fp32 in tensor memory"
            layer.last_info.update(backward_backend="b200-k16", backward_kernel=name)
            gw = None if use_main else dw.to(w.dtype)
            gb = None if use_main else db.to(b.dtype)
            return dx.to(x.dtype), gw, gb, None
        wabsmax = rowmax = None
        tc = layer.tensor_cores
        if tc and layer.plan.b200_dx_accum in ("auto", "fixed"):
            wabsmax = w.reshape(w.shape[0], -1).abs().amax(1).float().contiguous()
            rowmax = layer._bucket_rowmax()
        name = _native.k16_bwd(xc, layer._work(), w, b, layer.counts, c1t, dx, dw, db,
                               layer.layout.blocks_per_group, wabsmax=wabsmax, rowmax=rowmax, tensor_cores=tc)
        layer.last_info["dx_accumulation"] = "int32 fixed point" if wabsmax is not None else "fp32"
        layer.last_info.update(backward_backend="b200-k16", backward_kernel=name)
        gw = None if use_main else dw.to(w.dtype)
        gb = None if use_main else db.to(b.dtype)
        return dx.to(x.dtype), gw, gb, None


class CoverTopK16Layer(nn.Module):
    """The Cover-TopK/16 layer (module docstring).  Build with ``from_envelope`` / ``from_checkpoint``,
    restore with ``load_packed``; ``forward`` maps [..., D] to [..., G]."""

    graph_family = "cover-topk16"

    def __init__(self, low: Lowered, sg_feat: torch.Tensor, connectivity: ConnectivityPlan,
                 plan: Optional[PhysicalPlan] = None, dtype=torch.float32):
        super().__init__()
        L = low.layout
        self.layout = L
        self.connectivity = connectivity
        self.plan = plan or PhysicalPlan(grad_precision="split")
        self.spec = low.spec
        dev = low.indices.device
        self.register_buffer("indices", low.indices.contiguous())
        self.register_buffer("sg_feat", sg_feat.to(dev).contiguous())
        self.register_buffer("kg_buckets", low.kg_buckets.contiguous())
        self.register_buffer("kg_spec", torch.frombuffer(bytearray(low.spec.to_json().encode()),
                                                         dtype=torch.uint8).clone())
        self.register_buffer("env", low.env.contiguous())
        self.weight = nn.Parameter(low.weight.to(dtype).contiguous())
        self.bias = nn.Parameter(low.bias.to(dtype).contiguous())
        counts = KLayout(L.input_dim, L.hidden_dim, L.groups, 64, 16).counts_tensor(dev)
        self.register_buffer("counts", counts.contiguous(), persistent=False)
        self.register_buffer("counts_f", counts.to(torch.float32), persistent=False)
        self.envelope_KC = (64, 16)
        self.graph_stats = dict(records_16=low.records_16)
        self.cover_meta: dict = {}
        self.last_info: dict = {}
        self._work_cache = None

    # ------------------------------------------------------------------ construction
    @classmethod
    @torch.no_grad()
    def from_envelope(cls, weight: torch.Tensor, bias: torch.Tensor, *, input_dim: int, hidden_dim: int,
                      output_dim: int, connectivity: ConnectivityPlan, envelope_C: int = 256,
                      normalization: str = "none", plan: Optional[PhysicalPlan] = None, device=None,
                      dx_variant: str = "auto", envelope: Optional[Envelope] = None,
                      dtype=torch.float32) -> "CoverTopK16Layer":
        """Select the Cover-TopK/16 support from BF16 K64 envelope values ``weight [G, NB, C, 64]`` /
        ``bias [G, NB, C]`` (KLayout order) and lower it (cover_topk16.py:80-146).  ``dtype`` is the
        parameters' storage: float32 (fp32 kernels) or bfloat16 (the reference's storage and arithmetic,
        on the tensor cores)."""
        if normalization not in NORMALIZATIONS:
            raise ValueError(f"normalization {normalization!r} (one of {NORMALIZATIONS})")
        if connectivity.input_supergroup_dim != 64:
            raise ValueError(f"Cover-TopK/16 selects from S = 64 candidate sets (connectivity S = "
                             f"{connectivity.input_supergroup_dim})")
        t0 = time.perf_counter()
        env = envelope or Envelope.generate(input_dim, hidden_dim, output_dim, envelope_C, connectivity, weight, bias,
                                            device=device or weight.device)
        if env.graph_stats.get("normalized"):
            raise ValueError("this envelope was already energy-normalized: refusing to apply a second normalization")
        L = env.layout
        dev = env.weight.device
        gen_s = time.perf_counter() - t0
        t0 = time.perf_counter()
        sup = build_cover_topk(FAN_IN, L, env.kg_buckets, env.weight, Q=int(env.sg_feat.shape[0]), device=dev,
                               graph_seed=connectivity.seed)
        em = sup.element_mask(L)
        sel_s = time.perf_counter() - t0
        t0 = time.perf_counter()
        if normalization == "energy":
            w_new, b_new, nrec = normalize_energy(env.weight, env.bias, em, L.valid_mask(dev))
        else:
            w_new, b_new = env.weight * em.to(env.weight.dtype), env.bias.clone()
            nrec = dict(treatment="none", applied=False)
        menv = Envelope(L, w_new, b_new, env.sg_feat, env.kg_buckets, env.spec, connectivity, mask=em,
                        graph_stats=dict(env.graph_stats, normalized=normalization == "energy"))
        low = lower_env(menv, sup.env, source=f"local-support-{POLICY}-of-K64")
        lay = cls(low, env.sg_feat, connectivity, plan, dtype=dtype)
        lay.graph_stats.update(lowered_from_policy=POLICY, local_support=sup.fingerprint(), tile_width=FAN_IN)
        lay.dx_variant = dx_variant
        lay.cover_meta = dict(
            schema=SCHEMA, policy=POLICY, policy_version=LS_SCHEMA, rng_schema=RNG_SCHEMA, fan_in=FAN_IN,
            envelope=dict(K=64, C=L.block, S=connectivity.input_supergroup_dim, R=connectivity.partition_rounds,
                          Q=int(env.sg_feat.shape[0]), generation=connectivity.generation, seed=connectivity.seed,
                          spec=json.loads(env.spec.to_json())),
            executed=dict(K=FAN_IN, C=16, records_16=low.records_16),
            input_dim=input_dim, hidden_dim=hidden_dim, output_dim=output_dim,
            valid_slots=int(sup.enabled_slots()), biases=hidden_dim, support_fingerprint=sup.fingerprint(),
            support_stats={k: v for k, v in sup.stats.items() if k != "selection"},
            normalization=nrec, normalization_scale_bias=False,
            construction_seconds=dict(envelope_graph=gen_s, selection=sel_s, normalization_and_lowering=
                                      time.perf_counter() - t0))
        if lay.cover_meta["valid_slots"] != FAN_IN * hidden_dim:
            raise AssertionError("valid slots != 16 H")
        return lay

    @classmethod
    def from_checkpoint(cls, path, *, normalization: str = "none", plan: Optional[PhysicalPlan] = None,
                        device=None, dx_variant: str = "auto", input_dim: int = 1024, output_dim: int = 1024,
                        verify: bool = True) -> "CoverTopK16Layer":
        """``from_envelope`` on a K64 envelope checkpoint {rec, weight, bias, mask_bits} (cover_topk16.py:148-193)."""
        blob = torch.load(Path(path), map_location="cpu", weights_only=False)
        rec = blob["rec"]
        if rec.get("schema") != CKPT_SCHEMA:
            raise ValueError(f"{path}: schema {rec.get('schema')!r}, expected {CKPT_SCHEMA!r}")
        w, b = blob["weight"], blob["bias"]
        if blob.get("mask_bits") is not None:
            bits = blob["mask_bits"]
            m = ((bits[:, None] >> torch.arange(8, dtype=torch.uint8)) & 1).reshape(-1)[:w.numel()].view(w.shape)
            valid = KLayout(input_dim, int(rec["H"]), output_dim, 64, int(rec["C"])).valid_mask("cpu")
            if not bool(((m != 0) | ~valid[..., None]).all()):
                raise ValueError(f"{path}: the checkpoint's mask disables valid slots; Cover-TopK/16 selects from "
                                 "the unpruned envelope values")
        if verify and (tensor_sha256(w.view(torch.int16)) != rec["weight_sha256"] or
                       tensor_sha256(b.view(torch.int16)) != rec["bias_sha256"]):
            raise ValueError(f"{path}: weight / bias sha256 differ from the checkpoint record")
        sp = rec["spec"]
        if sp["K"] != 64:
            raise ValueError(f"{path}: envelope K = {sp['K']} (expected 64)")
        conn = ConnectivityPlan(sp["S"], sp["R"], sp.get("generation", "balanced_permutation"), sp["seed"])
        dev = torch.device(device or "cuda")
        env = Envelope.generate(input_dim, int(rec["H"]), output_dim, int(rec["C"]), conn, w.to(dev), b.to(dev),
                                device=dev)
        if json.loads(env.spec.to_json()) != sp:
            raise ValueError(f"{path}: checkpoint graph spec {sp} != regenerated {env.spec}")
        lay = cls.from_envelope(env.weight, env.bias, input_dim=input_dim, hidden_dim=int(rec["H"]),
                                output_dim=output_dim, connectivity=conn, envelope_C=int(rec["C"]),
                                normalization=normalization, plan=plan, device=dev, dx_variant=dx_variant,
                                envelope=env)
        lay.cover_meta["source_checkpoint"] = dict(weight_sha256=rec["weight_sha256"], bias_sha256=rec["bias_sha256"],
                                                   tag=(rec.get("meta") or {}).get("tag"), verified=verify)
        return lay

    # ------------------------------------------------------------------ persistence
    def immutable_fingerprints(self):
        return dict(indices=list(_fp_tensor(self.indices)), env=list(_fp_tensor(self.env)),
                    buckets=list(_fp_tensor(self.kg_buckets)), feat=list(_fp_tensor(self.sg_feat)))

    def save_packed(self, path) -> dict:
        """Frozen packed layer: compact indices / values / bias, env map, sets, buckets, spec, metadata and
        immutable-buffer fingerprints (cover_topk16.py:196-209)."""
        L = self.layout
        blob = dict(schema=PACKED_SCHEMA, meta=self.cover_meta,
                    layout=dict(input_dim=L.input_dim, hidden_dim=L.hidden_dim, output_dim=L.groups, fan_in=L.fan_in,
                                C=L.block),
                    connectivity=json.loads(self.connectivity.to_json()), spec=self.spec.to_json(),
                    envelope_KC=list(self.envelope_KC), fingerprints=self.immutable_fingerprints(),
                    state={k: v.detach().cpu() for k, v in self.state_dict().items()})
        Path(path).parent.mkdir(parents=True, exist_ok=True)
        torch.save(blob, path)
        return dict(path=str(path), fingerprints=blob["fingerprints"])

    @classmethod
    def load_packed(cls, path, *, device=None, plan: Optional[PhysicalPlan] = None,
                    dx_variant: str = "auto") -> "CoverTopK16Layer":
        """Restore a ``save_packed`` file (cover_topk16.py:211-233)."""
        blob = torch.load(Path(path), map_location="cpu", weights_only=True)
        if blob.get("schema") != PACKED_SCHEMA:
            raise ValueError(f"{path}: schema {blob.get('schema')!r}, expected {PACKED_SCHEMA!r}")
        lo, st = blob["layout"], blob["state"]
        spec = GraphSpec.from_json(blob["spec"])
        dev = torch.device(device or "cuda")
        L = KLayout(lo["input_dim"], lo["hidden_dim"], lo["output_dim"], lo["fan_in"], lo["C"])
        low = Lowered(L, st["indices"].to(dev), st["weight"].to(dev), st["bias"].to(dev), st["kg_buckets"].to(dev),
                      st["env"].to(dev), spec, int(blob["meta"].get("executed", {}).get("records_16", 0)))
        lay = cls(low, st["sg_feat"], ConnectivityPlan(**blob["connectivity"]), plan, dtype=st["weight"].dtype)
        lay.load_state_dict(st)
        lay.envelope_KC = tuple(blob["envelope_KC"])
        lay.cover_meta = blob["meta"]
        lay.dx_variant = dx_variant
        if lay.immutable_fingerprints() != blob["fingerprints"]:
            raise ValueError(f"{path}: immutable buffers differ from their recorded fingerprints")
        return lay

    # ------------------------------------------------------------------ execution
    def _work(self) -> dict:
        """The kernels' schedule (cached per device): the bucket list sorted by input set (stable, so runs
        of one set keep their order), ``q_off [Q+1]`` the bucket range of each set, ``rec_off [nb+1]`` the
        exclusive prefix sum of the buckets' record counts, with ``env`` and ``sg_feat``.  It plays the role
        of the reference's per-chunk item lists (experimental/kgen_graph.py:166-217)."""
        key = (self.kg_buckets.device, self.kg_buckets.data_ptr(), self.env.data_ptr(), self.sg_feat.data_ptr())
        if self._work_cache is None or self._work_cache[0] != key:
            b = self.kg_buckets.to(torch.int64)
            order = torch.sort(b[:, 0], stable=True).indices
            b = b[order]
            Q = int(self.sg_feat.shape[0])
            q_off = torch.searchsorted(b[:, 0].contiguous(), torch.arange(Q + 1, device=b.device))
            rec_off = torch.zeros(len(b) + 1, dtype=torch.int64, device=b.device)
            rec_off[1:] = torch.cumsum(b[:, 3], 0)
            if int(rec_off[-1]) >= 2 ** 31:
                raise ValueError("more than 2^31 records in the bucket list")
            sched = dict(buckets=b.to(torch.int32).contiguous(), q_off=q_off.to(torch.int32).contiguous(),
                         rec_off=rec_off.to(torch.int32).contiguous(), env=self.env.contiguous(),
                         feat=self.sg_feat.to(torch.int16).contiguous())
            self._work_cache = (key, sched)
        return self._work_cache[1]

    def _bucket_rowmax(self) -> torch.Tensor:
        """[nb] int32, per row of the schedule's bucket list: the largest number of the bucket's record
        inputs on one local position (the bound of the tensor-core backward's fixed-point dX tile).
        Depends only on the graph; cached with the schedule."""
        sched = self._work()
        if "rowmax" not in sched:
            bk = sched["buckets"].to(torch.int64)
            S, NB16 = int(self.sg_feat.shape[1]), self.layout.blocks_per_group
            nrec = bk[:, 3].clamp(min=0)
            bid = torch.repeat_interleave(torch.arange(bk.shape[0], device=bk.device), nrec)
            within = torch.arange(int(nrec.sum()), device=bk.device) - torch.repeat_interleave(
                torch.cumsum(nrec, 0) - nrec, nrec)
            f = (bk[:, 1] * NB16 + bk[:, 2])[bid] + within
            pos = self.env.reshape(-1, 16)[f].long().clamp(max=S - 1)
            cnt = torch.bincount((bid[:, None] * S + pos).reshape(-1), minlength=bk.shape[0] * S)
            sched["rowmax"] = cnt.reshape(-1, S).amax(1).to(torch.int32).contiguous()
        return sched["rowmax"]

    @property
    def tensor_cores(self) -> bool:
        """Whether the layer runs the tensor-core kernels: always for bf16 parameters; for fp32 ones, the
        three-term bf16 split kernels unless ``plan.b200_f32_tensor_cores == "off"``."""
        return self.weight.dtype == torch.bfloat16 or self.plan.b200_f32_tensor_cores == "auto"

    @property
    def tcgen05(self) -> bool:
        """Whether the forward runs on the tcgen05 tensor cores (gl_k16_fwd_t5 / gl_k16_fwd_t5_f32): tensor-core
        layers whose input sets have S = 64 positions, when ``plan.b200_tcgen05`` is "on" or "fwd" (off by
        default: the mma.sync forward is faster at config 4)."""
        return self.tensor_cores and self.plan.b200_tcgen05 in ("on", "fwd") and int(self.sg_feat.shape[1]) == 64

    @property
    def tcgen05_bwd(self) -> bool:
        """Whether the backward runs on the tcgen05 tensor cores (gl_k16_bwd_t5 / gl_k16_bwd_t5_f32): as
        ``tcgen05``, for ``plan.b200_tcgen05`` "on" or "bwd"."""
        return self.tensor_cores and self.plan.b200_tcgen05 in ("on", "bwd") and int(self.sg_feat.shape[1]) == 64

    def enable_main_grad(self):
        for p in (self.weight, self.bias):
            if getattr(p, "main_grad", None) is None:
                p.main_grad = torch.zeros(p.shape, device=p.device, dtype=torch.float32)

    def zero_main_grad(self):
        for p in (self.weight, self.bias):
            if getattr(p, "main_grad", None) is not None:
                p.main_grad.zero_()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.weight.dtype not in (torch.float32, torch.bfloat16):
            raise NotImplementedError("the B200 K16 kernels run fp32 or bf16 parameters")
        lead = x.shape[:-1]
        y = _K16Function.apply(x.reshape(-1, x.shape[-1]), self.weight, self.bias, self)
        return y.reshape(*lead, y.shape[-1])

    @property
    def metadata(self) -> dict:
        return self.cover_meta

    @property
    def normalization(self) -> dict:
        return self.cover_meta["normalization"]

    def extra_repr(self):
        m = self.cover_meta
        e = m.get("envelope", {})
        return (f"Cover-TopK/16: in={m.get('input_dim')}, hidden={m.get('hidden_dim', 0):,}, "
                f"out={m.get('output_dim')}, envelope K{e.get('K')}/C{e.get('C')} S{e.get('S')}/R{e.get('R')}, "
                f"executed K16/C16, normalization={m.get('normalization', {}).get('treatment')}")
