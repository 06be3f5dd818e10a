"""Generate the golden fixtures of tests/golden/ from the reference implementation.

Run in a checkout where the reference package ``sparse_pooling`` is importable:

    python tests/golden/make_golden.py --reference <dir containing sparse_pooling/>

What it writes (all from the reference's own code on the CPU):

* ``init_hashes.json`` — sha256 of the (indices, weights, bias) bytes produced by
  ``sparse_pooling.layout.init_parameters`` (layout.py:204-251) for a set of
  layouts, seeds and chunk sizes, plus the layout shapes.  The product's
  ``init_parameters`` must reproduce every hash bit for bit.
* ``fwdbwd_<case>.npz`` — Mode-A layers rebuilt from the same seeds (their hash
  is stored alongside), an input ``x`` and upstream gradient ``dy``, and the
  reference's ``reference_forward`` output ``y`` with its autograd gradients
  ``dx``, ``dw``, ``db``, computed in float64 (pytorch_reference.py:29-105) and
  stored as float32 (dw/db for the first 32 groups).  The "sum" cases use the reference's
  ``hidden_preactivations`` + activation + masked sum (the reference has no
  sum operator).  One case draws indices uniformly with replacement
  (duplicate indices inside a neuron).
* ``fwdbwd_modeb_<case>.npz`` — Mode-B layers (shared index records, canonical and
  fragment-packed storage) rebuilt from seeds, with the reference's float64
  ``reference_forward`` output and autograd gradients (dw/db in the layer's own
  storage layout, first groups only).
* ``fwdbwd_max_<case>.npz`` — max pooling (Mode A and Mode B) with the reference's
  ``reference_forward`` (winner = smallest slot attaining the max) and autograd gradients,
  plus the winner slots.
* ``fwdbwd_smooth_<case>.npz`` — LogMeanExp, power-mean and softmax-weighted pooling (Mode A
  and Mode B) with the reference's float64 ``reference_forward`` and autograd gradients.
* ``fwdbwd_topk_<case>.npz`` — top-K mean pooling (Mode A and Mode B) with the reference's float64
  ``reference_forward``, its selected slots and autograd gradients.
* ``fwdbwd_semantic_<case>.npz`` — two-level (semantic) pooling: level-1 shards, transform and
  level-2 operator, with the reference's float64 ``reference_forward`` and autograd gradients,
  including the transform / weighted-sum parameters' gradients.
* ``graph_hashes.json`` — sha256 of the reference's input-supergroup graphs: Mode-B
  ``supergroups.generate_indices`` (indices, feature sets, buckets) and the generalized
  ``experimental/kgen_graph.generate`` (K = 64 / C = 256 envelope, K = 16 / C = 16).
* ``kc_reference.npz`` — a small Cover-TopK/16 layer built by the reference
  (``CoverTopK16Layer.from_envelope``, cover_topk16.py:80-146) with its lowered storage and
  schedule buffers, an input, an upstream gradient, and the reference's float64 K/C model
  ``experimental/reference.grads`` (reference.py:21-27) evaluated on it: y, dx, dw, db.
* ``adam.npz`` — five steps of ``torch.optim.AdamW``/``Adam`` in float64, the
  recurrence the reference's optimizer test compares its fused kernel with
  (tests/test_optim.py:11-28; optim.py:39-42).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
GSUB = 32  # dw/db are stored for the first GSUB groups only (keeps the fixtures small)

# (name, D, H, G, B, seed, bias_std, pooling, activation, index rule)
CASES = [
    ("cfg1_mean_relu", 256, 65536, 256, 64, 0, 0.0, "mean", "relu", "distinct"),
    ("cfg1_sum_relu", 256, 65536, 256, 64, 0, 0.0, "sum", "relu", "distinct"),
    ("ragged_b37", 64, 4099, 16, 37, 1, 0.3, "mean", "relu", "distinct"),
    ("batch1", 64, 3000, 8, 1, 2, 0.2, "mean", "relu", "distinct"),
    ("projection_identity", 128, 64, 64, 37, 3, 0.2, "mean", "identity", "distinct"),
    ("gelu_mean", 64, 3000, 8, 16, 4, 0.2, "mean", "gelu", "distinct"),
    ("sum_identity_ragged", 96, 1001, 7, 5, 5, 0.1, "sum", "identity", "distinct"),
    ("uniform_dup_idx", 32, 2048, 8, 24, 6, 0.1, "mean", "relu", "uniform"),
]

# Mode B (C neurons share one index record): (name, D, H, G, C, packed, B, seed, bias_std, pooling, activation)
MODEB_CASES = [
    ("modeb_c8", 256, 65536, 256, 8, False, 64, 5, 0.1, "mean", "relu"),
    ("modeb_c64_packed_ragged", 512, 20000, 7, 64, True, 37, 6, 0.2, "mean", "relu"),
    ("modeb_c16_gelu", 300, 5000, 3, 16, False, 19, 7, 0.2, "mean", "gelu"),
    ("modeb_c32_packed_sum", 1024, 12288, 4, 32, True, 9, 8, 0.1, "sum", "relu"),
    ("modeb_c8_packed_identity", 128, 3001, 5, 8, True, 1, 9, 0.3, "mean", "identity"),
]

# Max pooling: (name, D, H, G, C (None = Mode A), packed, B, seed, bias_std, activation)
MAX_CASES = [
    ("max_modea_relu", 128, 6000, 12, None, False, 23, 11, 0.2, "relu"),
    ("max_modea_identity_ragged", 96, 1001, 7, None, False, 9, 12, 0.1, "identity"),
    ("max_modeb_c8_packed_gelu", 256, 7000, 5, 8, True, 17, 13, 0.2, "gelu"),
]

# Smooth pools: (name, D, H, G, C (None = Mode A), packed, B, seed, bias_std, type, parameters, activation)
SMOOTH_CASES = [
    ("lme_modea_t05", 128, 6000, 12, None, False, 23, 21, 0.2, "logmeanexp", {"temperature": 0.5}, "identity"),
    ("lme_modeb_c8_packed_t2", 256, 7000, 5, 8, True, 17, 22, 0.2, "logmeanexp", {"temperature": 2.0}, "relu"),
    ("power_modea_p2", 96, 1001, 7, None, False, 9, 23, 0.1, "power_mean", {"p": 2.0}, "relu"),
    ("power_modea_p3", 128, 4000, 6, None, False, 13, 24, 0.2, "power_mean", {"p": 3.0}, "relu"),
    ("power_modeb_c64_p4", 512, 20000, 3, 64, False, 11, 25, 0.2, "power_mean", {"p": 4.0}, "relu"),
    ("softmax_modea_b15", 128, 6000, 12, None, False, 23, 26, 0.2, "softmax_weighted", {"beta": 1.5}, "identity"),
    ("softmax_modeb_c16_gelu", 300, 5000, 3, 16, False, 19, 27, 0.2, "softmax_weighted", {"beta": 0.7}, "gelu"),
]

# Top-K mean: (name, D, H, G, C (None = Mode A), packed, B, seed, bias_std, k, activation)
TOPK_CASES = [
    ("modea_k8", 128, 6000, 12, None, False, 23, 41, 0.2, 8, "identity"),
    ("modea_k64_gelu", 96, 1001, 7, None, False, 9, 42, 0.1, 64, "gelu"),
    ("modea_k1_ragged", 64, 1003, 9, None, False, 5, 45, 0.3, 1, "relu"),
    ("modea_k16_small_groups", 64, 100, 9, None, False, 7, 46, 0.2, 16, "identity"),
    ("modeb_c8_packed_k4", 256, 7000, 5, 8, True, 17, 43, 0.2, 4, "relu"),
    ("modeb_c64_k32", 512, 20000, 3, 64, False, 11, 44, 0.2, 32, "identity"),
]

# Two-level pooling: (name, D, H, G, C (None = Mode A), packed, B, seed, bias_std, level 1, level 2,
# level1_checkpoint)
SEMANTIC_CASES = [
    ("modea_mean_max", 128, 6000, 12, None, False, 23, 31, 0.2,
     {"type": "mean", "neurons_per_shard": 128}, {"type": "max"}, "save"),
    ("modea_max_affine_wsum", 128, 6000, 12, None, False, 19, 32, 0.2,
     {"type": "max", "neurons_per_shard": 64, "transform": "affine"}, {"type": "weighted_sum"}, "save"),
    ("modeb_c8_lme_gate_softmax", 256, 6400, 5, 8, True, 17, 33, 0.2,
     {"type": "logmeanexp", "neurons_per_shard": 256, "transform": "gate", "temperature": 0.5},
     {"type": "softmax_weighted", "beta": 2.0}, "recompute"),
    ("modeb_c64_mean_act_topk", 512, 12288, 3, 64, False, 11, 34, 0.2,
     {"type": "mean", "neurons_per_shard": 512, "transform": "activation"}, {"type": "topk_mean", "k": 2}, "save"),
]

# (D, H, G, C, S, R, generation, seed): Mode-B input-supergroup graphs
GRAPH_CASES = [
    (256, 40000, 16, 8, 64, 2, "balanced_permutation", 0),
    (256, 40000, 16, 64, 32, 3, "balanced_permutation", 7),
    (128, 7777, 5, 16, 16, 1, "independent_subsets", 3),
    (512, 100000, 64, 32, 128, 4, "balanced_permutation", 11),
]
# (D, H, G, C, K, S, R, seed): generalized graphs (quantum 1), incl. the K64/C256 Cover-TopK16 envelope
KGEN_CASES = [
    (256, 3452, 8, 256, 64, 64, 16, 0),
    (1024, 65536, 64, 256, 64, 64, 8, 5),
    (256, 20000, 16, 16, 16, 64, 4, 2),
]

INIT_CASES = [
    # (D, H, G, C, shared, packed, seed, bias_std, chunk_records)
    (256, 65536, 256, 8, False, False, 0, 0.0, 1 << 22),
    (256, 65536, 256, 8, False, False, 7, 0.25, 1000),
    (64, 4099, 16, 8, False, False, 1, 0.3, 1 << 22),
    (64, 3001, 8, 16, True, False, 1, 0.5, 1 << 22),
    (64, 7000, 8, 32, True, True, 2, 0.1, 999),
    (1024, 30011, 16, 64, True, True, 3, 0.3, 1 << 22),
    (4096, 98304, 4, 8, False, False, 1, 0.1, 1 << 14),
]


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().cpu().numpy().tobytes()).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory that contains the sparse_pooling package")
    ap.add_argument("--only", choices=["smooth", "semantic", "topk"], help="write only this group of fixtures")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from sparse_pooling.config import LevelSpec, PoolingConfig
    from sparse_pooling.layout import SparseLayout, init_parameters
    from sparse_pooling.reference import pytorch_reference as ref

    torch.set_num_threads(8)
    if args.only == "smooth":
        smooth_fixtures(ref, LevelSpec, PoolingConfig, SparseLayout, init_parameters)
        return
    if args.only == "semantic":
        semantic_fixtures(ref, LevelSpec, PoolingConfig, SparseLayout, init_parameters)
        return
    if args.only == "topk":
        topk_fixtures(ref, LevelSpec, PoolingConfig, SparseLayout, init_parameters)
        return
    hashes = []
    for D, H, G, C, shared, packed, seed, bstd, chunk in INIT_CASES:
        L = SparseLayout(D, H, G, 8, C, shared, packed=packed)
        i, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=seed, bias_std=bstd, chunk_records=chunk)
        hashes.append(dict(layout=[D, H, G, 8, C, shared, packed], seed=seed, bias_std=bstd, chunk_records=chunk,
                           dtype="float32", index_shape=list(L.index_shape), weight_shape=list(L.weight_shape),
                           bias_shape=list(L.bias_shape), idx=sha(i), w=sha(w), b=sha(b)))
        # bf16 storage (the reference's default dtype) draws the same indices
        ib, wb, bb = init_parameters(L, "cpu", dtype=torch.bfloat16, seed=seed, bias_std=bstd, chunk_records=chunk)
        hashes.append(dict(hashes[-1], dtype="bfloat16", idx=sha(ib), w=sha(wb.view(torch.int16)),
                           b=sha(bb.view(torch.int16))))
    (HERE / "init_hashes.json").write_text(json.dumps(hashes, indent=1))

    for name, D, H, G, B, seed, bstd, pool, act, rule in CASES:
        L = SparseLayout(D, H, G, 8, 8, False)
        idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=seed, bias_std=bstd)
        gen = torch.Generator().manual_seed(1000 + seed)
        if rule == "uniform":
            idx = torch.randint(0, D, idx.shape, generator=gen, dtype=torch.int64).to(torch.int16)
            idx.view(G, -1, 8)[~L.valid_mask("cpu")] = 0
        x = torch.randn(B, D, generator=gen)
        xd = x.double().requires_grad_(True)
        wd = w.double().requires_grad_(True)
        bd = b.double().requires_grad_(True)
        if pool == "mean":
            cfg = PoolingConfig([LevelSpec("mean", activation=act)])
            y = ref.reference_forward(xd, idx, wd, bd, L, cfg)
        else:
            z = ref.hidden_preactivations(xd, idx, wd, bd, L)
            a = ref.activation(z, act)
            y = torch.where(L.valid_mask("cpu")[None], a, torch.zeros_like(a)).sum(-1)
        dy = torch.randn(y.shape, generator=gen)
        (y * dy.double()).sum().backward()
        # reference in float32 too: its deviation from the float64 values is recorded
        x32 = x.clone().requires_grad_(True)
        if pool == "mean":
            y32 = ref.reference_forward(x32, idx, w, b, L, PoolingConfig([LevelSpec("mean", activation=act)]))
        else:
            z32 = ref.hidden_preactivations(x32, idx, w, b, L)
            y32 = torch.where(L.valid_mask("cpu")[None], ref.activation(z32, act), torch.zeros_like(z32)).sum(-1)
        dev32 = float((y32.detach().double() - y.detach()).abs().max() / (y.detach().abs().max() + 1e-30))
        np.savez_compressed(
            HERE / f"fwdbwd_{name}.npz",
            meta=json.dumps(dict(name=name, D=D, H=H, G=G, B=B, seed=seed, bias_std=bstd, pool=pool, act=act,
                                 rule=rule, idx_sha=sha(idx), w_sha=sha(w), b_sha=sha(b),
                                 ref_fp32_vs_fp64_max_rel=dev32)),
            idx=idx.numpy() if rule == "uniform" else np.zeros(0, np.int16),
            x=x.numpy(), dy=dy.numpy(), y=y.detach().float().numpy(), dx=xd.grad.float().numpy(),
            dw=wd.grad[:GSUB].float().numpy(), db=bd.grad[:GSUB].float().numpy())

    for name, D, H, G, C, packed, B, seed, bstd, pool, act in MODEB_CASES:
        L = SparseLayout(D, H, G, 8, C, True, packed=packed)
        idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=seed, bias_std=bstd)
        gen = torch.Generator().manual_seed(2000 + seed)
        x = torch.randn(B, D, generator=gen)
        xd = x.double().requires_grad_(True)
        wd = w.double().requires_grad_(True)
        bd = b.double().requires_grad_(True)
        if pool == "mean":
            y = ref.reference_forward(xd, idx, wd, bd, L, PoolingConfig([LevelSpec("mean", activation=act)]))
        else:
            z = ref.hidden_preactivations(xd, idx, wd, bd, L)
            y = torch.where(L.canonical.valid_mask("cpu")[None], ref.activation(z, act), torch.zeros_like(z)).sum(-1)
        dy = torch.randn(y.shape, generator=gen)
        (y * dy.double()).sum().backward()
        np.savez_compressed(
            HERE / f"fwdbwd_{name}.npz",
            meta=json.dumps(dict(name=name, D=D, H=H, G=G, C=C, packed=packed, B=B, seed=seed, bias_std=bstd,
                                 pool=pool, act=act, rule="distinct", mode="B", idx_sha=sha(idx), w_sha=sha(w),
                                 b_sha=sha(b))),
            idx=np.zeros(0, np.int16), x=x.numpy(), dy=dy.numpy(), y=y.detach().float().numpy(),
            dx=xd.grad.float().numpy(), dw=wd.grad[:GSUB].float().numpy(), db=bd.grad[:GSUB].float().numpy())

    for name, D, H, G, C, packed, B, seed, bstd, act in MAX_CASES:
        L = SparseLayout(D, H, G, 8, C or 8, C is not None, packed=packed)
        idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=seed, bias_std=bstd)
        gen = torch.Generator().manual_seed(3000 + seed)
        x = torch.randn(B, D, generator=gen)
        xd = x.double().requires_grad_(True)
        wd = w.double().requires_grad_(True)
        bd = b.double().requires_grad_(True)
        y = ref.reference_forward(xd, idx, wd, bd, L, PoolingConfig([LevelSpec("max", activation=act)]))
        z = ref.hidden_preactivations(xd.detach(), idx, wd.detach(), bd.detach(), L)
        a = ref.activation(z, act)
        a = torch.where(L.canonical.valid_mask("cpu")[None], a, torch.full_like(a, float("-inf")))
        winner = torch.argmax(a, dim=-1).to(torch.int32)
        dy = torch.randn(y.shape, generator=gen)
        (y * dy.double()).sum().backward()
        np.savez_compressed(
            HERE / f"fwdbwd_{name}.npz",
            meta=json.dumps(dict(name=name, D=D, H=H, G=G, C=C, packed=packed, B=B, seed=seed, bias_std=bstd,
                                 pool="max", act=act, rule="distinct", mode="A" if C is None else "B",
                                 idx_sha=sha(idx), w_sha=sha(w), b_sha=sha(b))),
            idx=np.zeros(0, np.int16), x=x.numpy(), dy=dy.numpy(), y=y.detach().float().numpy(),
            winner=winner.numpy(), dx=xd.grad.float().numpy(), dw=wd.grad[:GSUB].float().numpy(),
            db=bd.grad[:GSUB].float().numpy())

    smooth_fixtures(ref, LevelSpec, PoolingConfig, SparseLayout, init_parameters)
    semantic_fixtures(ref, LevelSpec, PoolingConfig, SparseLayout, init_parameters)
    topk_fixtures(ref, LevelSpec, PoolingConfig, SparseLayout, init_parameters)

    # input-supergroup graphs (supergroups.py generate_indices; kgen_graph.py generate)
    from sparse_pooling.experimental import kgen_graph as KG
    from sparse_pooling.supergroups import ConnectivityPlan, generate_indices

    graphs = []
    for D, H, G, C, S, R, gen, seed in GRAPH_CASES:
        L = SparseLayout(D, H, G, 8, C, True)
        plan = ConnectivityPlan(S, R, gen, seed)
        idx, graph, _ = generate_indices(L, plan, "cpu")
        graphs.append(dict(kind="mode_b", layout=[D, H, G, 8, C, True], plan=json.loads(plan.to_json()),
                           idx=sha(idx), feat=sha(graph.feat), buckets=sha(graph.buckets),
                           shapes=[list(idx.shape), list(graph.feat.shape), list(graph.buckets.shape)]))
    for D, H, G, C, K, S, R, seed in KGEN_CASES:
        from sparse_pooling.experimental.kgen_layout import KLayout

        KL = KLayout(D, H, G, K, C)
        plan = ConnectivityPlan(S, R, "balanced_permutation", seed)
        counts = KL.counts_tensor("cpu")
        idx, feat, ubk, _ = KG.generate(D, counts, C, K, KL.blocks_per_group, 1, plan, "cpu")
        bk = KG.unit_to_block_buckets(ubk, counts, C, 1)
        graphs.append(dict(kind="kgen", layout=[D, H, G, K, C], plan=json.loads(plan.to_json()), idx=sha(idx),
                           feat=sha(feat), buckets=sha(ubk), block_buckets=sha(bk),
                           shapes=[list(idx.shape), list(feat.shape), list(ubk.shape), list(bk.shape)]))
    (HERE / "graph_hashes.json").write_text(json.dumps(graphs, indent=1))

    from sparse_pooling.cover_topk16 import CoverTopK16Layer
    from sparse_pooling.experimental import reference as KREF
    from sparse_pooling.experimental.kgen_layout import KLayout, init_parameters as init_envelope_parameters

    D, H, G, R = 256, 3452, 8, 16
    EL = KLayout(D, H, G, 64, 256)
    w64, b64 = init_envelope_parameters(EL, "cpu", dtype=torch.bfloat16, seed=1, bias_std=0.1)
    lay = CoverTopK16Layer.from_envelope(w64, b64, input_dim=D, hidden_dim=H, output_dim=G,
                                         connectivity=ConnectivityPlan(64, R, seed=4), device="cpu")
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(37, D, generator=gen)
    gy = torch.randn(37, G, generator=gen)
    counts = KLayout(D, H, G, 16, 16).counts_tensor("cpu")
    y, dx, dw, db = KREF.grads(x.double(), lay.indices.long(), lay.weight.detach().float().double(), lay.bias.detach().float().double(),
                               counts, gy.double())
    np.savez_compressed(HERE / "kc_reference.npz", meta=json.dumps(dict(D=D, H=H, G=G, R=R, seed=1, graph_seed=4)),
                        x=x.numpy(), gy=gy.numpy(), indices=lay.indices.numpy(), weight=lay.weight.detach().float().numpy(),
                        bias=lay.bias.detach().float().numpy(), counts=counts.numpy(), sg_feat=lay.sg_feat.numpy(),
                        kg_buckets=lay.kg_buckets.numpy(), env=lay.env.numpy(), y=y.numpy(), dx=dx.numpy(),
                        dw=dw.numpy(), db=db.numpy())

    torch.manual_seed(0)
    out = {}
    for tag, wdc in (("adamw", 0.1), ("adam", 0.0)):
        p0 = torch.randn(1000, dtype=torch.float64)
        q = torch.nn.Parameter(p0.clone())
        opt = torch.optim.AdamW([q], lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=wdc)
        gs, ps, ms, vs = [], [], [], []
        for _ in range(5):
            g = torch.randn(1000, dtype=torch.float64)
            q.grad = g.clone()
            opt.step()
            gs.append(g.numpy()); ps.append(q.detach().clone().numpy())
            ms.append(opt.state[q]["exp_avg"].clone().numpy()); vs.append(opt.state[q]["exp_avg_sq"].clone().numpy())
        out.update({f"{tag}_p0": p0.numpy(), f"{tag}_g": np.stack(gs), f"{tag}_p": np.stack(ps),
                    f"{tag}_m": np.stack(ms), f"{tag}_v": np.stack(vs), f"{tag}_wd": np.array(wdc)})
    np.savez_compressed(HERE / "adam.npz", lr=np.array(1e-2), beta1=np.array(0.9), beta2=np.array(0.999),
                        eps=np.array(1e-8), **out)
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


def smooth_fixtures(ref, LevelSpec, PoolingConfig, SparseLayout, init_parameters):
    for name, D, H, G, C, packed, B, seed, bstd, kind, params, act in SMOOTH_CASES:
        L = SparseLayout(D, H, G, 8, C or 8, C is not None, packed=packed)
        idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=seed, bias_std=bstd)
        gen = torch.Generator().manual_seed(4000 + seed)
        x = torch.randn(B, D, generator=gen)
        xd = x.double().requires_grad_(True)
        wd = w.double().requires_grad_(True)
        bd = b.double().requires_grad_(True)
        y = ref.reference_forward(xd, idx, wd, bd, L, PoolingConfig([LevelSpec(kind, activation=act, **params)]))
        dy = torch.randn(y.shape, generator=gen)
        (y * dy.double()).sum().backward()
        np.savez_compressed(
            HERE / f"fwdbwd_smooth_{name}.npz",
            meta=json.dumps(dict(name=name, D=D, H=H, G=G, C=C, packed=packed, B=B, seed=seed, bias_std=bstd,
                                 pool=kind, params=params, act=act, rule="distinct", mode="A" if C is None else "B",
                                 idx_sha=sha(idx), w_sha=sha(w), b_sha=sha(b))),
            idx=np.zeros(0, np.int16), x=x.numpy(), dy=dy.numpy(), y=y.detach().float().numpy(),
            dx=xd.grad.float().numpy(), dw=wd.grad[:GSUB].float().numpy(), db=bd.grad[:GSUB].float().numpy())


def semantic_fixtures(ref, LevelSpec, PoolingConfig, SparseLayout, init_parameters):
    import math

    for name, D, H, G, C, packed, B, seed, bstd, l1, l2, ckpt in SEMANTIC_CASES:
        L = SparseLayout(D, H, G, 8, C or 8, C is not None, packed=packed)
        idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=seed, bias_std=bstd)
        cfg = PoolingConfig([LevelSpec(**l1), LevelSpec(**l2)], level1_checkpoint=ckpt)
        S = math.ceil(L.max_group / l1["neurons_per_shard"])
        gen = torch.Generator().manual_seed(5000 + seed)
        x = torch.randn(B, D, generator=gen)
        tp = {}
        if l1.get("transform") in ("affine", "gate"):
            tp["alpha"] = 1.0 + 0.3 * torch.randn(G, S, generator=gen, dtype=torch.float64)
            tp["beta"] = 0.2 * torch.randn(G, S, generator=gen, dtype=torch.float64)
        if l2["type"] == "weighted_sum":
            tp["v"] = torch.randn(G, S, generator=gen, dtype=torch.float64) / S
        xd = x.double().requires_grad_(True)
        wd = w.double().requires_grad_(True)
        bd = b.double().requires_grad_(True)
        tpd = {k: v.clone().requires_grad_(True) for k, v in tp.items()}
        y = ref.reference_forward(xd, idx, wd, bd, L, cfg, tpd)
        dy = torch.randn(y.shape, generator=gen)
        (y * dy.double()).sum().backward()
        extra = {f"t_{k}": v.float().numpy() for k, v in tp.items()}
        extra.update({f"dt_{k}": v.grad.float().numpy() for k, v in tpd.items()})
        np.savez_compressed(
            HERE / f"fwdbwd_semantic_{name}.npz",
            meta=json.dumps(dict(name=name, D=D, H=H, G=G, C=C, packed=packed, B=B, seed=seed, bias_std=bstd,
                                 levels=[l1, l2], level1_checkpoint=ckpt, mode="A" if C is None else "B",
                                 idx_sha=sha(idx), w_sha=sha(w), b_sha=sha(b))),
            x=x.numpy(), dy=dy.numpy(), y=y.detach().float().numpy(), dx=xd.grad.float().numpy(),
            dw=wd.grad[:GSUB].float().numpy(), db=bd.grad[:GSUB].float().numpy(), **extra)


def topk_fixtures(ref, LevelSpec, PoolingConfig, SparseLayout, init_parameters):
    for name, D, H, G, C, packed, B, seed, bstd, k, act in TOPK_CASES:
        L = SparseLayout(D, H, G, 8, C or 8, C is not None, packed=packed)
        idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=seed, bias_std=bstd)
        gen = torch.Generator().manual_seed(6000 + seed)
        x = torch.randn(B, D, generator=gen)
        xd = x.double().requires_grad_(True)
        wd = w.double().requires_grad_(True)
        bd = b.double().requires_grad_(True)
        extra = {}
        y = ref.reference_forward(xd, idx, wd, bd, L, PoolingConfig([LevelSpec("topk_mean", activation=act, k=k)]),
                                  extra=extra)
        dy = torch.randn(y.shape, generator=gen)
        (y * dy.double()).sum().backward()
        np.savez_compressed(
            HERE / f"fwdbwd_topk_{name}.npz",
            meta=json.dumps(dict(name=name, D=D, H=H, G=G, C=C, packed=packed, B=B, seed=seed, bias_std=bstd,
                                 pool="topk_mean", k=k, act=act, rule="distinct", mode="A" if C is None else "B",
                                 idx_sha=sha(idx), w_sha=sha(w), b_sha=sha(b))),
            x=x.numpy(), dy=dy.numpy(), y=y.detach().float().numpy(), topk=extra["topk"].to(torch.int32).numpy(),
            dx=xd.grad.float().numpy(), dw=wd.grad[:GSUB].float().numpy(), db=bd.grad[:GSUB].float().numpy())


if __name__ == "__main__":
    main()
