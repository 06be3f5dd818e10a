"""Input-supergroup connectivity (mirror of sparse_pooling/supergroups.py and the
generalized generator of sparse_pooling/experimental/kgen_graph.py).

A ``ConnectivityPlan`` (S, R, generation, seed) partitions the D inputs R times
into D/S sets of S features (``feat [Q, S]``, Q = R*D/S); every index record
draws its K distinct inputs from one set.  The generator is reproduced draw for
draw (same torch generators, seeds, call order and chunking):

1. feature sets: R seeded permutations of the D inputs, each cut into D/S rows,
   rows sorted (supergroups.py:166-177);
2. balanced assignment of each output's assignment units (``quantum`` blocks)
   to the Q sets: quotas differing by at most one, extras rotating over the
   outputs, each output's partial tail unit placed greedily on the least-loaded
   position, positions mapped to sets in round-interleaved order
   (supergroups.py:126-163, kgen_graph.py:45-67);
3. buckets (q, g, first unit, unit count) sorted by (q, g) (supergroups.py:180-197);
4. records: per set q, one stream of permutations of its S local features cut
   into S/K records (or independent K-subsets), consumed in (g, block) order and
   stored sorted as global ids; blocks beyond the valid units copy the output's
   first record (supergroups.py:200-271, kgen_graph.py:86-151).

``generate_records`` with K = 8 and the Mode-B layout's unit size is the
production ``generate_indices``; with K = 64 / quantum = 1 it is the Cover-TopK16
envelope graph.  Nothing here touches a GPU kernel.
"""
from __future__ import annotations

import dataclasses
import json
import math
import time
from dataclasses import dataclass
from typing import Dict, Optional

import torch

from .layout import SparseLayout, _distinct_sorted_records

GENERATIONS = ("balanced_permutation", "independent_subsets")
GRAPH_VERSION = 1
GENERATOR = "kgen_balanced_permutation"   # kgen_graph.py:36-37
GENERATOR_VERSION = 1


@dataclass(frozen=True)
class ConnectivityPlan:
    """Logical connectivity: ``input_supergroup_dim`` = S, ``partition_rounds`` = R (supergroups.py:58-87)."""

    input_supergroup_dim: int
    partition_rounds: int
    generation: str = "balanced_permutation"
    seed: int = 0
    version: int = GRAPH_VERSION

    def __post_init__(self):
        if self.generation not in GENERATIONS:
            raise ValueError(f"unknown generation {self.generation!r}")
        if self.input_supergroup_dim < 8 or self.input_supergroup_dim % 8:
            raise ValueError("input_supergroup_dim must be a multiple of 8 (fan-in 8)")
        if self.partition_rounds < 1:
            raise ValueError("partition_rounds must be >= 1")

    def num_supergroups(self, input_dim: int) -> int:
        if input_dim % self.input_supergroup_dim:
            raise ValueError(f"input_supergroup_dim {self.input_supergroup_dim} must divide D = {input_dim}")
        return self.partition_rounds * input_dim // self.input_supergroup_dim

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self), sort_keys=True)

    @staticmethod
    def from_json(s: str) -> "ConnectivityPlan":
        return ConnectivityPlan(**json.loads(s))


@dataclass
class SupergroupGraph:
    """feat [Q, S] int16 sorted global ids of every set; buckets [n, 4] int32 (q, g, first unit, units)."""

    plan: Optional[ConnectivityPlan]
    feat: torch.Tensor
    buckets: torch.Tensor

    @property
    def Q(self) -> int:
        return self.feat.shape[0]

    @property
    def S(self) -> int:
        return self.feat.shape[1]

    def metadata_bytes(self) -> int:
        return self.feat.numel() * 2 + self.buckets.numel() * 4

    def to(self, device) -> "SupergroupGraph":
        return SupergroupGraph(self.plan, self.feat.to(device), self.buckets.to(device))


@dataclass(frozen=True)
class GraphSpec:
    """Provenance of a generated graph (kgen_graph.py:310-335)."""

    K: int
    C: int
    S: int
    R: int
    seed: int
    quantum: int
    generation: str = "balanced_permutation"
    generator: str = GENERATOR
    generator_version: int = GENERATOR_VERSION
    source: str = "generated"

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self), sort_keys=True)

    @staticmethod
    def from_json(s: str) -> "GraphSpec":
        return GraphSpec(**json.loads(s))

    def plan(self) -> ConnectivityPlan:
        return ConnectivityPlan(self.S, self.R, self.generation, self.seed)


def seeded_generator(seed: int, *salt: int, device="cpu") -> torch.Generator:
    """Independent generator per salt tuple: the seed is mixed as h <- (h * 0x9E3779B1 + s + 0x7F4A7C15)
    mod 2^48 for every salt s (supergroups.py:117-123)."""
    g = torch.Generator(device=device)
    h = seed & 0xFFFFFFFF
    for s in salt:
        h = (h * 0x9E3779B1 + s + 0x7F4A7C15) & 0xFFFFFFFFFFFF
    g.manual_seed(h)
    return g


def interleaved_order(Q: int, R: int) -> torch.Tensor:
    """Assignment position p -> set (round p % R, set p // R of that round)."""
    per = Q // R
    p = torch.arange(Q)
    return (p % R) * per + p // R


def valid_units(counts: torch.Tensor, C: int, quantum: int) -> torch.Tensor:
    """[G] assignment units (quantum blocks of C neurons) holding at least one valid neuron."""
    un = quantum * C
    return (counts.to(torch.int64) + un - 1) // un


def unit_quotas(nvu: torch.Tensor, Q: int, R: int):
    """(counts [G, Q] units of output g in set q, keys [G, Q] bucket order inside output g)."""
    nvu = nvu.to("cpu", torch.int64)
    G = nvu.numel()
    base, rem = nvu // Q, nvu % Q
    ptr = (torch.cumsum(rem, 0) - rem) % Q          # extras rotate over the outputs
    key = (torch.arange(Q)[None, :] - ptr[:, None]) % Q
    counts_pos = base[:, None] + (key < rem[:, None]).to(torch.int64)
    # each output's partial tail unit goes last, on its least-loaded nonempty position
    load = torch.zeros(Q, dtype=torch.int64)
    huge = torch.iinfo(torch.int64).max // 4
    for g in range(G):
        score = torch.where(counts_pos[g] > 0, load * (Q + 1) + key[g], torch.full_like(key[g], huge))
        p = int(torch.argmin(score))
        load[p] += 1
        key[g, p] = Q
    order = interleaved_order(Q, R)
    counts = torch.zeros((G, Q), dtype=torch.int64)
    keys = torch.zeros((G, Q), dtype=torch.int64)
    counts[:, order] = counts_pos
    keys[:, order] = key
    return counts, keys


def make_feature_sets(D: int, plan: ConnectivityPlan, device="cpu") -> torch.Tensor:
    """feat [Q, S] int16: R seeded permutations of range(D) cut into rows of S, rows sorted."""
    S, R = plan.input_supergroup_dim, plan.partition_rounds
    if S == D:
        if R != 1:
            raise ValueError("S = D is the unrestricted working-set control: use a single set (R = 1)")
        return torch.arange(D, dtype=torch.int16, device=device)[None]
    rounds = [torch.randperm(D, generator=seeded_generator(plan.seed, 1, r)).reshape(D // S, S) for r in range(R)]
    return torch.cat(rounds).sort(dim=1).values.to(torch.int16).to(device)


def bucket_table(D: int, nvu: torch.Tensor, plan: ConnectivityPlan):
    """(feat [Q, S] int16, buckets [n, 4] int32 (q, g, first unit, units)) on the CPU."""
    Q = plan.num_supergroups(D)
    feat = make_feature_sets(D, plan)
    counts, keys = unit_quotas(nvu, Q, plan.partition_rounds)
    order = torch.argsort(keys, dim=1)
    cnt_sorted = torch.gather(counts, 1, order)
    start = torch.empty_like(cnt_sorted)
    start.scatter_(1, order, torch.cumsum(cnt_sorted, 1) - cnt_sorted)
    qg = torch.nonzero(counts.t() > 0)                  # (q, g) ascending
    q_b, g_b = qg[:, 0], qg[:, 1]
    buckets = torch.stack([q_b, g_b, start[g_b, q_b], counts[g_b, q_b]], 1).to(torch.int32)
    return feat, buckets


@torch.no_grad()
def generate_records(D: int, counts: torch.Tensor, C: int, K: int, NB: int, quantum: int, plan: ConnectivityPlan,
                     device, chunk_elems: int = 1 << 26):
    """(records [G, NB, K] int16 global ids, feat [Q, S] int16, unit buckets [n, 4] int32, stats).

    ``counts`` [G] valid neurons per output, blocks of C neurons, assignment units of ``quantum`` blocks."""
    S = plan.input_supergroup_dim
    if S % K:
        raise ValueError(f"S = {S} must be a multiple of the fan-in K = {K}")
    t0 = time.perf_counter()
    dev = torch.device(device)
    G = counts.numel()
    Q = plan.num_supergroups(D)
    nvu = valid_units(counts, C, quantum)
    if int(nvu.max()) * quantum > NB:
        raise ValueError("NB too small for the valid units")
    feat, buckets = bucket_table(D, nvu, plan)
    q_b, g_b = buckets[:, 0].to(torch.int64), buckets[:, 1].to(torch.int64)
    rec = torch.empty((G, NB, K), dtype=torch.int16, device=dev)
    flat = rec.view(-1, K)
    blocks_b = buckets[:, 3].to(torch.int64) * quantum         # records consumed by each bucket
    blocks_q = torch.zeros(Q, dtype=torch.int64).index_add_(0, q_b, blocks_b)
    per_perm = S // K
    feat_d = feat.to(dev).to(torch.int64)
    dest0 = g_b * NB + buckets[:, 2].to(torch.int64) * quantum  # first destination block of each bucket
    off_b = torch.cumsum(blocks_b, 0) - blocks_b
    off_q = torch.cumsum(blocks_q, 0) - blocks_q
    q0 = 0
    while q0 < Q:  # batches of sets whose permutation buffers fit chunk_elems (the draw order is per set)
        q1, elems = q0, 0
        while q1 < Q and (q1 == q0 or elems + math.ceil(int(blocks_q[q1]) / per_perm) * S <= chunk_elems):
            elems += math.ceil(int(blocks_q[q1]) / per_perm) * S
            q1 += 1
        for q in range(q0, q1):
            n = int(blocks_q[q])
            if n == 0:
                continue
            gq = seeded_generator(plan.seed, 2, q, device=dev)
            if plan.generation == "balanced_permutation":
                nperm = math.ceil(n / per_perm)
                loc = torch.argsort(torch.rand((nperm, S), generator=gq, device=dev), dim=1)
                loc = loc.reshape(nperm * per_perm, K)[:n]
            else:
                loc = _distinct_sorted_records(n, S, K, gq, dev)
            glob = feat_d[q][loc.sort(dim=1).values]
            lo, hi = int(torch.searchsorted(q_b, q)), int(torch.searchsorted(q_b, q, right=True))
            nb = blocks_b[lo:hi].to(dev)
            within = torch.arange(n, device=dev) - torch.repeat_interleave((off_b[lo:hi] - off_q[q]).to(dev), nb)
            flat[torch.repeat_interleave(dest0[lo:hi].to(dev), nb) + within] = glob.to(torch.int16)
        q0 = q1
    pad = torch.arange(NB, device=dev)[None, :] >= (nvu.to(dev) * quantum)[:, None]
    rec[pad] = rec[:, :1, :].expand(G, NB, K)[pad]
    stats = {"generation_seconds": time.perf_counter() - t0}
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
        stats["generation_seconds"] = time.perf_counter() - t0
    return rec, feat.to(dev), buckets.to(dev), stats


@torch.no_grad()
def generate_indices(layout: SparseLayout, plan: ConnectivityPlan, device):
    """Mode-B canonical indices [G, NB, 8] int16, SupergroupGraph, stats (supergroups.py:200-271)."""
    if not layout.shared_indices:
        raise ValueError("input supergroups are defined for Mode B (shared index records)")
    counts = layout.counts_tensor("cpu")
    rec, feat, buckets, stats = generate_records(layout.input_dim, counts, layout.block, 8, layout.blocks_per_group,
                                                 layout.unit_blocks, plan, device)
    return rec, SupergroupGraph(plan, feat, buckets), stats


def unit_to_block_buckets(buckets: torch.Tensor, counts: torch.Tensor, C: int, quantum: int) -> torch.Tensor:
    """Unit buckets -> logical-block buckets (q, g, first block, blocks), trimmed to blocks holding
    valid neurons (kgen_graph.py:154-162)."""
    b = buckets.to(torch.int64)
    nvb = (counts.to(b.device).to(torch.int64) + C - 1) // C
    first = b[:, 2] * quantum
    end = torch.minimum(first + b[:, 3] * quantum, nvb[b[:, 1]])
    out = torch.stack([b[:, 0], b[:, 1], first, end - first], 1)
    return out[out[:, 3] > 0].to(torch.int32).contiguous()


def block_sets(G: int, NB: int, block_buckets: torch.Tensor, device) -> torch.Tensor:
    """[G*NB] int64 set q of every logical block (-1: in no bucket)."""
    b = block_buckets.to(device).to(torch.int64)
    rb = torch.repeat_interleave(torch.arange(len(b), device=device), b[:, 3])
    kb = torch.arange(len(rb), device=device) - torch.repeat_interleave(torch.cumsum(b[:, 3], 0) - b[:, 3], b[:, 3])
    bq = torch.full((G * NB,), -1, dtype=torch.int64, device=device)
    bq[b[rb, 1] * NB + b[rb, 2] + kb] = b[rb, 0]
    return bq


@torch.no_grad()
def validate_records(D: int, counts: torch.Tensor, C: int, K: int, rec: torch.Tensor, feat: torch.Tensor,
                     block_buckets: torch.Tensor, R: int) -> Dict:
    """Structural checks of a generated graph (raise on violation; kgen_graph.py:221-285): every valid block
    in exactly one bucket of its output; records sorted, distinct, in range and inside their set; every
    feature in exactly R sets; valid neurons sum to H."""
    dev = rec.device
    G, NB, Kx = rec.shape
    if Kx != K:
        raise AssertionError("record width != K")
    counts = counts.to(dev).to(torch.int64)
    nvb = (counts + C - 1) // C
    Q, S = feat.shape
    b = block_buckets.to(dev).to(torch.int64)
    if bool((b[:, 3] <= 0).any()):
        raise AssertionError("empty bucket")
    key = b[:, 0] * G + b[:, 1]
    if torch.unique(key).numel() != len(b) or not bool((key[1:] >= key[:-1]).all()):
        raise AssertionError("buckets are not unique and sorted by (set, output)")
    start = b[:, 1] * NB + b[:, 2]
    rb = torch.repeat_interleave(torch.arange(len(b), device=dev), b[:, 3])
    kb = torch.arange(len(rb), device=dev) - torch.repeat_interleave(torch.cumsum(b[:, 3], 0) - b[:, 3], b[:, 3])
    cover = torch.zeros(G * NB, dtype=torch.int64, device=dev).index_add_(0, start[rb] + kb, torch.ones_like(kb))
    valid_blk = (torch.arange(NB, device=dev)[None, :] < nvb[:, None]).reshape(-1)
    if not bool((cover[valid_blk] == 1).all()) or bool((cover[~valid_blk] != 0).any()):
        raise AssertionError("buckets do not cover exactly the valid blocks")
    rv = rec.view(-1, K)[valid_blk].to(torch.int64)
    if not bool((rv.sort(dim=1).values == rv).all()) or bool((rv[:, 1:] == rv[:, :-1]).any()):
        raise AssertionError("a record is not sorted and distinct")
    if int(rv.min()) < 0 or int(rv.max()) >= D:
        raise AssertionError("index out of range")
    featd = feat.to(dev).to(torch.int64)
    member = torch.zeros(D, dtype=torch.int64, device=dev).index_add_(0, featd.reshape(-1),
                                                                       torch.ones(Q * S, dtype=torch.int64, device=dev))
    if not bool((member == R).all()):
        raise AssertionError("a feature is not in exactly R sets")
    bq = block_sets(G, NB, b, dev)[valid_blk]
    onehot = torch.zeros((Q, D), dtype=torch.bool, device=dev)
    onehot.scatter_(1, featd, True)
    if not bool(onehot[bq[:, None], rv].all()):
        raise AssertionError("a record uses a feature outside its set")
    vn = torch.clamp(counts[:, None] - torch.arange(NB, device=dev)[None, :] * C, min=0, max=C).reshape(-1)[valid_blk]
    if int(vn.sum()) != int(counts.sum()):
        raise AssertionError("valid neurons in records != H")
    per_q = torch.zeros(Q, dtype=torch.int64, device=dev).index_add_(0, b[:, 0], b[:, 3])
    return dict(H=int(counts.sum()), logical_records=int(valid_blk.sum()), Q=Q, S=S, R=R, K=K, C=C, buckets=len(b),
                records_per_supergroup=dict(min=int(per_q.min()), max=int(per_q.max()),
                                            mean=float(per_q.double().mean())))
