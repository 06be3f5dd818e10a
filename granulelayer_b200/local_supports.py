"""Cover-TopK/16 support selection and one-time row normalization
(mirror of the "Cover-TopK" path of sparse_pooling/experimental/local_supports.py
and of sparse_pooling/experimental/row_normalize.py).

Given the K64 envelope (``kgen.Envelope``), every valid 16-neuron row group
u = (g, j, c // 16) keeps k = 16 of its record's 64 local inputs:

1. importance a[u, j] = sum over the valid neurons c of u of W_pre[u, c, j]^2 in
   float64, added sequentially over c = 0..15 (local_supports.py:208-222);
2. TopK: the k largest a[u, j], ties to the lower coordinate (stable
   descending sort; :279-282);
3. cover repair: inside each original record every one of its 64 inputs must be
   kept by at least one valid row group; while an input is uncovered, apply the
   swap (u, d -> j) of minimum a[u, d] - a[u, j] over uncovered j, groups u and
   kept donors d with record count >= 2, ties lexicographic in (j, u, d)
   (:293-373); records with m k < 64 are infeasible and raise.

All steps are float64/integer and order-determined, so the selection is
bit-exact with the reference (pinned by tests against its outputs).
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import torch

from .supergroups import block_sets

SCHEMA = "granule.local_supports/2"
RNG_SCHEMA = "granule.local_supports/1"     # key / fingerprint namespace of the reference
POLICY = "Cover-TopK"
COVER_CHUNK_RECORDS = 1 << 15
NORM_SCHEMA = "granule.row_normalize/1"
S_MAX, EPS_REL = 8.0, 1e-6


@dataclass
class LocalSupport:
    """``env`` [n16, k] int64 sorted local positions per row group (padded groups: arange(k), unused),
    ``nv`` [n16] valid neurons per group, ``q`` [n16] input set (-1 padded), ``subset`` [n16]."""

    policy: str
    k: int
    env: torch.Tensor
    nv: torch.Tensor
    q: torch.Tensor
    subset: torch.Tensor
    stats: dict = field(default_factory=dict)

    def group_mask(self) -> torch.Tensor:
        m = torch.zeros((self.env.shape[0], 64), dtype=torch.bool, device=self.env.device)
        m.scatter_(1, self.env, True)
        return m & (self.nv > 0)[:, None]

    def element_mask(self, L) -> torch.Tensor:
        """[G, NB, C, 64] uint8 enabled valid slots."""
        valid = L.valid_mask(self.env.device).reshape(self.env.shape[0], 16)
        return (self.group_mask()[:, None, :] & valid[:, :, None]).to(torch.uint8).view(L.weight_shape)

    def enabled_slots(self) -> int:
        return int(self.k * self.nv.sum())

    def fingerprint(self) -> str:
        """sha256 of (k, env rows of the valid groups, their group ids) (local_supports.py:148-155)."""
        h = hashlib.sha256(f"{RNG_SCHEMA}|support|k={self.k}".encode())
        gv = self.nv > 0
        h.update(self.env[gv].to(torch.int8).cpu().numpy().tobytes())
        h.update(torch.nonzero(gv).squeeze(1).to(torch.int64).cpu().numpy().tobytes())
        return h.hexdigest()


def geometry(L, buckets: torch.Tensor, *, Q: int, device="cpu") -> dict:
    """Row-group geometry of the envelope (local_supports.py:169-205): nv, q, valid groups uv (ascending),
    their rank inside the record, record id, groups per block, per-set counts (length Q)."""
    valid = L.valid_mask(device)
    nv = valid.reshape(-1, 16).sum(1).to(torch.int64)
    gpb = L.block // 16
    bq = block_sets(L.groups, L.blocks_per_group, buckets, device)
    n16 = nv.numel()
    u = torch.arange(n16, device=device)
    q = torch.where(nv > 0, bq[u // gpb], torch.full_like(u, -1))
    if bool(((nv > 0) & (q < 0)).any()):
        raise AssertionError("a valid row group lies in a block without an input set")
    uv = torch.nonzero(nv > 0).squeeze(1)
    rank_rec = uv % gpb
    blk = uv // gpb
    if bool((nv[uv[rank_rec > 0] - 1] != 16).any()):
        raise AssertionError("valid row groups of a block are not a prefix of full groups")
    rec_valid = (nv.view(-1, gpb) > 0).any(1)
    rec_id = torch.cumsum(rec_valid.to(torch.int64), 0) - 1
    Q = int(Q)
    if len(buckets) and (int(buckets[:, 0].min()) < 0 or int(buckets[:, 0].max()) >= Q):
        raise ValueError(f"a bucket's input set lies outside the Q = {Q} sets")
    m_q = torch.bincount(q[uv], minlength=Q)
    return dict(nv=nv, q=q, uv=uv, rank_rec=rank_rec, rec=rec_id[blk], gpb=gpb, Q=Q, records=int(rec_valid.sum()),
                m_q=m_q, groups_per_record=(nv.view(-1, gpb) > 0).sum(1)[rec_valid])


@torch.no_grad()
def feature_importance(w: torch.Tensor, L, device="cpu", chunk: int = 1 << 16) -> torch.Tensor:
    """[n16, 64] float64: sum over valid neurons c of a row group of W[u, c, j]^2, added in order c = 0..15."""
    n16 = L.groups * L.blocks_per_group * L.block // 16
    wv = w.reshape(n16, 16, 64)
    valid = L.valid_mask(w.device).reshape(n16, 16)
    out = torch.empty((n16, 64), dtype=torch.float64, device=device)
    for u0 in range(0, n16, chunk):
        v = wv[u0:u0 + chunk].double() * valid[u0:u0 + chunk, :, None]
        acc = v[:, 0] * v[:, 0]
        for c in range(1, 16):
            acc = acc + v[:, c] * v[:, c]
        out[u0:u0 + chunk] = acc.to(device)
    return out


def subset_score(a: torch.Tensor, env: torch.Tensor) -> torch.Tensor:
    """[n] float64 sum of a[i, env[i, :]], added in ascending coordinate order."""
    v = torch.gather(a, 1, env)
    acc = v[:, 0].clone()
    for i in range(1, v.shape[1]):
        acc = acc + v[:, i]
    return acc


def topk_select(a_v: torch.Tensor, k: int) -> torch.Tensor:
    """[n, k] sorted positions of the k largest importances, ties to the lower coordinate."""
    return torch.sort(a_v, dim=1, descending=True, stable=True).indices[:, :k].sort(1).values


@torch.no_grad()
def cover_repair(a_v: torch.Tensor, env0: torch.Tensor, rec: torch.Tensor, rank: torch.Tensor, k: int, gpb: int,
                 S: int = 64, chunk_records: int = COVER_CHUNK_RECORDS) -> dict:
    """Coverage repair of the supports env0 [n, k] of n valid groups (group i in record rec[i] at rank rank[i]).

    Records are independent and advance one swap per round.  For a group u the cheapest removable donor is
    d*(u) = first argmin {a[u, d] : d kept by u, count[d] >= 2}; the swap taken is the first minimum of
    a[u, d*(u)] - a[u, j] over uncovered j and groups u, enumerated j-major then u (lexicographic (j, u, d))."""
    dev = a_v.device
    nrec = int(rec.max()) + 1 if rec.numel() else 0
    slot = torch.full((nrec, gpb), -1, dtype=torch.int64, device=dev)
    slot[rec.to(dev), rank.to(dev)] = torch.arange(rec.numel(), device=dev)
    m = (slot >= 0).sum(1)
    if nrec and int((m * k).min()) < S:
        bad = int(torch.nonzero(m * k < S)[0])
        raise ValueError(f"Cover-TopK infeasible: record {bad} has {int(m[bad])} valid groups and k = {k} "
                         f"(m k = {int(m[bad]) * k} < {S})")
    env = env0.clone().to(dev)
    missing0 = torch.zeros(nrec, dtype=torch.int64, device=dev)
    swaps = torch.zeros(nrec, dtype=torch.int64, device=dev)
    loss = torch.zeros(nrec, dtype=torch.float64, device=dev)
    inf = torch.tensor(float("inf"), dtype=torch.float64, device=dev)
    coord = torch.arange(S, device=dev)
    rounds = 0
    for r0 in range(0, nrec, chunk_records):
        sl = slot[r0:r0 + chunk_records]
        present = sl >= 0
        gi = sl.clamp_min(0)
        A = torch.where(present[:, :, None], a_v[gi].to(torch.float64), torch.zeros((), dtype=torch.float64,
                                                                                      device=dev))
        X = torch.zeros(A.shape, dtype=torch.bool, device=dev)
        X.scatter_(2, env[gi], True)
        X &= present[:, :, None]
        cnt = X.sum(1)
        missing0[r0:r0 + len(sl)] = (cnt == 0).sum(1)
        act = torch.nonzero((cnt == 0).any(1)).squeeze(1)
        nr = 0
        while act.numel():
            Xa, Aa, ca = X[act], A[act], cnt[act]
            donor_ok = Xa & (ca >= 2)[:, None, :]
            dmin, dstar = torch.where(donor_ok, Aa, inf).min(2)
            can = (ca == 0)[:, None, :] & torch.isfinite(dmin)[:, :, None] & present[act][:, :, None]
            cost = torch.where(can, dmin[:, :, None] - Aa, inf)
            best, flat = cost.permute(0, 2, 1).reshape(len(act), -1).min(1)
            if not bool(torch.isfinite(best).all()):
                raise AssertionError("Cover-TopK: an uncovered input without a legal donor swap")
            j, u = flat // gpb, flat % gpb
            d = dstar[torch.arange(len(act), device=dev), u]
            X[act, u, d] = False
            X[act, u, j] = True
            cnt[act, d] -= 1
            cnt[act, j] += 1
            loss[act + r0] += best
            swaps[act + r0] += 1
            act = act[(cnt[act] == 0).any(1)]
            nr += 1
        rounds = max(rounds, nr)
        if not bool(((X.sum(2) == k) | ~present).all()) or not bool((X.sum(1) >= 1).all()):
            raise AssertionError("Cover-TopK: repaired record violates degree k / coverage >= 1")
        order = torch.where(X, coord, coord + S).sort(2).values[:, :, :k]
        env[gi[present]] = order[present]
    if not torch.equal(swaps, missing0):
        raise AssertionError("Cover-TopK: swap count differs from the initial number of missing inputs")
    return dict(env=env, missing0=missing0, swaps=swaps, loss=loss, rounds=rounds, groups_per_record=m)


def _dist(v: torch.Tensor) -> dict:
    v = v.double()
    return dict(min=float(v.min()), max=float(v.max()), mean=float(v.mean())) if v.numel() else {}


def energy_stats(a_v: torch.Tensor, env: torch.Tensor) -> dict:
    tot = a_v.sum(1)
    kept = subset_score(a_v, env)
    return dict(layer_fraction=float(kept.sum() / tot.sum()) if float(tot.sum()) > 0 else 0.0,
                zero_energy_groups=int((tot == 0).sum()))


@torch.no_grad()
def build_cover_topk(k: int, L, buckets: torch.Tensor, w: torch.Tensor, *, Q: int, device="cpu",
                     graph_seed: int = 0) -> LocalSupport:
    """The Cover-TopK local support of fan-in k (local_supports.py:600-787, policy "Cover-TopK")."""
    if 64 % k or k not in (8, 16):
        raise ValueError("local supports: k in (8, 16)")
    geo = geometry(L, buckets.cpu(), Q=Q)
    nv, q, uv = geo["nv"], geo["q"], geo["uv"]
    env = torch.arange(k, dtype=torch.int64).repeat(nv.numel(), 1)
    subset = torch.full((nv.numel(),), -1, dtype=torch.int64)
    a_v = feature_importance(w, L)[uv]
    topk = topk_select(a_v, k)
    rep = cover_repair(a_v, topk, geo["rec"], geo["rank_rec"], k, geo["gpb"])
    env[uv] = rep["env"]
    subset[uv] = 0
    sup = LocalSupport(POLICY, k, env.to(device), nv.to(device), q.to(device), subset.to(device))
    sup.stats = dict(schema=SCHEMA, rng_schema=RNG_SCHEMA, policy=POLICY, k=k, nkt=64 // k, graph_seed=graph_seed,
                     layout_seed=None, H=int(nv.sum()), W0=64 * int(nv.sum()), enabled_slots=sup.enabled_slots(),
                     rho_mask=k / 64, valid_groups=len(uv), partial_groups=int(((nv > 0) & (nv < 16)).sum()),
                     records=geo["records"], Q=geo["Q"],
                     energy_topk=energy_stats(a_v, topk), energy=energy_stats(a_v, rep["env"]),
                     repair=dict(swaps=int(rep["swaps"].sum()), records_repaired=int((rep["swaps"] > 0).sum()),
                                 rounds=rep["rounds"], missing0_per_record=_dist(rep["missing0"]),
                                 energy_loss_total=float(rep["loss"].sum())),
                     tie_break="TopK: stable descending sort; repair: lexicographic (j, u, d)")
    return sup


@torch.no_grad()
def row_scales_energy(w_pre: torch.Tensor, mask: torch.Tensor, valid: torch.Tensor, s_max: float = S_MAX,
                      eps_rel: float = EPS_REL, chunk: int = 1 << 21):
    """(s, k, E_dense, E_kept) per neuron row (row_normalize.py:43-73, treatment "energy"):
    s = min(s_max, sqrt(E_dense / max(E_kept, eps_rel E_dense))) with fp32 sums of the BF16 values; rows
    with k = 0 or padding get 0, an all-zero dense row 1."""
    wv, mv, vv = w_pre.reshape(-1, 64), mask.reshape(-1, 64), valid.reshape(-1)
    n = wv.shape[0]
    dev = w_pre.device
    s = torch.zeros(n, dtype=torch.float32, device=dev)
    kk = torch.zeros(n, dtype=torch.int64, device=dev)
    ed = torch.zeros(n, dtype=torch.float32, device=dev)
    ek = torch.zeros(n, dtype=torch.float32, device=dev)
    for i in range(0, n, chunk):
        w = wv[i:i + chunk].float()
        m = mv[i:i + chunk] != 0
        e = (w * w).sum(1)
        ekp = (w * w * m).sum(1)
        kc = m.sum(1)
        si = torch.clamp(torch.sqrt(e / torch.maximum(ekp, eps_rel * e)), max=s_max)
        si = torch.where(e > 0, si, torch.ones_like(si))
        s[i:i + chunk] = torch.where(vv[i:i + chunk] & (kc > 0), si, torch.zeros_like(si))
        kk[i:i + chunk], ed[i:i + chunk], ek[i:i + chunk] = kc, e, ekp
    return s, kk, ed, ek


@torch.no_grad()
def normalize_energy(w_pre: torch.Tensor, b: torch.Tensor, mask: torch.Tensor, valid: torch.Tensor,
                     s_max: float = S_MAX, eps_rel: float = EPS_REL, chunk: int = 1 << 21):
    """(w_new = BF16(s_i * (w_pre * mask)), b unchanged, record) (row_normalize.py:76-119, scale_bias=False)."""
    s, k, ed, ek = row_scales_energy(w_pre, mask, valid, s_max, eps_rel, chunk)
    out = torch.empty_like(w_pre)
    ov, wv, mv = out.view(-1, 64), w_pre.reshape(-1, 64), mask.reshape(-1, 64)
    for i in range(0, wv.shape[0], chunk):
        prod = wv[i:i + chunk].float() * (mv[i:i + chunk] != 0) * s[i:i + chunk, None]
        st = prod.to(w_pre.dtype)
        if bool(((st == 0) & (prod != 0)).any()):
            raise AssertionError("scaled weights rounded to zero (support would shrink)")
        ov[i:i + chunk] = st
    con = valid.reshape(-1) & (k > 0)
    rec = dict(schema=NORM_SCHEMA, treatment="energy", scale_bias=False, s_max=s_max, eps_rel=eps_rel,
               rows=int(valid.sum()), connected_rows=int(con.sum()),
               clipped=int((con & (s >= s_max)).sum()), scale=_dist(s[con]), applied=True)
    return out, b.clone(), rec
