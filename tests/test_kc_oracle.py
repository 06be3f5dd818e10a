"""The float64 K/C oracle and the Cover-TopK/16 construction against the reference's own outputs
(``tests/golden/kc_reference.npz``, made by ``make_golden.py`` from the reference's
``CoverTopK16Layer.from_envelope`` and ``experimental/reference.grads``), and the kernels' schedule."""
import json

import numpy as np
import torch

from conftest import GOLDEN
from granulelayer_b200.cover_topk16 import CoverTopK16Layer
from granulelayer_b200.kgen import KLayout, init_envelope_parameters
from granulelayer_b200.supergroups import ConnectivityPlan
from oracle import kc_oracle


def _fixture():
    d = np.load(GOLDEN / "kc_reference.npz")
    return json.loads(str(d["meta"])), {k: d[k] for k in d.files if k != "meta"}


def fixture_layer(device="cpu") -> CoverTopK16Layer:
    """The fixture's layer rebuilt by this package (bit-exact with the reference's, see below)."""
    meta, _ = _fixture()
    D, H, G, R = meta["D"], meta["H"], meta["G"], meta["R"]
    w, b = init_envelope_parameters(KLayout(D, H, G, 64, 256), "cpu", dtype=torch.bfloat16, seed=meta["seed"],
                                    bias_std=0.1)
    return CoverTopK16Layer.from_envelope(w, b, input_dim=D, hidden_dim=H, output_dim=G,
                                          connectivity=ConnectivityPlan(64, R, seed=meta["graph_seed"]),
                                          device=device)


def test_oracle_matches_reference_fixture():
    _, a = _fixture()
    y, dx, dw, db = kc_oracle.grads(a["x"], a["indices"], a["weight"], a["bias"], a["counts"], a["gy"])
    for name, v in (("y", y), ("dx", dx), ("dw", dw), ("db", db)):
        np.testing.assert_allclose(v, a[name], rtol=1e-12, atol=1e-15, err_msg=name)
    np.testing.assert_allclose(kc_oracle.forward(a["x"], a["indices"], a["weight"], a["bias"], a["counts"]), a["y"],
                               rtol=1e-12, atol=1e-15)


def test_construction_matches_reference_fixture():
    _, a = _fixture()
    lay = fixture_layer()
    assert np.array_equal(lay.indices.numpy(), a["indices"])
    assert np.array_equal(lay.weight.detach().numpy(), a["weight"])
    assert np.array_equal(lay.bias.detach().numpy(), a["bias"])
    assert np.array_equal(lay.sg_feat.numpy(), a["sg_feat"])
    assert np.array_equal(lay.kg_buckets.numpy(), a["kg_buckets"])
    assert np.array_equal(lay.env.numpy(), a["env"])
    assert np.array_equal(lay.counts.numpy(), a["counts"])


def test_oracle_slack_is_zero_away_from_the_jump():
    _, a = _fixture()
    *_, (sdx, sdw, sdb) = kc_oracle.grads(a["x"], a["indices"], a["weight"], a["bias"], a["counts"], a["gy"],
                                          slack=True)
    # continuous random inputs put no pre-activation within 1e-6 relative of 0
    assert sdx.max() == 0 and sdw.max() == 0 and sdb.max() == 0


def test_schedule_invariants():
    lay = fixture_layer()
    s = lay._work()
    bk = s["buckets"].long()
    q_off, rec_off = s["q_off"].long(), s["rec_off"].long()
    Q = lay.sg_feat.shape[0]
    assert bool((bk[1:, 0] >= bk[:-1, 0]).all()), "buckets sorted by set"
    assert q_off.shape == (Q + 1,) and int(q_off[0]) == 0 and int(q_off[-1]) == len(bk)
    for q in range(Q):
        assert bool((bk[q_off[q]:q_off[q + 1], 0] == q).all())
    assert torch.equal(rec_off[1:] - rec_off[:-1], bk[:, 3])
    # every valid 16-record of every output is in exactly one bucket
    L = lay.layout
    cover = torch.zeros(L.groups * L.blocks_per_group, dtype=torch.long)
    for q, g, j, n in bk.tolist():
        cover[g * L.blocks_per_group + j: g * L.blocks_per_group + j + n] += 1
    nvb = (lay.counts.long() + 15) // 16
    live = (torch.arange(L.blocks_per_group)[None, :] < nvb[:, None]).reshape(-1)
    assert bool((cover[live] == 1).all()) and bool((cover[~live] == 0).all())
    # every record's inputs are in its set: feat[q][env] == indices
    for q, g, j, n in bk.tolist()[:64]:
        f = g * L.blocks_per_group + j
        assert torch.equal(lay.sg_feat[q][lay.env[f:f + n].long()], lay.indices.view(-1, 16)[f:f + n])
