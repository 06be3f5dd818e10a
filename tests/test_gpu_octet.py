"""The octet arrangement (gl_group_octets) and the lane-per-neuron kernels (gl_fwd_octet_f32 /
gl_bwd_octet_f32), through the C ABI.

* The arrangement is a valid storage permutation (valid slots permuted within their group, padding slots
  in place, every record's inputs permuted), deterministic, and balanced: at the benchmarked geometry
  nearly every (octet, input position) reads 8 distinct residues d mod 8.
* The kernels match the float64 C oracle (the reference's algorithm, pytorch_reference.py:29-105) on
  slot-order and on octet-arranged storage, over ragged groups, D from 9 to 5000 (the fixed and the
  runtime tile offset), B from 1 to 256, mean / sum pools and the three activations.  Tolerances:
  forward rtol 1e-5 / atol 1e-6; dX, dW, db rtol 1e-4 / atol 1e-5, plus the oracle's allowance for
  (token, neuron) pairs on ReLU's jump.
* A token whose upstream gradient is NaN gets a NaN dX row, as fp32 arithmetic would give.
"""
import pytest
import torch

from conftest import assert_close
from granulelayer_b200 import _native
from granulelayer_b200.layout import SparseLayout, init_parameters
from oracle import oracle as O

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)
POOLS = {"mean": _native.POOL_MEAN, "sum": _native.POOL_SUM}


def _layer(D, H, G, seed=0, bias_std=0.2, rule="distinct"):
    L = SparseLayout(D, H, G, 8, 8, False)
    idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=seed, bias_std=bias_std)
    if rule == "uniform":
        gen = torch.Generator().manual_seed(seed + 100)
        valid = L.valid_mask("cpu").reshape(G, -1, 8)[..., None]
        idx = torch.where(valid, torch.randint(0, D, idx.shape, generator=gen).to(torch.int16), idx)
    return L, idx, w, b


def _arrange(L, idx):
    """(order, kperm) [G, NB*8] of gl_group_octets."""
    G, NB = L.groups, L.blocks_per_group
    o = torch.empty((G, NB * 8), dtype=torch.int32, device="cuda")
    kp = torch.empty_like(o)
    _native.group_octets(idx.cuda(), L.counts_tensor("cuda").to(torch.int32), L.input_dim, NB, 0, G, o, kp)
    torch.cuda.synchronize()
    return o.cpu(), kp.cpu()


def _inputs_of(kp):
    sh = torch.arange(0, 24, 3, dtype=torch.int32)
    return ((kp[:, :, None] >> sh) & 7).long()


def _apply(t, order, kp):
    """A parameter-shaped tensor in the arranged storage order."""
    G, slots = order.shape
    per = t.numel() // (G * slots)
    v = torch.gather(t.reshape(G, slots, per), 1, order.long()[:, :, None].expand(G, slots, per))
    if per == 8:
        v = torch.gather(v, 2, _inputs_of(kp))
    return v.reshape(t.shape)


def _interleave(t):
    """Weights / dW in the octet weight layout the kernels read: per block of 32 records, the records'
    weights 0-3 (16 bytes each), then their weights 4-7."""
    G = t.shape[0]
    return t.reshape(G, -1, 32, 2, 4).transpose(2, 3).reshape(t.shape).contiguous()


@pytest.mark.parametrize("rule", ["distinct", "uniform"])
def test_octet_arrangement_is_valid_deterministic_and_balanced(rule):
    D, G = 4096, 3
    L, idx, _, _ = _layer(D, 3 * 24576 - 5, G, seed=7, rule=rule)    # ragged: counts 24573 / 24573 / 24573
    order, kp = _arrange(L, idx)
    order2, kp2 = _arrange(L, idx)
    assert torch.equal(order, order2) and torch.equal(kp, kp2), "the arrangement is deterministic"
    counts = L.counts_tensor("cpu")
    slots = L.blocks_per_group * 8
    ks = _inputs_of(kp)
    assert torch.equal(ks.sort(dim=2).values, torch.arange(8).expand_as(ks)), "kperm rows are permutations"
    for g in range(G):
        n = int(counts[g])
        assert torch.equal(order[g, :n].sort().values, torch.arange(n, dtype=torch.int32))
        assert torch.equal(order[g, n:], torch.arange(n, slots, dtype=torch.int32))
        assert torch.equal(ks[g, n:], torch.arange(8).expand(slots - n, 8))
    stored = _apply(idx, order, kp).reshape(G, slots, 8).long()
    distinct = 0
    total = 0
    for g in range(G):
        n = int(counts[g]) // 8 * 8
        res = (stored[g, :n] & 7).reshape(-1, 8, 8)             # [octet, record, column]
        onehot = torch.nn.functional.one_hot(res, 8).sum(1)      # [octet, column, residue]
        distinct += int((onehot.max(-1).values == 1).sum())
        total += onehot.shape[0] * 8
    frac = distinct / total
    assert frac > 0.9, f"only {frac:.3f} of the (octet, column) pairs read 8 distinct residues"


def _oracle(L, idx, w, b, x, dy, pool, act):
    c = L.counts_tensor("cpu").numpy()
    args = (x.numpy(), idx.numpy(), w.numpy(), b.numpy(), c)
    pre = O.forward(*args, pool, act)
    dx, dw, db, sdx, sdw, sdb = O.backward(*args, dy.numpy(), pool, act, slack=True)
    return [torch.from_numpy(a) for a in (pre, dx, dw, db, sdx, sdw, sdb)]


def _run(L, idx, w, b, x, gpre, pool, act):
    dev = "cuda"
    idx, w, b, x, gpre = idx.to(dev), w.to(dev), b.to(dev), x.to(dev), gpre.to(dev)
    counts = L.counts_tensor(dev).to(torch.int32)
    G, NB, B = L.groups, L.blocks_per_group, x.shape[0]
    pre = torch.full((B, G), float("nan"), device=dev)
    wabsmax = torch.empty(G, device=dev)
    _native.fwd_octet(x, idx, w, b, counts, pre, NB, 0, G, POOLS[pool], _native.ACT_IDS[act], wabsmax=wabsmax)
    rowmax = torch.empty(G, device=dev, dtype=torch.int32)
    _native.group_index_maxcount(idx, counts, L.input_dim, NB, 0, G, rowmax)
    dx = torch.zeros(B, L.input_dim, device=dev)
    dw, db = torch.zeros_like(w), torch.zeros_like(b)
    _native.bwd_octet(x, idx, w, b, counts, gpre, dx, dw, db, NB, 0, G, POOLS[pool], _native.ACT_IDS[act],
                      wabsmax, rowmax)
    torch.cuda.synchronize()
    want_wmax = w.reshape(G, -1).abs().amax(1)
    assert torch.equal(wabsmax, want_wmax), "the forward's max |w| per group"
    return pre.cpu(), dx.cpu(), dw.cpu(), db.cpu()


CASES = [  # D, H, G, B, pool, act
    (4096, 2 * 24576, 2, 256, "mean", "relu"),
    (256, 65536, 256, 64, "sum", "relu"),
    (100, 5003, 7, 37, "mean", "gelu"),
    (9, 3000, 3, 5, "mean", "identity"),
    (5000, 20011, 3, 33, "sum", "relu"),
    (1024, 8192, 4, 1, "mean", "relu"),
]


@pytest.mark.parametrize("arranged", [False, True])
@pytest.mark.parametrize("D,H,G,B,pool,act", CASES)
def test_octet_kernels_match_oracle(D, H, G, B, pool, act, arranged):
    L, idx, w, b = _layer(D, H, G, seed=D + B)
    gen = torch.Generator().manual_seed(B)
    x = torch.randn(B, D, generator=gen)
    dy = torch.randn(B, G, generator=gen)
    pre, odx, odw, odb, sdx, sdw, sdb = _oracle(L, idx, w, b, x, dy, pool, act)
    if arranged:
        order, kp = _arrange(L, idx)
        idx, w, b = _apply(idx, order, kp), _apply(w, order, kp), _apply(b, order, kp)
        odw, sdw = _apply(odw, order, kp), _apply(sdw, order, kp)
        odb, sdb = _apply(odb, order, kp), _apply(sdb, order, kp)
    w, odw, sdw = _interleave(w), _interleave(odw), _interleave(sdw)
    y, dx, dw, db = _run(L, idx, w, b, x, dy, pool, act)
    assert_close(y, pre, what="y", **FWD)
    assert_close(dx, odx, what="dx", slack=sdx, **BWD)
    assert_close(dw, odw, what="dw", slack=sdw, **BWD)
    assert_close(db, odb, what="db", slack=sdb, **BWD)


def test_octet_backward_marks_a_nan_token():
    L, idx, w, b = _layer(256, 4096, 4, seed=3)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(6, 256, generator=gen)
    dy = torch.randn(6, 4, generator=gen)
    dy[2, 1] = float("nan")
    _, dx, _, _ = _run(L, idx, w, b, x, dy, "mean", "relu")
    assert torch.isnan(dx[2]).all()
    assert torch.isfinite(dx[[0, 1, 3, 4, 5]]).all()


def test_octet_entry_points_reject_what_they_do_not_run():
    L, idx, w, b = _layer(64, 1024, 2)
    dev = "cuda"
    idx, w, b = idx.to(dev), w.to(dev), b.to(dev)
    counts = L.counts_tensor(dev).to(torch.int32)
    x = torch.randn(4, 64, device=dev)
    pre = torch.empty(4, 2, device=dev)
    with pytest.raises(_native.NativeLibraryError, match=r"\[-4\]"):      # max pooling: not these kernels
        _native.fwd_octet(x, idx, w, b, counts, pre, L.blocks_per_group, 0, 2, _native.POOL_MAX, 1)
    dx = torch.zeros(4, 64, device=dev)
    with pytest.raises(_native.NativeLibraryError, match=r"\[-1\]"):      # the fixed-point bounds are required
        lib = _native.load()
        a = _native.GlBwdArgs()
        a.x, a.idx, a.w, a.b, a.counts = (_native._ptr(t) for t in (x, idx, w, b, counts))
        a.gpre, a.dx, a.dw, a.db = (_native._ptr(t) for t in (pre, dx, torch.zeros_like(w), torch.zeros_like(b)))
        a.B, a.D, a.NB, a.g0, a.g1, a.ldx, a.ldg, a.lddx = 4, 64, L.blocks_per_group, 0, 2, 64, 2, 64
        a.pool, a.act = _native.POOL_MEAN, 1
        _native._check(lib, lib.gl_bwd_octet_f32(_native.ctypes.byref(a), None), "gl_bwd_octet_f32")
    big = torch.zeros(4, 8000, device=dev)
    with pytest.raises(_native.NativeLibraryError, match=r"\[-5\]"):      # two tiles of 8000 features
        L2 = SparseLayout(8000, 1024, 2, 8, 8, False)
        i2, w2, b2 = init_parameters(L2, dev, dtype=torch.float32, seed=1)
        _native.fwd_octet(big, i2, w2, b2, L2.counts_tensor(dev).to(torch.int32), pre, L2.blocks_per_group, 0, 2,
                          _native.POOL_MEAN, 1)


def test_drop_in_layer_with_octet_layout():
    """SparsePoolingLayer(weight_layout="octet"): the same outputs and gradients as the reference-layout layer
    (through the octet kernels), its state dict in the reference's slot order bit for bit, and a state dict
    loaded into it runs the loaded parameters."""
    from granulelayer_b200 import SparsePoolingLayer

    D, H, G, B = 4096, 2 * 24576 + 1003, 3, 64
    kw = dict(shared_neurons=None, pooling="mean", dtype=torch.float32, seed=9, bias_std=0.1)
    ref = SparsePoolingLayer(D, H, G, **kw).cuda()
    lay = SparsePoolingLayer(D, H, G, weight_layout="octet", **kw).cuda()
    gen = torch.Generator().manual_seed(4)
    x = torch.randn(B, D, generator=gen).cuda()
    dy = torch.randn(B, G, generator=gen).cuda()
    outs = []
    for m in (ref, lay):
        xr = x.clone().requires_grad_(True)
        y = m(xr)
        y.backward(dy)
        outs.append((y.detach(), xr.grad))
    assert lay.last_info["forward_kernel"] == "gl_fwd_octet_f32"
    assert lay.last_info["backward_kernel"] == "gl_bwd_octet_prefix_f32"
    assert_close(outs[1][0], outs[0][0], what="y", **FWD)
    assert_close(outs[1][1], outs[0][1], what="dx", **BWD)
    assert_close(lay.canonical(lay.weight.grad), ref.weight.grad, what="dw", **BWD)
    assert_close(lay.canonical(lay.bias.grad), ref.bias.grad, what="db", **BWD)
    assert not torch.equal(lay.weight.detach(), ref.weight.detach()), "the octet layer stores permuted records"
    sd, rsd = lay.state_dict(), ref.state_dict()
    assert sd.keys() == rsd.keys()
    for k in rsd:
        assert torch.equal(sd[k].cpu(), rsd[k].cpu()), f"{k}: the octet layer's checkpoint differs"
    ci, cw, cb = lay.canonical_parameters()
    assert torch.equal(ci, ref.indices) and torch.equal(cw, ref.weight.detach()) and torch.equal(cb, ref.bias.detach())
    other = SparsePoolingLayer(D, H, G, **dict(kw, seed=10)).cuda()
    lay.load_state_dict(other.state_dict())
    y2, y3 = lay(x), other(x)
    assert lay.last_info["forward_kernel"] == "gl_fwd_octet_f32"
    assert_close(y2.detach(), y3.detach(), what="y after load", **FWD)


@pytest.mark.parametrize("D,pool,accum", [(8000, "mean", "auto"), (256, "max", "auto"), (256, "mean", "fp32")])
def test_octet_layout_keeps_slot_order_where_its_kernels_do_not_run(D, pool, accum):
    """An octet layer that the lane-per-neuron kernels cannot run (input too wide for their tiles, a pool
    other than mean / sum, fp32 dX atomics asked for) keeps the reference's storage and the generic kernels."""
    from granulelayer_b200 import PhysicalPlan, SparsePoolingLayer

    kw = dict(shared_neurons=None, pooling=pool, dtype=torch.float32, seed=2, bias_std=0.1,
              plan=PhysicalPlan(b200_dx_accum=accum))
    ref = SparsePoolingLayer(D, 4096, 4, **kw).cuda()
    lay = SparsePoolingLayer(D, 4096, 4, weight_layout="octet", **kw).cuda()
    x = torch.randn(8, D, device="cuda")
    y, yr = lay(x), ref(x)
    assert lay._order is None and torch.equal(lay.weight.detach(), ref.weight.detach())
    assert lay.last_info.get("forward_kernel") != "gl_fwd_octet_f32"
    assert_close(y.detach(), yr.detach(), what="y", **FWD)


@pytest.mark.parametrize("rule", ["distinct", "uniform"])
def test_feature_prefix_counts_record_inputs(rule):
    """gl_group_feature_prefix: per feature, the record inputs of the valid records of groups g0 .. g0+i-1
    (duplicate indices counted with their multiplicity), over a sub-range of the groups."""
    D, G = 300, 7
    L, idx, _, _ = _layer(D, 7 * 900 - 13, G, seed=5, rule=rule)
    g0, g1 = 2, 6
    out = torch.empty((g1 - g0 + 1) * D, dtype=torch.int32, device="cuda")
    _native.group_feature_prefix(idx.cuda(), L.counts_tensor("cuda").to(torch.int32), D, L.blocks_per_group, g0, g1,
                                 out)
    counts = L.counts_tensor("cpu")
    want = torch.zeros(g1 - g0 + 1, D, dtype=torch.int64)
    for i, g in enumerate(range(g0, g1)):
        rec = idx[g].reshape(-1, 8)[: int(counts[g])].reshape(-1).long()
        want[i + 1] = want[i] + torch.bincount(rec, minlength=D)
    assert torch.equal(out.cpu().reshape(g1 - g0 + 1, D).long(), want)


@pytest.mark.parametrize("rule", ["distinct", "uniform"])
def test_prefix_backward_equals_the_plain_one(rule):
    """gl_bwd_octet_prefix_f32 accumulates the rounding's raw bits and subtracts the offsets at the flush:
    with one group chunk per token block (so every dx element receives one flush) its dx is bit for bit that
    of gl_bwd_octet_f32; dw / db agree within the backward tolerance (their global reductions' order varies)."""
    D, H, G, B = 512, 4 * 3000 + 77, 4, 37
    L, idx, w, b = _layer(D, H, G, seed=11, rule=rule)
    order, kp = _arrange(L, idx)
    idx, w, b = _apply(idx, order, kp), _interleave(_apply(w, order, kp)), _apply(b, order, kp)
    dev = "cuda"
    idx, w, b = idx.to(dev), w.to(dev), b.to(dev)
    counts = L.counts_tensor(dev).to(torch.int32)
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(B, D, generator=gen).to(dev)
    gpre = torch.randn(B, G, generator=gen).to(dev)
    NB = L.blocks_per_group
    wabsmax = w.reshape(G, -1).abs().amax(1).contiguous()
    rowmax = torch.empty(G, device=dev, dtype=torch.int32)
    _native.group_index_maxcount(idx, counts, D, NB, 0, G, rowmax)
    prefix = torch.empty((G + 1) * D, dtype=torch.int32, device=dev)
    _native.group_feature_prefix(idx, counts, D, NB, 0, G, prefix)
    outs = []
    for fp in (None, prefix):
        dx = torch.zeros(B, D, device=dev)
        dw, db = torch.zeros_like(w), torch.zeros_like(b)
        _native.bwd_octet(x, idx, w, b, counts, gpre, dx, dw, db, NB, 0, G, POOLS["mean"], _native.ACT_IDS["relu"],
                          wabsmax, rowmax, groups_per_cta=G, feat_prefix=fp)
        torch.cuda.synchronize()
        outs.append((dx.cpu(), dw.cpu(), db.cpu()))
    assert torch.equal(outs[0][0], outs[1][0]), "dx of the folded flush"
    assert_close(outs[1][1], outs[0][1], what="dw", **BWD)
    assert_close(outs[1][2], outs[0][2], what="db", **BWD)
