"""bf16 Mode-B layers on the tensor cores (gl_fwd_shared_tc): x rounded to bf16 as the reference's
compute dtype (autograd.py:349-354), bf16 x bf16 products exact in fp32, so the pooled output matches
the float64 oracle evaluated on the rounded x and the bf16 parameters (rtol 1e-5 / atol 1e-6, ReLU
boundary slack); max winners equal the oracle's (smallest slot on ties); the token tile does not
change a bit of the output; the gradients of the layer match the oracle on the same rounded x
(rtol 1e-4 / atol 1e-5, plus, for the tensor-core backward, the error of the reference's "split"
gradient precision: dz carried as hi + lo bf16, at most 2^-18 of each term, admitted as 1e-5 of the
sum of the magnitudes of each element's terms)."""
import numpy as np
import pytest
import torch

from conftest import assert_close, modeb_as_mode_a
from granulelayer_b200 import PhysicalPlan, SparsePoolingLayer, _native
from granulelayer_b200.supergroups import ConnectivityPlan
from oracle import oracle as O
from oracle import pool_oracle as P

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def _layer(C, pooling, D, H, G, seed=4, plan=None):
    return SparsePoolingLayer(D, H, G, shared_neurons=C, weight_layout="packed", pooling=pooling,
                              dtype=torch.bfloat16, seed=seed, bias_std=0.2,
                              plan=plan or PhysicalPlan()).cuda()


def _oracle_params(lay):
    L = lay.layout
    idx, w, b = modeb_as_mode_a(L, lay.indices.cpu(), lay.weight.detach().cpu().double(),
                                lay.bias.detach().cpu().double())
    return L, idx.numpy(), w.numpy(), b.numpy(), L.counts_tensor("cpu").numpy()


def _rounded(x):
    return x.to(torch.bfloat16).double().numpy()


SPLIT = 1e-5   # dz carried as hi + lo bf16: |error| <= 2^-18 of each term, plus fp32 summation


def _split_slack(xn, idx, w, b, counts, dyn, kind, act):
    """Per-element allowance of the split-precision backward: SPLIT * the sum of the magnitudes of the
    terms of each dX and dW element (float64, from the Mode-A tensors of the layer)."""
    x = torch.from_numpy(np.asarray(xn))
    G = idx.shape[0]
    idx_f = torch.from_numpy(np.asarray(idx)).reshape(-1, 8).long()
    w_f = torch.from_numpy(np.asarray(w)).reshape(-1, 8)
    b_f = torch.from_numpy(np.asarray(b)).reshape(-1)
    per = idx_f.shape[0] // G
    grp = torch.arange(idx_f.shape[0]) // per
    valid = (torch.arange(idx_f.shape[0]) % per) < torch.from_numpy(np.asarray(counts)).long()[grp]
    z = b_f[None, :] + (w_f[None, :, :] * x[:, idx_f]).sum(-1)
    dact = {"relu": (z > 0).double(), "identity": torch.ones_like(z),
            "gelu": 0.5 * (1 + torch.erf(z / 2 ** 0.5)) + z * torch.exp(-0.5 * z * z) / (2 * np.pi) ** 0.5}[act]
    c1 = torch.from_numpy(np.asarray(dyn))[:, grp]
    if kind == "mean":
        c1 = c1 / torch.from_numpy(np.asarray(counts)).double()[grp][None, :]
    adz = (c1 * dact).abs() * valid[None, :]
    mdx = torch.zeros_like(x)
    for k in range(8):
        mdx.index_add_(1, idx_f[:, k], adz * w_f[:, k].abs()[None, :])
    mdw = (adz[:, :, None] * x[:, idx_f].abs()).sum(0)
    return SPLIT * mdx.numpy(), SPLIT * mdw.numpy()


def _tc_forward(lay, x, tokens=0, winners=False):
    L = lay.layout
    pool = {"mean": _native.POOL_MEAN, "sum": _native.POOL_SUM, "max": _native.POOL_MAX}[lay.cfg.levels[0].type]
    pre = torch.empty(x.shape[0], L.groups, device="cuda")
    win = torch.full((x.shape[0], L.groups), -7, device="cuda", dtype=torch.int32) if winners else None
    _native.fwd_shared_tc(x, lay.indices, lay.weight.detach(), lay.bias.detach(), L.counts_tensor("cuda"), pre,
                          L.blocks_per_group, L.block, 0, L.groups, pool,
                          _native.ACT_IDS[lay.cfg.levels[0].activation], tokens=tokens, winners=win)
    torch.cuda.synchronize()
    return pre, win


@pytest.mark.parametrize("C", [8, 16, 32, 64])
@pytest.mark.parametrize("pool,act", [("mean", "relu"), ("sum", "identity"), ("max", "identity"),
                                      ("mean", "gelu"), ("max", "relu")])
@pytest.mark.parametrize("D", [512, 4096])
def test_forward_against_oracle(C, pool, act, D):
    G, B = 7, 37
    H = G * 64 * C * 3 - 5 * C - 3          # ragged groups: padding slots inside the last quad
    lay = _layer(C, {"type": pool, "activation": act}, D, H, G, seed=C + D)
    gen = torch.Generator().manual_seed(C)
    x = torch.randn(B, D, generator=gen)
    pre, win = _tc_forward(lay, x.cuda(), winners=pool == "max")
    L, idx, w, b, counts = _oracle_params(lay)
    xn = _rounded(x)
    if pool == "max":
        ref, rwin = P.max_forward(xn, idx, w, b, counts, act)
        assert_close(pre.cpu(), ref, what="max pre", **FWD)
        assert torch.equal(win.cpu(), torch.from_numpy(np.asarray(rwin)).to(torch.int32)), "max winners"
    else:
        ref = O.forward(xn, idx, w, b, counts, pool, act)
        if pool == "sum":   # compare per neuron: the fp32 error of a sum grows with the group size
            n = torch.from_numpy(counts).double()
            pre, ref = pre.cpu().double() / n, torch.from_numpy(np.asarray(ref)) / n
        assert_close(pre.cpu(), ref, what=f"{pool} pre", **FWD)


@pytest.mark.parametrize("C", [8, 64])
@pytest.mark.parametrize("pool", ["mean", "max"])
def test_token_tile_does_not_change_the_output(C, pool):
    D, H, G, B = 1024, 40000, 5, 70
    lay = _layer(C, pool, D, H, G, seed=9)
    x = torch.randn(B, D, generator=torch.Generator().manual_seed(2)).cuda()
    outs = [_tc_forward(lay, x, tokens=t, winners=pool == "max") for t in (16, 32, 64)]
    for pre, win in outs[1:]:
        assert torch.equal(pre, outs[0][0])
        if pool == "max":
            assert torch.equal(win, outs[0][1])


def _layer_grads_against_oracle(lay, B, seed=5):
    """Forward + backward of a bf16 layer against the float64 oracle on x rounded to bf16."""
    D, G = lay.layout.input_dim, lay.layout.groups
    lay.enable_main_grad()
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(B, D, generator=gen)
    dy = torch.randn(B, G, generator=gen)
    xg = x.cuda().requires_grad_(True)
    y = lay(xg)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    assert lay.last_info["forward_kernel"].startswith("gl_fwd_shared_tc")
    L, idx, w, b, counts = _oracle_params(lay)
    xn, dyn = _rounded(x), dy.double().numpy()
    kind, act = lay.cfg.levels[0].type, lay.cfg.levels[0].activation
    if kind == "max":
        pre, win = P.max_forward(xn, idx, w, b, counts, act)
        g_pre = dyn * (pre > 0)                                  # default out-activation ReLU
        odx, odw, odb = P.max_backward(xn, idx, w, b, counts, g_pre, act, winner=win)
        y_ref, sdx, sdw, sdb = np.maximum(pre, 0), 0.0, None, None
    else:
        y_ref = O.forward(xn, idx, w, b, counts, kind, act)
        odx, odw, odb, sdx, sdw, sdb = O.backward(xn, idx, w, b, counts, dyn, kind, act, slack=True)
        mdx, mdw = _split_slack(xn, idx, w, b, counts, dyn, kind, act)
        sdx, sdw = np.asarray(sdx) + mdx, np.asarray(sdw).reshape(mdw.shape) + mdw
    shape_w, shape_b = (L.groups, L.blocks_per_group, L.block, 8), (L.groups, L.blocks_per_group, L.block)
    odw = L.pack_weights(torch.from_numpy(np.asarray(odw)).reshape(shape_w))
    odb = L.pack_bias(torch.from_numpy(np.asarray(odb)).reshape(shape_b))
    if sdw is not None:
        sdw = L.pack_weights(torch.from_numpy(np.asarray(sdw)).reshape(shape_w))
        sdb = L.pack_bias(torch.from_numpy(np.asarray(sdb)).reshape(shape_b))
    yv, yr = y.detach().cpu().double(), torch.as_tensor(np.asarray(y_ref))
    if kind == "sum":   # compared per neuron: the fp32 error of a sum grows with the group size
        n = torch.from_numpy(np.asarray(counts)).double()
        yv, yr = yv / n, yr / n
    assert_close(yv, yr, what="y", **FWD)
    assert_close(xg.grad.cpu(), odx, what="dx", slack=sdx, **BWD)
    assert_close(lay.weight.main_grad.cpu(), odw, what="dw", slack=sdw, **BWD)
    assert_close(lay.bias.main_grad.cpu(), odb, what="db", slack=sdb, **BWD)


@pytest.mark.parametrize("C", [8, 16, 32, 64])
@pytest.mark.parametrize("pooling", ["mean", "sum", "max", {"type": "mean", "activation": "gelu"}])
@pytest.mark.parametrize("D", [512, 2048])
def test_layer_gradients_on_rounded_x(C, pooling, D):
    lay = _layer(C, pooling, D, 24000 - 3 * C - 1, 6, seed=C)
    _layer_grads_against_oracle(lay, 45)
    kind = pooling if isinstance(pooling, str) else pooling["type"]
    if kind != "max":
        assert lay.last_info["backward_kernel"] == "gl_bwd_shared_tc"


@pytest.mark.parametrize("C", [8, 16, 64])
@pytest.mark.parametrize("pooling,accum", [("mean", "auto"), ("sum", "auto"), ("mean", "fp32"),
                                           ({"type": "mean", "activation": "gelu"}, "auto"),
                                           ({"type": "sum", "activation": "identity"}, "auto")])
@pytest.mark.parametrize("S,R,B", [(64, 4, 45), (128, 2, 150)])
def test_input_set_backward_against_oracle(C, pooling, accum, S, R, B):
    """Layers with input-supergroup connectivity run the input-set backward (gl_bwd_shared_tc_sets):
    a CTA stages only its set's S rows; the gradients match the oracle as the generic kernel's do,
    with the int32 fixed-point and the fp32 dX tile, over ragged groups and several token tiles."""
    lay = SparsePoolingLayer(1024, 30000 - 5 * C - 3, 7, shared_neurons=C, weight_layout="packed", pooling=pooling,
                             dtype=torch.bfloat16, seed=C + S, bias_std=0.2, connectivity=ConnectivityPlan(S, R, seed=3),
                             plan=PhysicalPlan(b200_dx_accum=accum, cuda_input_supergroup_backend="grouped")).cuda()
    _layer_grads_against_oracle(lay, B, seed=S)
    assert lay.last_info["forward_kernel"] == "gl_fwd_shared_tc_sets"
    assert lay.last_info["backward_kernel"] == "gl_bwd_shared_tc_sets"
    assert lay.last_info["dx_accumulation"].startswith("int32" if accum == "auto" else "fp32")


@pytest.mark.parametrize("mode", ["generic", "auto"])
def test_input_set_layers_take_the_generic_kernel_where_it_fits(mode):
    lay = SparsePoolingLayer(1024, 20000, 5, shared_neurons=8, weight_layout="packed", pooling="mean",
                             dtype=torch.bfloat16, seed=1, connectivity=ConnectivityPlan(64, 4, seed=3),
                             plan=PhysicalPlan(cuda_input_supergroup_backend=mode)).cuda()
    _layer_grads_against_oracle(lay, 33)
    assert lay.last_info["backward_kernel"] == "gl_bwd_shared_tc"


@pytest.mark.parametrize("C", [8, 64])
def test_large_input_dim_sets_and_fallbacks(C):
    """D = 4096: the generic tensor-core backward's tiles do not fit, so "auto" runs the input-set
    backward (S = 256 rows per CTA); the forward still fits its 16-token slab.  Without connectivity
    the same layer's backward falls back to the fp32 kernels on the rounded x."""
    D = 4096
    with_sets = SparsePoolingLayer(D, 40000, 6, shared_neurons=C, weight_layout="packed", pooling="mean",
                                   dtype=torch.bfloat16, seed=7, bias_std=0.2,
                                   connectivity=ConnectivityPlan(256, 2, seed=1)).cuda()
    _layer_grads_against_oracle(with_sets, 40)
    assert with_sets.last_info["forward_kernel"] == "gl_fwd_shared_tc_sets"
    assert with_sets.last_info["backward_kernel"] == "gl_bwd_shared_tc_sets"
    plain = _layer(C, "mean", D, 40000, 6, seed=8)
    _layer_grads_against_oracle(plain, 40)
    assert plain.last_info["backward_kernel"] == "gl_bwd_shared_f32"


def test_plan_off_runs_the_fp32_kernels_on_the_same_rounded_x():
    D, H, G, B = 512, 12000, 4, 9
    x = torch.randn(B, D, generator=torch.Generator().manual_seed(8)).cuda()
    on = _layer(8, "mean", D, H, G, seed=1)
    off = _layer(8, "mean", D, H, G, seed=1, plan=PhysicalPlan(b200_bf16_tensor_cores="off"))
    y_on, y_off = on(x), off(x)
    assert on.last_info["forward_kernel"] == "gl_fwd_shared_tc"
    assert off.last_info["forward_kernel"] == "gl_fwd_shared_f32"
    assert_close(y_on.detach().cpu(), y_off.detach().cpu(), what="tensor cores vs fp32 kernels", **FWD)


def _bwd_tc(lay, x, gpre, tokens, fixed, calls=1):
    L = lay.layout
    w = lay.weight.detach()
    rt = lay._runtime()
    wabsmax = w.reshape(L.groups, -1).abs().amax(1).float().contiguous() if fixed else None
    rowmax = rt.record_rowmax() if fixed else None
    dx = torch.zeros(x.shape, device="cuda")
    dw = torch.zeros(lay.weight.shape, device="cuda")
    db = torch.zeros(lay.bias.shape, device="cuda")
    for _ in range(calls):
        _native.bwd_shared_tc(x, lay.indices, w, lay.bias.detach(), L.counts_tensor("cuda"), gpre, dx, dw, db,
                              L.blocks_per_group, L.block, 0, L.groups, _native.POOL_MEAN, _native.ACT_IDS["relu"],
                              tokens=tokens, wabsmax=wabsmax, rowmax=rowmax)
    torch.cuda.synchronize()
    return dx.cpu(), dw.cpu(), db.cpu()


@pytest.mark.parametrize("C", [8, 64])
def test_backward_tiles_and_dx_accumulation_agree(C):
    """Token tiles 16 and 32, with the fp32-atomic and the int32 fixed-point dX tile, give the same
    gradients within the dX tolerance; a second call adds the same amounts again (accumulation)."""
    D, H, G, B = 1024, 30000, 5, 50
    lay = _layer(C, "mean", D, H, G, seed=3)
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(B, D, generator=gen).cuda()
    gpre = torch.randn(B, G, generator=gen).cuda()
    ref = _bwd_tc(lay, x, gpre, 32, False)
    for tokens, fixed in ((16, False), (32, True), (16, True)):
        out = _bwd_tc(lay, x, gpre, tokens, fixed)
        for name, u, v in zip(("dx", "dw", "db"), out, ref):
            assert_close(u, v, what=f"{name} tokens={tokens} fixed={fixed}", **BWD)
    twice = _bwd_tc(lay, x, gpre, 32, True, calls=2)
    for name, u, v in zip(("dx", "dw", "db"), twice, ref):
        assert_close(u, 2 * v, what=f"{name} twice", **BWD)


def test_layer_uses_fixed_point_tile_and_fp32_on_request():
    D, H, G, B = 512, 16000, 4, 20
    x = torch.randn(B, D, generator=torch.Generator().manual_seed(6)).cuda()
    for accum, want in (("auto", "int32 fixed point"), ("fp32", "fp32 atomics")):
        lay = _layer(8, "mean", D, H, G, seed=2, plan=PhysicalPlan(b200_dx_accum=accum))
        lay(x.clone().requires_grad_(True)).sum().backward()
        assert lay.last_info["backward_kernel"] == "gl_bwd_shared_tc"
        assert lay.last_info["dx_accumulation"].startswith(want)


def test_fixed_point_nan_token():
    """A non-finite coefficient makes its token's dx row NaN; the other tokens are unaffected."""
    D, H, G, B = 512, 16000, 4, 20
    lay = _layer(8, "mean", D, H, G, seed=5)
    gen = torch.Generator().manual_seed(7)
    x = torch.randn(B, D, generator=gen).cuda()
    gpre = torch.randn(B, G, generator=gen).cuda()
    clean = _bwd_tc(lay, x, gpre, 32, True)
    gpre[3, 1] = float("nan")
    dx, _, _ = _bwd_tc(lay, x, gpre, 32, True)
    assert torch.isnan(dx[3]).all()
    keep = torch.arange(B) != 3
    assert torch.isfinite(dx[keep]).all()
    # the cross-block fp32 reductions of the fast backward are not bitwise repeatable
    assert_close(dx[keep], clean[0][keep], what="other tokens", **BWD)
