"""bf16 parameters (the reference's default layer dtype, layer.py:43) on the GPU: the kernels read
bf16 weights and biases, compute in fp32 and write fp32 gradients, so a bf16 layer matches the
float64 oracle evaluated on its exact bf16 values (forward rtol 1e-5 / atol 1e-6; dX, dW, db rtol
1e-4 / atol 1e-5 on the fp32 main_grad; like the reference's, a bf16 layer computes on x rounded to
bf16 (autograd.py:349-354), and the oracle sees the same rounded x); the fused Adam updates bf16 parameters and moments as the
reference's optimizer does (optim.py:26-126)."""
import numpy as np
import pytest
import torch

from conftest import assert_close, modeb_as_mode_a
from granulelayer_b200 import FusedAdamW, SparsePoolingLayer, _native
from oracle import oracle as O
from oracle import pool_oracle as P

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def _oracle_params(lay):
    L = lay.layout
    idx, w, b = lay.indices.cpu(), lay.weight.detach().cpu().double(), lay.bias.detach().cpu().double()
    if L.shared_indices:
        idx, w, b = modeb_as_mode_a(L, idx, w, b)
    return L, idx.numpy(), w.numpy(), b.numpy(), L.counts_tensor("cpu").numpy()


def _to_layout(L, dw, db):
    dwc = torch.from_numpy(np.asarray(dw)).reshape(L.groups, L.blocks_per_group, L.block, 8)
    dbc = torch.from_numpy(np.asarray(db)).reshape(L.groups, L.blocks_per_group, L.block)
    if L.packed:
        return L.pack_weights(dwc), L.pack_bias(dbc)
    return dwc, dbc


@pytest.mark.parametrize("C,packed", [(None, False), (8, True), (64, False)])
@pytest.mark.parametrize("pooling", ["mean", "max", {"type": "topk_mean", "k": 4},
                                     {"type": "logmeanexp", "temperature": 0.5}])
def test_bf16_layers_against_oracle(C, packed, pooling):
    D, H, G, B = 512, 20000, 10, 29
    lay = SparsePoolingLayer(D, H, G, shared_neurons=C, weight_layout="packed" if packed else "canonical",
                             pooling=pooling, dtype=torch.bfloat16, seed=4, bias_std=0.2).cuda()
    assert lay.weight.dtype == torch.bfloat16
    lay.enable_main_grad()
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(B, D, generator=gen)
    dy = torch.randn(B, G, generator=gen)
    xg = x.cuda().requires_grad_(True)
    y = lay(xg)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    L, idx, w, b, counts = _oracle_params(lay)
    kind = pooling if isinstance(pooling, str) else pooling["type"]
    act = lay.cfg.levels[0].activation
    xn, dyn = x.numpy().astype(np.float64), dy.numpy().astype(np.float64)
    xn = x.to(torch.bfloat16).double().numpy()   # a bf16 layer computes on x rounded to bf16
    if kind == "mean":
        pre = O.forward(xn, idx, w, b, counts, "mean", act)
        odx, odw, odb, sdx, sdw, sdb = O.backward(xn, idx, w, b, counts, dyn, "mean", act, slack=True)
        y_ref = pre
    elif kind == "max":
        pre, win = P.max_forward(xn, idx, w, b, counts, act)
        g_pre = dyn * (pre > 0)                                  # default out-activation ReLU
        odx, odw, odb = P.max_backward(xn, idx, w, b, counts, g_pre, act, winner=win)
        y_ref, sdx, sdw, sdb = np.maximum(pre, 0), 0.0, 0.0, 0.0
    elif kind == "topk_mean":
        y_ref, slots = P.topk_forward(xn, idx, w, b, counts, 4, act)
        odx, odw, odb = P.topk_backward(xn, idx, w, b, counts, dyn, 4, act, slots=slots)
        sdx = sdw = sdb = 0.0
    else:
        y_ref = P.smooth_forward(xn, idx, w, b, counts, kind, act, tau=0.5)
        odx, odw, odb = P.smooth_backward(xn, idx, w, b, counts, dyn, kind, act, tau=0.5)
        sdx = sdw = sdb = 0.0
    odw, odb = _to_layout(L, odw, odb)
    if not np.isscalar(sdw):
        sdw, sdb = _to_layout(L, sdw, sdb)
    assert_close(y.detach().cpu(), y_ref, what="y", **FWD)
    assert_close(xg.grad.cpu(), odx, what="dx", slack=sdx, **BWD)
    assert_close(lay.weight.main_grad.cpu(), odw, what="dw", slack=sdw, **BWD)
    assert_close(lay.bias.main_grad.cpu(), odb, what="db", slack=sdb, **BWD)


def test_bf16_grad_without_main_grad_is_bf16():
    lay = SparsePoolingLayer(256, 6000, 4, shared_neurons=8, pooling="mean", dtype=torch.bfloat16, seed=1).cuda()
    lay(torch.randn(8, 256).cuda()).sum().backward()
    assert lay.weight.grad.dtype == torch.bfloat16 and lay.bias.grad.dtype == torch.bfloat16


def _torch_adam(p, g, m, v, lr, b1, b2, eps, wd, t):
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    upd = (m / (1 - b1 ** t)) / (torch.sqrt(v / (1 - b2 ** t)) + eps)
    return p * (1 - lr * wd) - lr * upd, m, v


def test_adam_bf16_moments_and_master_weights():
    """moments="bf16", master_weights=True: the update runs in fp32 on the master copy; moments and
    the parameter are stored rounded to nearest (optim.py:47-53)."""
    n = 1 << 16
    gen = torch.Generator().manual_seed(0)
    p0 = torch.randn(n, generator=gen).bfloat16().cuda()
    p = torch.nn.Parameter(p0.clone())
    opt = FusedAdamW([p], lr=1e-3, weight_decay=0.1, moments="bf16", master_weights=True)
    master = p0.float().clone()
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    for t in range(1, 4):
        g = torch.randn(n, generator=gen).cuda()
        p.main_grad = g.clone()
        opt.step()
        master, m, v = _torch_adam(master, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.1, t)
        m, v = m.bfloat16().float(), v.bfloat16().float()
        assert float(p.main_grad.abs().max()) == 0.0
    st = opt.state[p]
    assert st["m"].dtype == torch.bfloat16 and st["master"].dtype == torch.float32
    # the bf16 moments of the emulation and of the kernel may round a near-tie differently (the
    # kernel forms 1 - beta in fp32): one bf16 ulp of m or v moves an update by ~0.4% of lr
    assert torch.allclose(st["master"], master, rtol=1e-5, atol=3 * 1e-3 * 2 ** -8)
    assert torch.equal(p.detach(), st["master"].bfloat16())
    for name, ref in (("m", m), ("v", v)):
        # the kernel and the emulation may round near-ties differently (the kernel forms 1 - beta in
        # fp32 and may contract to FMA), and a one-ulp difference propagates through the next steps'
        # cancellations: check that they agree on average far below an ulp and nowhere by more than
        # a few ulps of the moment's scale
        diff = (st[name].float() - ref).abs()
        scale = float(ref.abs().mean())
        assert float(diff.mean()) < 2 ** -10 * scale, name
        assert float(diff.max()) <= 2 ** -5 * float(ref.abs().max()), name


def test_adam_bf16_stochastic_rounding_is_unbiased():
    """Without a master copy a bf16 parameter is rounded stochastically (optim.py:55-62): updates far
    below half an ulp move the mean by the fp32 amount, where rounding to nearest would not move it."""
    n = 1 << 20
    p = torch.nn.Parameter(torch.ones(n, dtype=torch.bfloat16, device="cuda"))
    opt = FusedAdamW([p], lr=1e-4, moments="fp32")             # |update| = lr = 1e-4 < ulp(1)/2 = 3.9e-3
    p.main_grad = torch.ones(n, device="cuda")
    opt.step()
    mean = float(p.detach().float().mean())
    assert abs(mean - (1.0 - 1e-4)) < 2e-5
    vals = set(torch.unique(p.detach().float()).tolist())
    assert vals <= {1.0, float(torch.tensor(1.0 - 2 ** -8))}   # truncation towards one of the two neighbours
    q = torch.nn.Parameter(torch.ones(n, dtype=torch.bfloat16, device="cuda"))
    opt2 = FusedAdamW([q], lr=1e-4, moments="fp32", stochastic_rounding=False)
    q.main_grad = torch.ones(n, device="cuda")
    opt2.step()
    assert float(q.detach().float().mean()) == 1.0
