"""The Cover-TopK/16 forward and backward on the tcgen05 tensor cores (gl_k16_fwd_t5 / gl_k16_bwd_t5 for
bf16 parameters, gl_k16_fwd_t5_f32 / gl_k16_bwd_t5_f32 for fp32 ones on three-term bf16 splits), through the
C ABI: against the float64 K/C oracle (experimental/reference.py:7-27) on the layer's own parameters (x
rounded to bf16 for the bf16 layer, as the reference's arithmetic does), and against the mma.sync entries
on the same inputs.  Tolerances: forward rtol 1e-5 / atol 1e-6; gradients rtol 1e-4 / atol 1e-5 plus the
oracle's ReLU-boundary allowance and, for bf16 parameters, the split-precision allowance (1e-5 of the sum
of the magnitudes of each element's terms: dz is carried as hi + lo bf16 in dX, dW and db).  No wait for
the tensor cores may run out (status 0)."""
import numpy as np
import pytest
import torch

from conftest import assert_close
from granulelayer_b200 import _native
from granulelayer_b200.cover_topk16 import CoverTopK16Layer
from granulelayer_b200.kgen import KLayout, init_envelope_parameters
from granulelayer_b200.supergroups import ConnectivityPlan
from oracle import kc_oracle

pytestmark = pytest.mark.gpu

FWD_TOL = dict(rtol=1e-5, atol=1e-6)


def _layer(D, H, G, R, dtype, seed=1, bias_std=0.1):
    w, b = init_envelope_parameters(KLayout(D, H, G, 64, 256), "cuda", dtype=torch.bfloat16, seed=seed,
                                    bias_std=bias_std)
    return CoverTopK16Layer.from_envelope(w, b, input_dim=D, hidden_dim=H, output_dim=G,
                                          connectivity=ConnectivityPlan(64, R, seed=seed + 3), device="cuda",
                                          dtype=dtype)


def _forward(lay, x, t5=True):
    sched, L = lay._work(), lay.layout
    pre = torch.zeros(x.shape[0], L.groups, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    w, b = lay.weight.detach(), lay.bias.detach()
    if t5:
        name = _native.k16_fwd_t5(x, sched, w, b, lay.counts, pre, L.blocks_per_group, status=status)
    else:
        name = _native.k16_fwd(x, sched, w, b, lay.counts, pre, L.blocks_per_group, tensor_cores=True)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"{name}: a wait for the tensor cores ran out"
    return pre.cpu(), name


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(512, 20000, 16, 16), (256, 6000, 4, 8), (1024, 50688, 24, 16)])
@pytest.mark.parametrize("B", [1, 37, 300])
def test_t5_forward_against_oracle(shape, B, dtype):
    D, H, G, R = shape
    lay = _layer(D, H, G, R, dtype)
    gen = torch.Generator().manual_seed(B + D)
    x = torch.randn(B, D, generator=gen)
    if dtype == torch.bfloat16:
        x = x.to(torch.bfloat16).float()
    y, name = _forward(lay, x.cuda())
    assert name == ("gl_k16_fwd_t5" if dtype == torch.bfloat16 else "gl_k16_fwd_t5_f32")
    ry = kc_oracle.forward(x.double().numpy(), lay.indices.cpu().numpy(), lay.weight.detach().double().cpu().numpy(),
                           lay.bias.detach().double().cpu().numpy(), lay.counts.cpu().numpy(), act="relu")
    assert_close(y, ry, what="y", **FWD_TOL)
    y_tc, _ = _forward(lay, x.cuda(), t5=False)
    assert_close(y, y_tc, what="y vs mma.sync", **FWD_TOL)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_t5_forward_config4_slice(dtype):
    """Config-4 geometry (D = 4096, 24,576 neurons per output, S = 64, R = 64) on 6 outputs, batch 512."""
    lay = _layer(4096, 6 * 24576, 6, 64, dtype, seed=3)
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(512, 4096, generator=gen)
    if dtype == torch.bfloat16:
        x = x.to(torch.bfloat16).float()
    y, _ = _forward(lay, x.cuda())
    ry = kc_oracle.forward(x.double().numpy(), lay.indices.cpu().numpy(), lay.weight.detach().double().cpu().numpy(),
                           lay.bias.detach().double().cpu().numpy(), lay.counts.cpu().numpy(), act="relu")
    assert_close(y, ry, what="y", **FWD_TOL)


GRAD_TOL = dict(rtol=1e-4, atol=1e-5)
SPLIT = 1e-5


def _backward(lay, x, gy, t5=True):
    sched, L = lay._work(), lay.layout
    w, b = lay.weight.detach(), lay.bias.detach()
    c1t = (gy.cuda() / lay.counts_f[None, :]).t().contiguous()
    dx = torch.zeros_like(x)
    dw = torch.zeros(w.shape, device="cuda")
    db = torch.zeros(b.shape, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    if t5:
        name = _native.k16_bwd_t5(x, sched, w, b, lay.counts, c1t, dx, dw, db, L.blocks_per_group, status=status)
    else:
        name = _native.k16_bwd(x, sched, w, b, lay.counts, c1t, dx, dw, db, L.blocks_per_group, tensor_cores=True)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"{name}: a wait for the tensor cores ran out"
    return dx.cpu(), dw.cpu(), db.cpu(), name


def _split_slack(x, idx, w, b, counts, gy):
    """SPLIT * the magnitude sums of the terms of every dx, dw and db element (float64)."""
    x = torch.from_numpy(x).double()
    NB = idx.shape[1]
    fi = torch.from_numpy(idx).long().reshape(-1, 16)
    wf = torch.from_numpy(w).double().reshape(-1, 16, 16)
    bf = torch.from_numpy(b).double().reshape(-1, 16)
    grp = torch.arange(fi.shape[0]) // NB
    slot = (torch.arange(fi.shape[0]) % NB)[:, None] * 16 + torch.arange(16)[None, :]
    valid = slot < torch.from_numpy(counts).long()[grp][:, None]
    xg = x[:, fi]
    z = bf[None] + torch.einsum("fnk,bfk->bfn", wf, xg)
    c1 = torch.from_numpy(gy).double()[:, grp] / torch.from_numpy(counts).double()[grp][None]
    adz = (c1[:, :, None] * (z > 0).double()).abs() * valid[None]
    mdx = torch.zeros_like(x)
    mdx.index_add_(1, fi.reshape(-1), torch.einsum("bfn,fnk->bfk", adz, wf.abs()).reshape(x.shape[0], -1))
    mdw = torch.einsum("bfn,bfk->fnk", adz, xg.abs())
    mdb = adz.sum(0)
    return SPLIT * mdx.numpy(), SPLIT * mdw.reshape(w.shape).numpy(), SPLIT * mdb.reshape(b.shape).numpy()


def _check_backward(lay, x, gy):
    bf16 = lay.weight.dtype == torch.bfloat16
    if bf16:
        x = x.to(torch.bfloat16).float()
    dx, dw, db, name = _backward(lay, x.cuda(), gy)
    assert name == ("gl_k16_bwd_t5" if bf16 else "gl_k16_bwd_t5_f32")
    xr, idx = x.double().numpy(), lay.indices.cpu().numpy()
    w, b = lay.weight.detach().double().cpu().numpy(), lay.bias.detach().double().cpu().numpy()
    counts = lay.counts.cpu().numpy()
    _, rdx, rdw, rdb, (sdx, sdw, sdb) = kc_oracle.grads(xr, idx, w, b, counts, gy.double().numpy(), act="relu",
                                                        slack=True)
    sdx, sdw, sdb = np.asarray(sdx), np.asarray(sdw).reshape(w.shape), np.asarray(sdb).reshape(b.shape)
    if bf16:
        mdx, mdw, mdb = _split_slack(xr, idx, w, b, counts, gy.double().numpy())
        sdx, sdw, sdb = sdx + mdx, sdw + mdw, sdb + mdb
    assert_close(dx, rdx, what="dx", slack=sdx, **GRAD_TOL)
    assert_close(dw, rdw, what="dw", slack=sdw, **GRAD_TOL)
    assert_close(db, rdb, what="db", slack=sdb, **GRAD_TOL)
    tdx, tdw, tdb, _ = _backward(lay, x.cuda(), gy, t5=False)
    assert_close(dx, tdx, what="dx vs mma.sync", slack=2 * sdx, **GRAD_TOL)
    assert_close(dw, tdw, what="dw vs mma.sync", slack=2 * sdw, **GRAD_TOL)
    assert_close(db, tdb, what="db vs mma.sync", slack=2 * sdb, **GRAD_TOL)
    return dx, dw, db


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(512, 20000, 16, 16), (256, 6000, 4, 8), (1024, 50688, 24, 16)])
@pytest.mark.parametrize("B", [1, 37, 300])
def test_t5_backward_against_oracle(shape, B, dtype):
    D, H, G, R = shape
    lay = _layer(D, H, G, R, dtype)
    gen = torch.Generator().manual_seed(B + D + 1)
    _check_backward(lay, torch.randn(B, D, generator=gen), torch.randn(B, G, generator=gen))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_t5_backward_config4_slice(dtype):
    """Config-4 geometry (D = 4096, 24,576 neurons per output, S = 64, R = 64) on 6 outputs, batch 512."""
    lay = _layer(4096, 6 * 24576, 6, 64, dtype, seed=3)
    gen = torch.Generator().manual_seed(4)
    _check_backward(lay, torch.randn(512, 4096, generator=gen), torch.randn(512, 6, generator=gen))


@pytest.mark.parametrize("mode", ["bwd", "on"])
def test_t5_layer_routing_through_autograd(mode):
    """PhysicalPlan(b200_tcgen05="bwd" | "on") routes the fp32 layer's autograd backward (and, for "on", its
    forward) to the tcgen05 entries; outputs and gradients match the float64 oracle."""
    from granulelayer_b200.config import PhysicalPlan

    D, H, G, R, B = 512, 20000, 16, 16, 200
    w, b = init_envelope_parameters(KLayout(D, H, G, 64, 256), "cuda", dtype=torch.bfloat16, seed=6, bias_std=0.1)
    lay = CoverTopK16Layer.from_envelope(w, b, input_dim=D, hidden_dim=H, output_dim=G,
                                         connectivity=ConnectivityPlan(64, R, seed=9), device="cuda",
                                         plan=PhysicalPlan(grad_precision="split", b200_tcgen05=mode))
    gen = torch.Generator().manual_seed(2)
    x, gy = torch.randn(B, D, generator=gen), torch.randn(B, G, generator=gen)
    xg = x.cuda().requires_grad_(True)
    y = lay(xg)
    y.backward(gy.cuda())
    assert lay.last_info["backward_kernel"] == "gl_k16_bwd_t5_f32"
    assert lay.last_info["forward_kernel"] == ("gl_k16_fwd_t5_f32" if mode == "on" else "gl_k16_fwd_tc_f32")
    assert lay.last_info["dx_accumulation"] == "fp32 in tensor memory"
    ry, rdx, rdw, rdb, (sdx, sdw, sdb) = kc_oracle.grads(
        x.double().numpy(), lay.indices.cpu().numpy(), lay.weight.detach().double().cpu().numpy(),
        lay.bias.detach().double().cpu().numpy(), lay.counts.cpu().numpy(), gy.double().numpy(), act="relu",
        slack=True)
    assert_close(y.detach(), ry, what="y", **FWD_TOL)
    assert_close(xg.grad, rdx, what="dx", slack=sdx, **GRAD_TOL)
    assert_close(lay.weight.grad, rdw, what="dw", slack=sdw, **GRAD_TOL)
    assert_close(lay.bias.grad, rdb, what="db", slack=sdb, **GRAD_TOL)
