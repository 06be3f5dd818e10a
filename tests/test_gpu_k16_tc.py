"""The Cover-TopK/16 layer with bf16 parameters on the tensor cores (gl_k16_fwd_tc / gl_k16_bwd_tc):
the reference's kgen arithmetic -- bf16 parameters, x rounded to bf16, exact bf16 products summed in
fp32, the backward's dz carried as hi + lo bf16 ("split" precision).  Checked against the float64 K/C
oracle (experimental/reference.py:7-27) evaluated on the rounded x and the bf16 parameters: forward
rtol 1e-5 / atol 1e-6; dx, dw, db rtol 1e-4 / atol 1e-5 plus the oracle's ReLU-boundary allowance and
the split-precision allowance (1e-5 of the sum of the magnitudes of each element's terms; the split dz
errs by at most 2^-18 of each term)."""
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
GRAD_TOL = dict(rtol=1e-4, atol=1e-5)
SPLIT = 1e-5


def _layer(D, H, G, R, seed=1, bias_std=0.1):
    w, b = init_envelope_parameters(KLayout(D, H, G, 64, 256), "cuda", dtype=torch.bfloat16, seed=seed,
                                    bias_std=bias_std)
    return CoverTopK16Layer.from_envelope(w, b, input_dim=D, hidden_dim=H, output_dim=G,
                                          connectivity=ConnectivityPlan(64, R, seed=seed + 3), device="cuda",
                                          dtype=torch.bfloat16)


def _split_slack(x, idx, w, b, counts, gy):
    """SPLIT * the magnitude sums of the terms of every dx and dw element (float64)."""
    x = torch.from_numpy(x).double()
    G, NB = idx.shape[:2]
    fi = torch.from_numpy(idx).long().reshape(-1, 16)                  # [F, 16] features
    wf = torch.from_numpy(w).double().reshape(-1, 16, 16)              # [F, n, k]
    bf = torch.from_numpy(b).double().reshape(-1, 16)
    grp = torch.arange(fi.shape[0]) // NB
    slot = (torch.arange(fi.shape[0]) % NB)[:, None] * 16 + torch.arange(16)[None, :]
    valid = slot < torch.from_numpy(counts).long()[grp][:, None]        # [F, 16]
    xg = x[:, fi]                                                       # [B, F, 16 k]
    z = bf[None] + torch.einsum("fnk,bfk->bfn", wf, xg)
    c1 = torch.from_numpy(gy).double()[:, grp] / torch.from_numpy(counts).double()[grp][None]
    adz = (c1[:, :, None] * (z > 0).double()).abs() * valid[None]       # [B, F, n]
    mdx = torch.zeros_like(x)
    contrib = torch.einsum("bfn,fnk->bfk", adz, wf.abs())               # [B, F, k]
    mdx.index_add_(1, fi.reshape(-1), contrib.reshape(x.shape[0], -1))
    mdw = torch.einsum("bfn,bfk->fnk", adz, xg.abs())
    return SPLIT * mdx.numpy(), SPLIT * mdw.reshape(w.shape).numpy()


def _check(lay, x, gy):
    """Forward and backward against the oracle; the gradients are read from the fp32 main_grad (a bf16
    parameter's .grad is its gradient rounded to bf16, as the reference returns it)."""
    lay.enable_main_grad()
    lay.zero_main_grad()
    xg = x.cuda().requires_grad_(True)
    y = lay(xg)
    y.backward(gy.cuda())
    torch.cuda.synchronize()
    assert lay.last_info["forward_kernel"] == "gl_k16_fwd_tc"
    assert lay.last_info["backward_kernel"] == "gl_k16_bwd_tc"
    assert lay.last_info["dx_accumulation"] == "int32 fixed point"
    xr = x.to(torch.bfloat16).double().numpy()
    idx = lay.indices.cpu().numpy()
    w = lay.weight.detach().double().cpu().numpy()
    b = lay.bias.detach().double().cpu().numpy()
    counts = lay.counts.cpu().numpy()
    ry, rdx, rdw, rdb, (sdx, sdw, sdb) = kc_oracle.grads(xr, idx, w, b, counts, gy.double().numpy(), act="relu",
                                                         slack=True)
    mdx, mdw = _split_slack(xr, idx, w, b, counts, gy.double().numpy())
    assert_close(y.detach(), ry, what="y", **FWD_TOL)
    assert_close(xg.grad, rdx, what="dx", slack=np.asarray(sdx) + mdx, **GRAD_TOL)
    assert_close(lay.weight.main_grad, rdw, what="dw", slack=np.asarray(sdw).reshape(mdw.shape) + mdw, **GRAD_TOL)
    assert_close(lay.bias.main_grad, rdb, what="db", slack=sdb, **GRAD_TOL)


@pytest.mark.parametrize("shape", [(512, 20000, 16, 16), (256, 6000, 4, 8), (1024, 50688, 24, 16)])
@pytest.mark.parametrize("B", [1, 37, 300])
def test_bf16_layers_against_oracle(shape, B):
    D, H, G, R = shape
    lay = _layer(D, H, G, R)
    assert lay.weight.dtype == torch.bfloat16
    gen = torch.Generator().manual_seed(B + D)
    _check(lay, torch.randn(B, D, generator=gen), torch.randn(B, G, generator=gen))


def test_bf16_config4_shape_slice():
    """Config-4 geometry (D = 4096, 24,576 neurons per output, S = 64, R = 64) on 6 outputs, batch 512."""
    lay = _layer(4096, 6 * 24576, 6, 64, seed=3)
    gen = torch.Generator().manual_seed(3)
    _check(lay, torch.randn(512, 4096, generator=gen), torch.randn(512, 6, generator=gen))


def test_token_tiles_agree():
    """Explicit token tiles of the forward (32, 64, 128) and backward (32, 64, 128), and the backward's
    fp32 and int32 fixed-point dX tiles, give the same results within the tolerances (the order of the
    fp32 atomics differs)."""
    lay = _layer(512, 20000, 16, 16, seed=5)
    sched, L = lay._work(), lay.layout
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(200, 512, generator=gen).to(torch.bfloat16).float().cuda()
    c1t = torch.randn(16, 200, generator=gen).cuda()
    wabsmax = lay.weight.detach().reshape(16, -1).abs().amax(1).float().contiguous()
    rowmax = lay._bucket_rowmax()
    outs = []
    for tok, fixed in ((32, False), (64, False), (128, False), (64, True), (32, True), (128, True)):
        pre = torch.zeros(200, 16, device="cuda")
        _native.k16_fwd(x, sched, lay.weight.detach(), lay.bias.detach(), lay.counts, pre, L.blocks_per_group,
                        tokens=tok)
        dx = torch.zeros_like(x)
        dw = torch.zeros(lay.weight.shape, device="cuda")
        db = torch.zeros(lay.bias.shape, device="cuda")
        _native.k16_bwd(x, sched, lay.weight.detach(), lay.bias.detach(), lay.counts, c1t, dx, dw, db,
                        L.blocks_per_group, tokens=tok, wabsmax=wabsmax if fixed else None,
                        rowmax=rowmax if fixed else None)
        torch.cuda.synchronize()
        outs.append((pre.cpu(), dx.cpu(), dw.cpu(), db.cpu()))
    for o in outs[1:]:
        assert_close(o[0], outs[0][0], what="pre", **FWD_TOL)
        for name, u, v in zip(("dx", "dw", "db"), o[1:], outs[0][1:]):
            assert_close(u, v, what=name, **GRAD_TOL)
