"""K16/C16 kernels of the Cover-TopK/16 layer with fp32 parameters on the GPU against the float64 K/C
oracle (restating experimental/reference.py:7-27; pinned to the reference's own outputs in
test_kc_oracle.py), for both kernel families: the tensor-core kernels on three-term bf16 splits
(gl_k16_*_tc_f32, "tc", the default) and the fp32 SIMT kernels (gl_k16_*_f32, "simt",
``b200_f32_tensor_cores="off"``).  Tolerances: forward rtol 1e-5 / atol 1e-6; dx, dw, db rtol 1e-4 /
atol 1e-5, plus the oracle's per-element allowance for pre-activations on ReLU's jump."""
import dataclasses

import numpy as np
import pytest
import torch

from conftest import assert_close
from granulelayer_b200 import _native
from granulelayer_b200.config import PhysicalPlan
from granulelayer_b200.cover_topk16 import CoverTopK16Layer
from granulelayer_b200.kgen import KLayout, init_envelope_parameters
from granulelayer_b200.supergroups import ConnectivityPlan
from oracle import kc_oracle
from test_kc_oracle import _fixture, fixture_layer

pytestmark = pytest.mark.gpu

FWD_TOL = dict(rtol=1e-5, atol=1e-6)
GRAD_TOL = dict(rtol=1e-4, atol=1e-5)


KERNELS = ["tc", "simt"]
NAMES = {"tc": ("gl_k16_fwd_tc_f32", "gl_k16_bwd_tc_f32"), "simt": ("gl_k16_fwd_f32", "gl_k16_bwd_f32")}


def _plan(kernels):
    return PhysicalPlan(grad_precision="split", b200_f32_tensor_cores="auto" if kernels == "tc" else "off")


def _layer(D, H, G, R, seed=1, bias_std=0.1, device="cuda", kernels="tc"):
    w, b = init_envelope_parameters(KLayout(D, H, G, 64, 256), device, dtype=torch.bfloat16, seed=seed,
                                    bias_std=bias_std)
    return CoverTopK16Layer.from_envelope(w, b, input_dim=D, hidden_dim=H, output_dim=G,
                                          connectivity=ConnectivityPlan(64, R, seed=seed + 3), device=device,
                                          plan=_plan(kernels))


def _host(lay):
    return (lay.indices.cpu().numpy(), lay.weight.detach().cpu().numpy(), lay.bias.detach().cpu().numpy(),
            lay.counts.cpu().numpy())


def _check_layer(lay, x, gy, act="relu"):
    xg = x.cuda().requires_grad_(True)
    y = lay(xg)
    y.backward(gy.cuda())
    kernels = "tc" if lay.tensor_cores else "simt"
    assert (lay.last_info["forward_kernel"], lay.last_info["backward_kernel"]) == NAMES[kernels]
    idx, w, b, counts = _host(lay)
    ry, rdx, rdw, rdb, (sdx, sdw, sdb) = kc_oracle.grads(x.numpy(), idx, w, b, counts, gy.numpy(), act=act,
                                                         slack=True)
    assert_close(y.detach(), ry, what="y", **FWD_TOL)
    assert_close(xg.grad, rdx, what="dx", slack=sdx, **GRAD_TOL)
    assert_close(lay.weight.grad, rdw, what="dw", slack=sdw, **GRAD_TOL)
    assert_close(lay.bias.grad, rdb, what="db", slack=sdb, **GRAD_TOL)


@pytest.mark.parametrize("kernels", KERNELS)
def test_reference_fixture(kernels):
    """The reference's own layer and float64 outputs, end to end through the layer."""
    _, a = _fixture()
    lay = fixture_layer("cuda")
    lay.plan = dataclasses.replace(lay.plan, b200_f32_tensor_cores="auto" if kernels == "tc" else "off")
    x = torch.from_numpy(a["x"]).cuda().requires_grad_(True)
    y = lay(x)
    y.backward(torch.from_numpy(a["gy"]).cuda())
    assert_close(y.detach(), a["y"], what="y", **FWD_TOL)
    assert_close(x.grad, a["dx"], what="dx", **GRAD_TOL)
    assert_close(lay.weight.grad, a["dw"], what="dw", **GRAD_TOL)
    assert_close(lay.bias.grad, a["db"], what="db", **GRAD_TOL)
    assert lay.last_info["forward_backend"] == "b200-k16"
    assert (lay.last_info["forward_kernel"], lay.last_info["backward_kernel"]) == NAMES[kernels]


@pytest.mark.parametrize("shape", [(512, 20000, 16, 16), (256, 6000, 4, 8), (1024, 50688, 24, 16)])
@pytest.mark.parametrize("B", [1, 37, 300])
@pytest.mark.parametrize("kernels", KERNELS)
def test_random_layers(shape, B, kernels):
    D, H, G, R = shape
    lay = _layer(D, H, G, R, kernels=kernels)
    gen = torch.Generator().manual_seed(B + D)
    x = torch.randn(B, D, generator=gen)
    gy = torch.randn(B, G, generator=gen)
    _check_layer(lay, x, gy)


@pytest.mark.parametrize("kernels", KERNELS)
def test_config4_shape_slice(kernels):
    """Config-4 geometry (D = 4096, 24,576 neurons per output, S = 64, R = 64) on 8 outputs, batch 512."""
    lay = _layer(4096, 8 * 24576, 8, 64, seed=3, kernels=kernels)
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(512, 4096, generator=gen)
    gy = torch.randn(512, 8, generator=gen)
    _check_layer(lay, x, gy)


@pytest.mark.parametrize("tokens", [(64, 32), (128, 96), (192, 128)])
def test_token_chunks_and_identity(tokens):
    """Explicit token chunks (forward: multiples of 64, backward: of 32) over a ragged batch of 200."""
    ftok, btok = tokens
    lay = _layer(512, 20000, 16, 16)
    sched = lay._work()
    gen = torch.Generator().manual_seed(ftok + btok)
    B = 200
    x = torch.randn(B, 512, generator=gen)
    gy = torch.randn(B, 16, generator=gen)
    idx, w, b, counts = _host(lay)
    NB16 = lay.layout.blocks_per_group
    for act_name, act in (("relu", 1), ("identity", 0)):
        ry, rdx, rdw, rdb, (sdx, sdw, sdb) = kc_oracle.grads(x.numpy(), idx, w, b, counts, gy.numpy(),
                                                             act=act_name, slack=True)
        xc = x.cuda()
        pre = torch.zeros(B, 16, device="cuda")
        _native.k16_fwd(xc, sched, lay.weight.detach(), lay.bias.detach(), lay.counts, pre, NB16, act=act,
                        tokens=ftok)
        c1t = (gy.cuda() / lay.counts_f[None]).t().contiguous()
        dx = torch.zeros_like(xc)
        dw = torch.zeros_like(lay.weight.detach())
        db = torch.zeros_like(lay.bias.detach())
        _native.k16_bwd(xc, sched, lay.weight.detach(), lay.bias.detach(), lay.counts, c1t, dx, dw, db, NB16,
                        act=act, tokens=btok)
        assert_close(pre, ry, what=f"y {act_name}", **FWD_TOL)
        assert_close(dx, rdx, what=f"dx {act_name}", slack=sdx, **GRAD_TOL)
        assert_close(dw, rdw, what=f"dw {act_name}", slack=sdw, **GRAD_TOL)
        assert_close(db, rdb, what=f"db {act_name}", slack=sdb, **GRAD_TOL)


@pytest.mark.parametrize("tiles", [(32, 32, False), (64, 64, True), (128, 32, True), (128, 64, False),
                                   (128, 128, True), (64, 128, False)])
def test_split_token_tiles_and_identity(tiles):
    """The split tensor-core entries at explicit token tiles (32, 64, 128) with the int32 fixed-point or the
    fp32 dX tile, ReLU and identity, over a ragged batch of 200, against the oracle."""
    ftok, btok, fixed = tiles
    lay = _layer(512, 20000, 16, 16)
    sched = lay._work()
    gen = torch.Generator().manual_seed(ftok + btok)
    B = 200
    x = torch.randn(B, 512, generator=gen)
    gy = torch.randn(B, 16, generator=gen)
    idx, w, b, counts = _host(lay)
    NB16 = lay.layout.blocks_per_group
    wd, bd = lay.weight.detach(), lay.bias.detach()
    wabsmax = wd.reshape(16, -1).abs().amax(1).contiguous() if fixed else None
    rowmax = lay._bucket_rowmax() if fixed else None
    for act_name, act in (("relu", 1), ("identity", 0)):
        ry, rdx, rdw, rdb, (sdx, sdw, sdb) = kc_oracle.grads(x.numpy(), idx, w, b, counts, gy.numpy(),
                                                             act=act_name, slack=True)
        xc = x.cuda()
        pre = torch.zeros(B, 16, device="cuda")
        assert _native.k16_fwd(xc, sched, wd, bd, lay.counts, pre, NB16, act=act, tokens=ftok,
                               tensor_cores=True) == "gl_k16_fwd_tc_f32"
        c1t = (gy.cuda() / lay.counts_f[None]).t().contiguous()
        dx = torch.zeros_like(xc)
        dw = torch.zeros_like(wd)
        db = torch.zeros_like(bd)
        assert _native.k16_bwd(xc, sched, wd, bd, lay.counts, c1t, dx, dw, db, NB16, act=act, tokens=btok,
                               wabsmax=wabsmax, rowmax=rowmax, tensor_cores=True) == "gl_k16_bwd_tc_f32"
        assert_close(pre, ry, what=f"y {act_name}", **FWD_TOL)
        assert_close(dx, rdx, what=f"dx {act_name}", slack=sdx, **GRAD_TOL)
        assert_close(dw, rdw, what=f"dw {act_name}", slack=sdw, **GRAD_TOL)
        assert_close(db, rdb, what=f"db {act_name}", slack=sdb, **GRAD_TOL)


def test_split_terms_reproduce_fp32_products():
    """Weights and inputs whose products need all of fp32's 24 significand bits (1 + 2^-23 multiples):
    the split kernels keep them, a one-term bf16 product would lose them."""
    lay = _layer(256, 6000, 4, 8, bias_std=0.0)
    with torch.no_grad():
        lay.weight.mul_(1 + 2.0 ** -23).add_(torch.sign(lay.weight) * 2.0 ** -20)
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(64, 256, generator=gen) * (1 + 2.0 ** -22)
    _check_layer(lay, x, torch.randn(64, 4, generator=gen))


@pytest.mark.parametrize("kernels", KERNELS)
def test_main_grad_accumulates(kernels):
    lay = _layer(256, 6000, 4, 8, kernels=kernels)
    lay.enable_main_grad()
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(64, 256, generator=gen).cuda()
    gy = torch.randn(64, 4, generator=gen).cuda()
    lay(x).backward(gy)
    w1, b1 = lay.weight.main_grad.clone(), lay.bias.main_grad.clone()
    assert lay.weight.grad is None
    lay(x).backward(gy)
    assert_close(lay.weight.main_grad, 2 * w1.double(), rtol=1e-5, atol=1e-7, what="main_grad w")
    assert_close(lay.bias.main_grad, 2 * b1.double(), rtol=1e-5, atol=1e-7, what="main_grad b")


@pytest.mark.parametrize("kernels", KERNELS)
def test_padding_slots_get_no_gradient(kernels):
    lay = _layer(256, 6000, 4, 8, kernels=kernels)   # 1500 neurons per output: the last 16-record is partly padding
    x = torch.randn(32, 256).cuda()
    lay(x).sum().backward()
    L = lay.layout
    s = torch.arange(L.blocks_per_group * 16, device="cuda")
    pad = (s[None, :] >= lay.counts[:, None]).view(L.groups, L.blocks_per_group, 16)
    assert bool(pad.any())
    assert float(lay.weight.grad[pad].abs().max()) == 0.0
    assert float(lay.bias.grad[pad].abs().max()) == 0.0


def test_bad_arguments_are_rejected_before_launch():
    lay = _layer(256, 6000, 4, 8)
    sched = dict(lay._work())
    NB16 = lay.layout.blocks_per_group
    x = torch.randn(8, 256, device="cuda")
    pre = torch.zeros(8, 4, device="cuda")
    w, b = lay.weight.detach(), lay.bias.detach()
    bad = dict(sched, env=torch.zeros(lay.env.numel() + 1, dtype=torch.uint8, device="cuda")[1:])
    with pytest.raises(_native.NativeLibraryError, match="align"):
        _native.k16_fwd(x, bad, w, b, lay.counts, pre, NB16)
    with pytest.raises(_native.NativeLibraryError):
        _native.k16_fwd(x, sched, w, b, lay.counts, pre, NB16, act=2)     # GELU is not built for K16
    with pytest.raises(_native.NativeLibraryError):
        _native.k16_fwd(x, sched, w, b, lay.counts, pre, NB16, tokens=48)  # not a multiple of 64
    _native.k16_fwd(x[:0], sched, w, b, lay.counts, pre[:0], NB16)         # empty batch: no work
    with pytest.raises(_native.NativeLibraryError):
        _native.k16_fwd(x, sched, w, b, lay.counts, pre, NB16, tokens=48, tensor_cores=True)  # 32, 64 or 128
    with pytest.raises(_native.NativeLibraryError, match="align"):
        _native.k16_fwd(x, bad, w, b, lay.counts, pre, NB16, tensor_cores=True)
    with pytest.raises(ValueError):
        _native.k16_bwd(x, sched, w, b, lay.counts, pre.t().contiguous(), x.clone(), w.clone(), b.clone(), NB16,
                        wabsmax=w.reshape(4, -1).abs().amax(1), rowmax=lay._bucket_rowmax())   # SIMT: no bounds
    _native.k16_fwd(x[:0], sched, w, b, lay.counts, pre[:0], NB16, tensor_cores=True)
