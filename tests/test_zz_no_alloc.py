"""The allocation-free deterministic Mode-B backward (gl_bwd_shared_det_static_f32), called through
the C ABI, gives bit for bit the results of gl_bwd_shared_det_f32 (which takes a caller-allocated
int64 dX buffer): both run the same deterministic kernels on the same inputs, so any difference
means the fixed scratch was not fully cleared or was addressed wrongly.  Two calls in a row use
different batch sizes and gradients, so a second call cannot lean on zeros left by the first; fp32
and bf16 parameters are both covered.

It serves callers that cannot allocate device memory where the backward runs (a plugin whose host
framework owns all device memory, a loop that cannot afford cudaMalloc's synchronisation); its
scratch is a fixed array inside the library, so problems beyond B * D = 2^20 are rejected.

This file is named to be collected last: the entry point shares one scratch array per device
across calls, and the test must pass both alone in a fresh process and after every other test."""
import pytest
import torch

from granulelayer_b200 import PhysicalPlan, SparsePoolingLayer, _native

pytestmark = pytest.mark.gpu


def _layer(C=16, packed=True, D=512, H=30000, G=6, dtype=torch.float32):
    return SparsePoolingLayer(D, H, G, shared_neurons=C, weight_layout="packed" if packed else "canonical",
                              pooling={"type": "mean", "activation": "relu"}, dtype=dtype, seed=5,
                              bias_std=0.2, plan=PhysicalPlan(reduction="deterministic")).cuda()


def _inputs(lay, B, seed):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(B, lay.layout.input_dim, generator=gen).cuda()
    gpre = torch.randn(B, lay.layout.groups, generator=gen).cuda()
    return x, gpre


def _run(lay, x, gpre, static):
    """dx, dw, db of one deterministic backward through the C ABI (fresh zeroed outputs)."""
    L, rt = lay.layout, lay._runtime()
    w, b = lay.weight.detach(), lay.bias.detach()
    qscale, qinv = rt.det_scales(w, gpre)
    dx = torch.zeros_like(x)
    dw = torch.zeros(w.shape, device=w.device, dtype=torch.float32)
    db = torch.zeros(b.shape, device=b.device, dtype=torch.float32)
    args = (x, lay.indices, w, b, rt.counts_i32, gpre, dx, dw, db, L.blocks_per_group, L.block, 0, L.groups,
            _native.POOL_MEAN, _native.ACT_IDS["relu"], L.packed)
    if static:
        _native.bwd_shared_det_static(*args, qscale, qinv)
    else:
        dxq = torch.zeros(x.shape, device=x.device, dtype=torch.int64)
        _native.bwd_shared_det(*args, dxq, qscale, qinv)
    torch.cuda.synchronize()
    return dx, dw, db


@pytest.mark.parametrize("C,packed,dtype", [(16, True, torch.float32), (64, False, torch.float32),
                                            (16, True, torch.bfloat16)])
def test_static_scratch_matches_caller_scratch_twice(C, packed, dtype):
    lay = _layer(C, packed, dtype=dtype)
    n0 = _native.launch_count()
    for B, seed in ((37, 1), (96, 2)):      # the second call uses more of the scratch than the first
        x, gpre = _inputs(lay, B, seed)
        want = _run(lay, x, gpre, static=False)
        got = _run(lay, x, gpre, static=True)
        for name, g, e in zip(("dx", "dw", "db"), got, want):
            assert torch.equal(g, e), f"B={B} {name}: max |diff| {float((g - e).abs().max())}"
        assert float(got[0].abs().sum()) > 0
    assert _native.launch_count() - n0 >= 8     # both entry points ran the library's kernels


def test_static_scratch_rejects_oversized_problem():
    lay = _layer(16, True)
    B = _native.DET_STATIC_MAX_ELEMS // lay.layout.input_dim + 1     # B * D just over the fixed scratch
    x, gpre = _inputs(lay, B, 3)
    with pytest.raises(_native.NativeLibraryError, match=r"fixed scratch .*\[-8\]"):
        _run(lay, x, gpre, static=True)
