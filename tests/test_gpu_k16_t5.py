"""The Cover-TopK/16 forward on the tcgen05 tensor cores (gl_k16_fwd_t5 for bf16 parameters,
gl_k16_fwd_t5_f32 for fp32 ones on three-term bf16 splits), through the C ABI: against the float64 K/C
oracle (experimental/reference.py:7-27) on the layer's own parameters (x rounded to bf16 for the bf16
layer, as the reference's arithmetic does), and against the mma.sync entries on the same inputs.
Tolerance: forward rtol 1e-5 / atol 1e-6.  No wait for the tensor cores may run out (status 0)."""
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
