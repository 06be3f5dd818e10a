"""Parity at the geometry bench.py times (BASELINE configs 2 and 3), against the float64 C oracle.

The benchmarked layer has D = 4096 inputs and groups of n_g = 24,576 neurons; its backward runs the
T = 4 fixed-point dX tile, whose per-group scale depends on the group's largest per-feature record
count (rowmax) and on max |w|, and at B = 1024 the dW / db sums collect 256 token tiles of global
reductions.  These tests run exactly that: slices of whole 24,576-neuron groups at B = 256 and 1024,
with the reference's index rule (distinct, sorted per neuron, layout.py:204-251) and with the
configs' literal rule (uniform with replacement, stored int16 since D = 4096), through

  * the drop-in SparsePoolingLayer with both dX accumulators (int32 fixed point and fp32 atomics);
  * the bench's engine, GroupShardedLayer (bank-ordered storage, single-rank group);
  * the C ABI with 8 groups per thread block, as the full-size launch uses.

Tolerances: forward rtol 1e-5 / atol 1e-6; dX, dW, db rtol 1e-4 / atol 1e-5, plus the oracle's
per-element allowance for (token, neuron) pairs on ReLU's jump."""
import socket

import pytest
import torch

from conftest import assert_close
from granulelayer_b200 import PhysicalPlan, SparsePoolingLayer, _native
from oracle import oracle as O

pytestmark = pytest.mark.gpu

D, NG = 4096, 24576
FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)
_cache = {}


def _params(rule, G, plan=None):
    """A G-group slice of the benchmarked layer on the CPU, seed 1 (config 2)."""
    lay = SparsePoolingLayer(D, G * NG, G, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=1,
                             bias_std=0.1, plan=plan)
    if rule == "uniform":
        gen = torch.Generator().manual_seed(11)
        with torch.no_grad():
            lay.indices.copy_(torch.randint(0, D, lay.indices.shape, generator=gen).to(torch.int16))
    return lay


def _inputs(B, G):
    gen = torch.Generator().manual_seed(100 + B)
    return torch.randn(B, D, generator=gen), torch.randn(B, G, generator=gen)


def _oracle(rule, B, G):
    key = (rule, B, G)
    if key not in _cache:
        lay = _params(rule, G)
        x, dy = _inputs(B, G)
        c = lay.layout.counts_tensor("cpu").numpy()
        args = (x.numpy(), lay.indices.numpy(), lay.weight.detach().numpy(), lay.bias.detach().numpy(), c)
        pre = O.forward(*args)
        dx, dw, db, sdx, sdw, sdb = O.backward(*args, dy.numpy(), slack=True)
        _cache.clear()
        _cache[key] = (pre, dx, dw, db, sdx, sdw, sdb)
    return _cache[key]


def _check(got, want, what):
    y, dx, dw, db = got
    pre, odx, odw, odb, sdx, sdw, sdb = want
    assert_close(y, pre, what=f"{what} y", **FWD)
    assert_close(dx, odx, what=f"{what} dx", slack=sdx, **BWD)
    assert_close(dw, odw, what=f"{what} dw", slack=sdw, **BWD)
    assert_close(db, odb, what=f"{what} db", slack=sdb, **BWD)


def _step(lay, x, dy, canon=None):
    xr = x.cuda().requires_grad_(True)
    y = lay(xr)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    gw, gb = lay.weight.grad, lay.bias.grad
    if canon is not None:
        gw, gb = canon(gw), canon(gb)
    return y.detach().cpu(), xr.grad.cpu(), gw.cpu(), gb.cpu()


@pytest.mark.parametrize("B", [256, 1024])
@pytest.mark.parametrize("rule", ["distinct", "uniform"])
@pytest.mark.parametrize("accum", ["fixed", "fp32"])
def test_layer_at_bench_geometry(rule, B, accum):
    G = 2
    lay = _params(rule, G, PhysicalPlan(b200_dx_accum=accum)).cuda()
    x, dy = _inputs(B, G)
    got = _step(lay, x, dy)
    assert lay.last_info["dx_accumulation"] == ("int32 fixed point" if accum == "fixed" else "fp32 atomics")
    _check(got, _oracle(rule, B, G), f"layer {rule} B={B} {accum}")


def _single_rank_group():
    import torch.distributed as dist

    if not dist.is_initialized():
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        dist.init_process_group("gloo", rank=0, world_size=1, init_method=f"tcp://127.0.0.1:{port}")
    return dist


@pytest.mark.parametrize("B", [256, 1024])
@pytest.mark.parametrize("rule", ["distinct", "uniform"])
def test_bench_engine_shard_at_bench_geometry(rule, B):
    from granulelayer_b200.distributed import GroupShardedLayer

    dist = _single_rank_group()
    try:
        G = 2
        full = _params(rule, G).cuda()
        shard = GroupShardedLayer.from_full(full)
        assert shard.neuron_order is not None
        x, dy = _inputs(B, G)
        got = _step(shard, x, dy, canon=shard.canonical)
        assert shard.input_order is not None, "GPU shards are stored in octet order"
        info = shard.runtime().last_info
        assert (info["forward_kernel"], info["backward_kernel"]) == ("gl_fwd_octet_f32", "gl_bwd_octet_prefix_f32")
        _check(got, _oracle(rule, B, G), f"shard {rule} B={B}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rule", ["distinct", "uniform"])
def test_eight_groups_per_block_at_bench_geometry(rule):
    """The C ABI with 8 groups per thread block (the full-size launch's chunk), B = 1024."""
    G, B = 8, 1024
    lay = _params(rule, G)
    x, dy = _inputs(B, G)
    L = lay.layout
    idx, w, b = lay.indices.cuda(), lay.weight.detach().cuda(), lay.bias.detach().cuda()
    counts = L.counts_tensor("cuda").to(torch.int32)
    xc, gpre = x.cuda(), dy.cuda()      # mean: dL/dpre = dy (the kernel divides by n_g itself)
    NB = L.blocks_per_group
    pre = torch.empty(B, G, device="cuda")
    wabsmax = torch.empty(G, device="cuda")
    _native.fwd(xc, idx, w, b, counts, pre, NB, 0, G, _native.POOL_MEAN, 1, groups_per_cta=8, wabsmax=wabsmax)
    rowmax = torch.empty(G, device="cuda", dtype=torch.int32)
    _native.group_index_maxcount(idx, counts, D, NB, 0, G, rowmax)
    dx = torch.zeros(B, D, device="cuda")
    dw, db = torch.zeros_like(w), torch.zeros_like(b)
    _native.bwd(xc, idx, w, b, counts, gpre, dx, dw, db, NB, 0, G, _native.POOL_MEAN, 1, groups_per_cta=8,
                wabsmax=wabsmax, rowmax=rowmax)
    torch.cuda.synchronize()
    _check((pre.cpu(), dx.cpu(), dw.cpu(), db.cpu()), _oracle(rule, B, G), f"C ABI {rule} gpc=8")
