"""Group sharding over NCCL on 2, 4 and 8 GPUs (each world size skipped with fewer devices).

Each rank shards the same seeded layer (GroupShardedLayer.from_full, bank-ordered storage), runs
forward + backward through the C ABI, all-gathers the pooled output and all-reduces dX, and the
results are compared with the CPU oracle of the full layer.  Then one overlapped ShardedTrainStep
with FusedAdamW (lr 1e-3, fp32 moments) runs on the same inputs:
  * its pooled output and dX match the oracle;
  * the first moment it stored, m = (1 - b1) g, holds the gradient the step used: g = m / (1 - b1)
    must match the oracle's dW / db (slot order, via canonical()) within the backward tolerance;
  * the updated parameters equal the oracle's Adam step (oracle/gl_oracle.c glo_adam, the
    reference's optim.py:39-42) applied to the old parameters and that gradient.
Ranks are child processes; NVLS is off and the process group has a short timeout.
"""
import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch

from conftest import assert_close

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 or more GPUs")]

D, H, G, B = 256, 65536, 256, 64
LR, BETAS, EPS = 1e-3, (0.9, 0.999), 1e-8


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_layer():
    from granulelayer_b200 import SparsePoolingLayer

    return SparsePoolingLayer(D, H, G, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=0,
                              bias_std=0.1)


def _inputs():
    gen = torch.Generator().manual_seed(3)
    return torch.randn(B, D, generator=gen), torch.randn(B, G, generator=gen)


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        from granulelayer_b200 import FusedAdamW
        from granulelayer_b200.distributed import GroupShardedLayer, ShardedTrainStep

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        lay = GroupShardedLayer.from_full(_full_layer()).to(dev)
        lay.reorder_neurons()   # bank-aware storage order (the default for shards built on a GPU)
        assert lay.neuron_order is not None
        x, dy = _inputs()
        xr = x.to(dev).requires_grad_(True)
        y = lay(xr)
        (y * dy.to(dev)).sum().backward()
        out = dict(y=y.detach().cpu().numpy(), dx=xr.grad.cpu().numpy(),
                   dw=lay.canonical(lay.weight.grad).cpu().numpy(), db=lay.canonical(lay.bias.grad).cpu().numpy(),
                   g0=lay.g0, g1=lay.g1)
        lay.weight.grad = lay.bias.grad = None
        # one overlapped training step with a real learning rate
        w0, b0 = lay.canonical_shard()[1:]
        opt = FusedAdamW([lay.weight, lay.bias], lr=LR, betas=BETAS, eps=EPS, moments="fp32")
        step = ShardedTrainStep(lay, opt)
        y2, dx2 = step.step(x.to(dev), dy.to(dev))
        torch.cuda.synchronize()
        out.update(y2=y2.cpu().numpy(), dx2=dx2.cpu().numpy(), w0=w0.cpu().numpy(), b0=b0.cpu().numpy(),
                   w1=lay.canonical(lay.weight.detach()).cpu().numpy(),
                   b1=lay.canonical(lay.bias.detach()).cpu().numpy(),
                   mw=lay.canonical(opt.state[lay.weight]["m"]).cpu().numpy(),
                   mb=lay.canonical(opt.state[lay.bias]["m"]).cpu().numpy(),
                   gz=float(lay.weight.main_grad.abs().max()))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", out))
    except Exception:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_layer_and_train_step_match_oracle(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import oracle as O

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, status, payload = q.get(timeout=600)
            res[r] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    full = _full_layer()
    x, dy = _inputs()
    c = full.layout.counts_tensor("cpu").numpy()
    args = (x.numpy(), full.indices.numpy(), full.weight.detach().numpy(), full.bias.detach().numpy(), c)
    y = O.forward(*args)
    dx, dw, db, sdx, sdw, sdb = O.backward(*args, dy.numpy(), slack=True)
    covered = np.zeros(G, bool)
    for r in range(world):
        status, o = res[r]
        assert status == "ok", o
        g0, g1 = o["g0"], o["g1"]
        covered[g0:g1] = True
        assert_close(o["y"], y, 1e-5, 1e-6, f"rank {r} y")
        assert_close(o["dx"], dx, 1e-4, 1e-5, f"rank {r} dx", slack=sdx)
        assert_close(o["dw"], dw[g0:g1], 1e-4, 1e-5, f"rank {r} dw", slack=sdw[g0:g1])
        assert_close(o["db"], db[g0:g1], 1e-4, 1e-5, f"rank {r} db", slack=sdb[g0:g1])
        assert_close(o["y2"], y, 1e-5, 1e-6, f"rank {r} y (train step)")
        assert_close(o["dx2"], dx, 1e-4, 1e-5, f"rank {r} dx (train step)", slack=sdx)
        assert o["gz"] == 0.0, "the fused optimizer leaves main_grad zeroed"
        for name, m, p0, p1, ref, sl in (("w", o["mw"], o["w0"], o["w1"], dw[g0:g1], sdw[g0:g1]),
                                         ("b", o["mb"], o["b0"], o["b1"], db[g0:g1], sdb[g0:g1])):
            g_used = m.astype(np.float64) / (1.0 - BETAS[0])
            assert_close(g_used, ref, 1e-4, 1e-5, f"rank {r} gradient the step used for {name}", slack=sl)
            want, _, _ = O.adam_step(p0, g_used, np.zeros_like(g_used), np.zeros_like(g_used), LR, BETAS[0],
                                     BETAS[1], EPS, 0.0, 1)
            assert_close(p1, want, 1e-6, 1e-7, f"rank {r} {name} after the Adam step")
            assert float(np.abs(p1 - p0).max()) > 0.5 * LR, f"rank {r} {name}: the step moved nothing"
    assert covered.all(), "the shards cover every group"
