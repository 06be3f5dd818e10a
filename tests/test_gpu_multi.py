"""Group sharding over NCCL on 2+ GPUs (skipped with fewer devices).

Each rank shards the same seeded layer (GroupShardedLayer.from_full), runs
forward + backward through the C ABI, all-gathers the pooled output and
all-reduces dX, and compares with the CPU oracle of the full layer.  Ranks are
child processes; NVLS is off and the process group has a short timeout.
"""
import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch

from conftest import assert_close

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 or more GPUs")]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        from granulelayer_b200 import SparsePoolingLayer
        from granulelayer_b200.distributed import GroupShardedLayer, ShardedTrainStep

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        full = SparsePoolingLayer(256, 65536, 256, shared_neurons=None, pooling="mean", dtype=torch.float32,
                                  seed=0, bias_std=0.1)
        lay = GroupShardedLayer.from_full(full).to(dev)
        lay.reorder_neurons()   # bank-aware storage order (the default for shards built on a GPU)
        assert lay.neuron_order is not None
        gen = torch.Generator().manual_seed(3)
        x = torch.randn(64, 256, generator=gen)
        dy = torch.randn(64, 256, generator=gen)
        xr = x.to(dev).requires_grad_(True)
        y = lay(xr)
        (y * dy.to(dev)).sum().backward()
        out = (y.detach().cpu().numpy(), xr.grad.cpu().numpy(), lay.canonical(lay.weight.grad).cpu().numpy(),
               lay.canonical(lay.bias.grad).cpu().numpy(), lay.g0, lay.g1)
        # the overlapped train step gives the same pooled output and dX
        from granulelayer_b200 import FusedAdamW

        step = ShardedTrainStep(lay, FusedAdamW([lay.weight, lay.bias], lr=0.0, moments="fp32"))
        y2, dx2 = step.step(x.to(dev), dy.to(dev))
        out = out + (y2.cpu().numpy(), dx2.cpu().numpy())
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", out))
    except Exception:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc()))


def test_two_gpu_sharded_layer_matches_oracle():
    from granulelayer_b200 import SparsePoolingLayer
    from oracle import oracle as O

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, status, payload = q.get(timeout=300)
        res[r] = (status, payload)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    full = SparsePoolingLayer(256, 65536, 256, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=0,
                              bias_std=0.1)
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(64, 256, generator=gen)
    dy = torch.randn(64, 256, generator=gen)
    c = full.layout.counts_tensor("cpu").numpy()
    args = (x.numpy(), full.indices.numpy(), full.weight.detach().numpy(), full.bias.detach().numpy(), c)
    y = O.forward(*args)
    dx, dw, db, sdx, sdw, sdb = O.backward(*args, dy.numpy(), slack=True)
    for r in range(world):
        status, payload = res[r]
        assert status == "ok", payload
        ys, dxs, dws, dbs, g0, g1, y2, dx2 = payload
        assert_close(ys, y, 1e-5, 1e-6, "y")
        assert_close(dxs, dx, 1e-4, 1e-5, "dx", slack=sdx)
        assert_close(dws, dw[g0:g1], 1e-4, 1e-5, "dw", slack=sdw[g0:g1])
        assert_close(dbs, db[g0:g1], 1e-4, 1e-5, "db", slack=sdb[g0:g1])
        assert_close(y2, y, 1e-5, 1e-6, "y (train step)")
        assert_close(dx2, dx, 1e-4, 1e-5, "dx (train step)", slack=sdx)
