"""Group sharding across ranks (granulelayer_b200/distributed.py), on CPU gloo ranks.

The launch backend is replaced by a test double that computes the forward and
backward with the CPU oracle, so the sharding, all-gather and all-reduce logic
is exercised exactly as on GPUs (NCCL there, gloo here).  A failure test makes
one rank exit before a collective and checks that its peer fails instead of
hanging.
"""
import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist

from granulelayer_b200.distributed import GroupShardedLayer, ShardedTrainStep, gather_columns, shard_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleRuntime:
    """Level1Runtime stand-in for CPU tensors (test double; uses the oracle)."""

    def __init__(self, lay):
        self.level = lay.cfg.levels[0]
        self.lay = lay
        self.idx = lay.indices

    def forward(self, x, w, b, track_ids=False):
        from oracle import oracle as O

        pre = O.forward(x.numpy(), self.idx.numpy(), w.detach().numpy(), b.detach().numpy(),
                        self.lay.counts.numpy(), self.level.type, self.level.activation)
        return {"pre": torch.from_numpy(pre).float()}

    def backward(self, x, w, b, g_pre, saved, policy, dw_buf, db_buf, recomputed=False):
        from oracle import oracle as O

        dx, dw, db = O.backward(x.numpy(), self.idx.numpy(), w.detach().numpy(), b.detach().numpy(),
                                self.lay.counts.numpy(), g_pre.double().numpy(), self.level.type,
                                self.level.activation)
        dw_buf += torch.from_numpy(dw).float()
        db_buf += torch.from_numpy(db).float()
        return torch.from_numpy(dx).float()


class NoOpt:
    def step(self):
        pass


def _full_layer(D, H, G, seed):
    from granulelayer_b200 import SparsePoolingLayer

    return SparsePoolingLayer(D, H, G, shared_neurons=None, pooling="mean", dtype=torch.float32, seed=seed,
                              bias_std=0.2)


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        D, H, G, B = 48, 2600, 5, 7
        full = _full_layer(D, H, G, seed=3)
        gen = torch.Generator().manual_seed(9)
        x = torch.randn(B, D, generator=gen)
        dy = torch.randn(B, G, generator=gen)
        if mode == "gather":
            g0, g1 = shard_range(G, rank, world)
            local = torch.arange(B * G, dtype=torch.float32).view(B, G)[:, g0:g1].contiguous()
            out = gather_columns(local, G)
            q.put((rank, "ok", out.numpy()))
        elif mode in ("layer", "step"):
            lay = GroupShardedLayer.from_full(full, runtime_factory=OracleRuntime)
            if mode == "layer":
                xr = x.clone().requires_grad_(True)
                y = lay(xr)
                (y * dy).sum().backward()
                q.put((rank, "ok", (y.detach().numpy(), xr.grad.numpy(), lay.weight.grad.numpy(),
                                    lay.bias.grad.numpy(), lay.g0, lay.g1)))
            else:
                step = ShardedTrainStep(lay, NoOpt())
                y, dx = step.step(x, dy)
                q.put((rank, "ok", (y.numpy(), dx.numpy(), lay.weight.main_grad.numpy(),
                                    lay.bias.main_grad.numpy(), lay.g0, lay.g1)))
        elif mode == "state":
            lay = GroupShardedLayer.from_full(full, runtime_factory=OracleRuntime)
            sd = lay.full_state_dict()
            other = GroupShardedLayer.from_full(_full_layer(D, H, G, seed=4), runtime_factory=OracleRuntime)
            other.load_full_state_dict(sd)
            same = all(torch.equal(a, b) for a, b in zip(other.canonical_shard(), lay.canonical_shard()))
            q.put((rank, "ok", ({k: v.numpy() for k, v in sd.items()}, same)))
        elif mode == "dead_peer":
            if rank == 1:
                q.put((rank, "ok", "left before the collective"))
            else:
                try:
                    gather_columns(torch.ones(B, 3), G)
                    q.put((rank, "no-error", None))
                except Exception as e:  # noqa: BLE001
                    q.put((rank, "raised", type(e).__name__))
            q.close()
            q.join_thread()  # flush the message before leaving without the usual teardown
            os._exit(0)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc()))


def _run(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, status, payload = q.get(timeout=timeout)
        out[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("G,P", [(4096, 8), (5, 2), (7, 3), (3, 3), (1, 1)])
def test_shard_range_partitions_groups(G, P):
    spans = [shard_range(G, r, P) for r in range(P)]
    assert spans[0][0] == 0 and spans[-1][1] == G
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_gather_columns_uneven():
    out = _run("gather")
    expect = np.arange(7 * 5, dtype=np.float32).reshape(7, 5)
    for r in range(2):
        assert out[r][0] == "ok", out[r][1]
        np.testing.assert_array_equal(out[r][1], expect)


def _reference(D=48, H=2600, G=5, B=7):
    from oracle import oracle as O

    full = _full_layer(D, H, G, seed=3)
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(B, D, generator=gen)
    dy = torch.randn(B, G, generator=gen)
    c = full.layout.counts_tensor("cpu").numpy()
    args = (x.numpy(), full.indices.numpy(), full.weight.detach().numpy(), full.bias.detach().numpy(), c)
    y = O.forward(*args)
    dx, dw, db = O.backward(*args, dy.numpy())
    return y, dx, dw, db


@pytest.mark.parametrize("mode", ["layer", "step"])
def test_sharded_layer_equals_full_layer(mode):
    y, dx, dw, db = _reference()
    out = _run(mode)
    for r in range(2):
        status, payload = out[r]
        assert status == "ok", payload
        ys, dxs, dws, dbs, g0, g1 = payload
        np.testing.assert_allclose(ys, y, rtol=1e-6, atol=1e-7)      # all-gathered pooled output
        np.testing.assert_allclose(dxs, dx, rtol=1e-5, atol=1e-6)    # all-reduced dX
        np.testing.assert_allclose(dws, dw[g0:g1], rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(dbs, db[g0:g1], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("world", [2, 3])
def test_full_state_dict_is_the_single_gpu_state_dict(world):
    """Sharded checkpoints gather to the drop-in layer's state dict, bit for bit, and load back."""
    full = _full_layer(48, 2600, 5, seed=3)
    ref = {k: v.numpy() for k, v in full.state_dict().items()}
    out = _run("state", world=world)
    for r in range(world):
        status, payload = out[r]
        assert status == "ok", payload
        sd, same = payload
        assert set(sd) == set(ref)
        for k in ref:
            np.testing.assert_array_equal(sd[k], ref[k])
        assert same


def test_dead_peer_fails_instead_of_hanging():
    out = _run("dead_peer", timeout=90)
    status, payload = out[0]
    assert status == "raised", f"rank 0: {status} {payload}"
