"""Octet storage helpers on the CPU: ``apply_`` / ``canonical`` are inverse for every tensor shape a layer
stores (indices, weights, bias), and the weights land where the lane-per-neuron kernels read them (record p's
input c at float 256 * (p // 32) + 4 * (p % 32) + c for c < 4, + 128 for c >= 4)."""
import pytest
import torch

from granulelayer_b200 import octet_storage
from granulelayer_b200.layout import SparseLayout


def _random_arrangement(G, slots, seed):
    gen = torch.Generator().manual_seed(seed)
    order = torch.stack([torch.randperm(slots, generator=gen) for _ in range(G)]).to(torch.int32)
    cols = torch.stack([torch.randperm(8, generator=gen) for _ in range(G * slots)]).reshape(G, slots, 8)
    kperm = (cols.to(torch.int32) << torch.arange(0, 24, 3, dtype=torch.int32)).sum(-1).to(torch.int32)
    return order, kperm, cols


@pytest.mark.parametrize("G,NB", [(1, 4), (3, 8), (5, 12)])
def test_apply_and_canonical_are_inverse_and_place_weights_for_the_kernels(G, NB):
    slots = NB * 8
    order, kperm, cols = _random_arrangement(G, slots, seed=G * 100 + NB)
    gen = torch.Generator().manual_seed(7)
    idx = torch.randint(0, 4096, (G, NB, 8, 8), generator=gen, dtype=torch.int16)
    w = torch.randn(G, NB, 8, 8, generator=gen)
    b = torch.randn(G, NB, 8, generator=gen)
    si, sw, sb = idx.clone(), w.clone(), b.clone()
    for t in (si, sw, sb):
        octet_storage.apply_(t, order, kperm)
    for got, want in ((si, idx), (sw, w), (sb, b)):
        assert torch.equal(octet_storage.canonical(got, order, kperm), want)
    flat_i, flat_w = si.reshape(G, slots * 8), sw.reshape(G, slots * 8)
    src_i, src_w = idx.reshape(G, slots, 8), w.reshape(G, slots, 8)
    for g in range(G):
        for p in range(0, slots, max(1, slots // 13)):
            n = int(order[g, p])
            for c in range(8):
                k = int(cols[g, p, c])
                assert int(flat_i[g, 8 * p + c]) == int(src_i[g, n, k])            # indices: record layout
                off = 256 * (p // 32) + 4 * (p % 32) + (c & 3) + (128 if c >= 4 else 0)
                assert float(flat_w[g, off]) == float(src_w[g, n, k])              # weights: interleaved
            assert float(sb.reshape(G, slots)[g, p]) == float(b.reshape(G, slots)[g, n])


def test_unsupported_names_what_the_octet_kernels_do_not_run():
    lay_a = SparseLayout(256, 4096, 4, 8, 8, False)
    lay_b = SparseLayout(256, 4096, 4, 8, 8, True)
    assert "Mode B" in octet_storage.unsupported(lay_b, "mean", torch.float32, "cpu")
    assert "pool" in octet_storage.unsupported(lay_a, "max", torch.float32, "cpu")
    assert "fp32 only" in octet_storage.unsupported(lay_a, "mean", torch.bfloat16, "cpu")
    assert "GPU" in octet_storage.unsupported(lay_a, "sum", torch.float32, "cpu")
