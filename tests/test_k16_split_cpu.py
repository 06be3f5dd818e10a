"""The arithmetic of the fp32 tensor-core Cover-TopK16 kernels (gl_k16_fwd_tc_f32 / gl_k16_bwd_tc_f32),
restated on the CPU: every fp32 value v with 2^-110 <= |v| below bf16's largest is the exact sum of its
three bf16 terms (v1 = bf16(v), v2 = bf16(v - v1), v3 = bf16(v - v1 - v2), round to nearest even as the
kernels' cvt.rn.bf16x2.f32); below 2^-110 the third term loses what lies under bf16's smallest subnormal,
2^-133.  A product from the six term pairs i + j <= 2 is within 2^-23 |a||b| of a*b, and a whole layer
computed with that arithmetic in fp32 meets the GPU tests' fp32 tolerances against the float64 oracle."""
import numpy as np
import torch


def _split3(v: torch.Tensor):
    t0 = v.to(torch.bfloat16).float()
    r = v - t0
    t1 = r.to(torch.bfloat16).float()
    t2 = (r - t1).to(torch.bfloat16).float()
    return t0, t1, t2


def _samples(n=200_000, seed=0):
    gen = torch.Generator().manual_seed(seed)
    mant = torch.rand(n, generator=gen) + 1.0
    expo = torch.randint(-120, 120, (n,), generator=gen).float()
    sign = torch.where(torch.rand(n, generator=gen) < 0.5, -1.0, 1.0)
    v = (sign * mant * torch.pow(2.0, expo)).float()
    # full 24-bit significands, values just below bf16 rounding ties, subnormals and zero
    extra = torch.tensor([1 + 2 ** -23, 1 + 2 ** -8, 1 + 2 ** -8 + 2 ** -23, 1 - 2 ** -24, 3.0e38, -3.0e38,
                          1.17549435e-38, 2 ** -140, -(2 ** -149), 0.0, -0.0], dtype=torch.float32)
    return torch.cat([v, extra])


def test_three_terms_are_exact():
    v = _samples()
    t0, t1, t2 = _split3(v)
    assert torch.equal(t2.to(torch.bfloat16).float(), t2)                # the third term is a bf16 value
    total = t0.double() + t1.double() + t2.double()
    normal = v.abs() >= 2.0 ** -110
    assert torch.equal(total[normal], v.double()[normal])
    assert float((total - v.double()).abs().max()) < 2.0 ** -133
    assert int((~normal).sum()) >= 3 and bool(((total != v.double()) & ~normal).any())


def test_six_pair_products_are_within_fp32_rounding():
    a, b = _samples(seed=1), _samples(seed=2)
    keep = (a.abs() < 1e18) & (b.abs() < 1e18) & (a.abs() > 1e-18) & (b.abs() > 1e-18)
    a, b = a[keep], b[keep]
    ta, tb = _split3(a), _split3(b)
    approx = torch.zeros_like(a, dtype=torch.float64)
    for s in (2, 1, 0):
        for i in range(s + 1):
            approx += ta[i].double() * tb[s - i].double()      # each bf16 x bf16 product is exact in fp32
    exact = a.double() * b.double()
    err = (approx - exact).abs() / exact.abs()
    assert float(err.max()) <= 1.01 * 2.0 ** -23
    # one bf16 term (the bf16 layer's operand rounding) would not be: its error reaches ~2^-8
    one = (ta[0].double() * tb[0].double() - exact).abs() / exact.abs()
    assert float(one.max()) > 2.0 ** -10


def test_dot_products_match_fp32_accumulation():
    """A 16-term dot product from the six pair sums (accumulated in fp32, the MMA accumulator) agrees
    with the float64 dot product as closely as an fp32 FMA chain does."""
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(4096, 16, generator=gen)
    w = torch.randn(4096, 16, generator=gen) / 8
    tx, tw = _split3(x), _split3(w)
    acc = torch.zeros(4096, dtype=torch.float32)
    for s in (2, 1, 0):
        for i in range(s + 1):
            acc = acc + (tx[i] * tw[s - i]).sum(1, dtype=torch.float32)
    fma = torch.zeros(4096, dtype=torch.float32)
    for k in range(16):
        fma = fma + x[:, k] * w[:, k]
    exact = (x.double() * w.double()).sum(1)
    mag = (x.double() * w.double()).abs().sum(1)
    e_split = ((acc.double() - exact).abs() / mag).max()
    e_fma = ((fma.double() - exact).abs() / mag).max()
    assert float(e_split) < 4 * max(float(e_fma), 2.0 ** -24)
    assert np.isfinite(float(e_split))


def _pairsum(ta, tb, eq):
    """Sum over the term pairs i + j <= 2 (smallest first) of einsum(eq, a_i, b_j) in fp32: the kernels'
    six MMAs, whose bf16 x bf16 products are exact in the fp32 accumulator."""
    acc = None
    for s in (2, 1, 0):
        for i in range(s + 1):
            term = torch.einsum(eq, ta[i], tb[s - i])
            acc = term if acc is None else acc + term
    return acc


def _emulate(x, idx, w, b, counts, gy):
    """y, dx, dw, db of the split kernels restated in torch fp32 (module docstring): x, w and dz as three
    bf16 terms, ReLU, Mean pooling over the valid slots, dX = dz w, dW = dz^T x, db = sum dz."""
    G, NB, C, K = w.shape
    B, D = x.shape
    xg = x[:, idx]                                                       # [B, G, NB, K]
    tx, tw = _split3(xg), _split3(w)
    z = b[None] + _pairsum(tx, tw, "tgnk,gnck->tgnc")
    slot = torch.arange(NB * C).view(NB, C)
    valid = (slot[None] < counts.view(-1, 1, 1)).float()                 # [G, NB, C]
    cnt = counts.float()
    y = (torch.relu(z) * valid[None]).sum((2, 3)) / cnt[None]
    dz = (gy / cnt[None])[:, :, None, None] * (z > 0).float() * valid[None]
    td = _split3(dz)
    dw = _pairsum(td, tx, "tgnc,tgnk->gnck")
    db = dz.sum(0)
    dxg = _pairsum(td, tw, "tgnc,gnck->tgnk")
    dx = torch.zeros(B, D).index_add_(1, idx.reshape(-1), dxg.reshape(B, -1))
    return y, dx, dw, db


def test_split_arithmetic_meets_the_fp32_tolerances():
    """The whole layer computed with the split kernels' arithmetic agrees with the float64 K/C oracle at
    the GPU tests' fp32 tolerances (forward rtol 1e-5 / atol 1e-6; gradients rtol 1e-4 / atol 1e-5 plus
    the oracle's ReLU-boundary allowance), on weights that need all 24 significand bits."""
    from conftest import assert_close
    from granulelayer_b200.cover_topk16 import CoverTopK16Layer
    from granulelayer_b200.kgen import KLayout, init_envelope_parameters
    from granulelayer_b200.supergroups import ConnectivityPlan
    from oracle import kc_oracle

    D, H, G = 256, 3452, 8
    w64, b64 = init_envelope_parameters(KLayout(D, H, G, 64, 256), "cpu", dtype=torch.bfloat16, seed=1,
                                        bias_std=0.1)
    lay = CoverTopK16Layer.from_envelope(w64, b64, input_dim=D, hidden_dim=H, output_dim=G,
                                         connectivity=ConnectivityPlan(64, 16, seed=4), device="cpu")
    w = lay.weight.detach().clone()
    w.mul_(1 + 2.0 ** -23).add_(torch.sign(w) * 2.0 ** -20)
    b = lay.bias.detach()
    idx, counts = lay.indices.long(), lay.counts
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(48, D, generator=gen)
    gy = torch.randn(48, G, generator=gen)
    y, dx, dw, db = _emulate(x, idx, w, b, counts, gy)
    ry, rdx, rdw, rdb, (sdx, sdw, sdb) = kc_oracle.grads(x.numpy(), idx.numpy(), w.numpy(), b.numpy(),
                                                         counts.numpy(), gy.numpy(), act="relu", slack=True)
    assert_close(y, ry, rtol=1e-5, atol=1e-6, what="y")
    assert_close(dx, rdx, rtol=1e-4, atol=1e-5, what="dx", slack=sdx)
    assert_close(dw, rdw, rtol=1e-4, atol=1e-5, what="dw", slack=sdw)
    assert_close(db, rdb, rtol=1e-4, atol=1e-5, what="db", slack=sdb)
    # a single bf16 term per operand (no split) is outside the forward tolerance on the same layer
    z1 = b[None] + torch.einsum("tgnk,gnck->tgnc", _split3(x[:, idx])[0], _split3(w)[0])
    slot = torch.arange(w.shape[1] * 16).view(w.shape[1], 16)
    y1 = (torch.relu(z1) * (slot[None] < counts.view(-1, 1, 1))[None]).sum((2, 3)) / counts.float()[None]
    assert float(((y1.double() - torch.from_numpy(ry)).abs() - (1e-6 + 1e-5 * torch.from_numpy(ry).abs())).max()) > 0
