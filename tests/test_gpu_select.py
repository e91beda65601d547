"""Kernels chosen by lyth_b200_select and launched by lyth_b200_launch with arguments in
declaration order (lyth-cuda's Arg slots), bit for bit against the evaluator -- the path a
`lyth run` would take through this back end."""
import numpy as np
import pytest
import torch

import lyth_b200 as lb
from lyth_b200 import circuit as cc
from oracle import oracle as orc
from lyth_b200 import examples as ex
from tests.conftest import bits

pytestmark = pytest.mark.gpu


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def test_streams_through_select(cuda):
    n = (1 << 16) + 5
    x, y = orc.uniform(1, n), orc.uniform(2, n)
    xd, yd = dev(x, cuda), dev(y, cuda)
    ex.saxpy().select().launch([n, 2.5, xd, yd])
    assert np.array_equal(bits(yd.cpu().numpy()), bits(orc.saxpy(2.5, x, y)))
    xd, yd, zd = dev(x, cuda), dev(y, cuda), torch.empty(n, device=cuda)
    ex.lerp().select().launch([n, 0.3, xd, yd, zd])
    assert np.array_equal(bits(zd.cpu().numpy()), bits(orc.lerp(0.3, x, y)))
    yd = dev(y, cuda)
    ex.horner().select().launch([n, 0.1, 0.2, 0.3, 0.4, xd, yd])
    assert np.array_equal(bits(yd.cpu().numpy()), bits(orc.horner(0.1, 0.2, 0.3, 0.4, x)))


def test_transpose_and_reductions_through_select(cuda):
    rows, cols = 257, 300
    a = orc.uniform(3, rows * cols)
    bd = torch.empty(cols * rows, device=cuda)
    ex.transpose(True).select().launch([rows, cols, dev(a, cuda), bd])
    assert np.array_equal(bd.cpu().numpy(), orc.transpose(rows, cols, a))
    n = 100_003
    x, y = orc.uniform(4, n), orc.uniform(5, n)
    grid = int(lb.lib.lyth_b200_reduce_grid(n))
    part = torch.empty(grid, device=cuda)
    ex.reduction("dot").select().launch([n, dev(x, cuda), dev(y, cuda), part])
    want = orc.reduce(orc.SUM, x, y, grid=grid)
    assert np.array_equal(bits(part.cpu().numpy()), bits(want))
    part = torch.empty(grid, device=cuda)
    ex.reduction("max").select().launch([n, dev(x, cuda), part])
    assert np.array_equal(bits(part.cpu().numpy()), bits(orc.reduce(orc.MAX, x, grid=grid)))


@pytest.mark.parametrize("q", [0, 3, 9])
def test_gates_through_select(cuda, q):
    nq = 12
    n = 1 << nq
    re, im = orc.random_state(40 + q, nq)
    m = cc.f32s(cc.zyz(0.3, 1.1, -0.7))
    qr, qi = torch.empty(n, device=cuda), torch.empty(n, device=cuda)
    ex.gate_q().select().launch([n, 1 << q] + m + [dev(re, cuda), dev(im, cuda), qr, qi])
    wr, wi = orc.gate_q(1 << q, m, re, im)
    assert np.array_equal(bits(qr.cpu().numpy()), bits(wr)) and np.array_equal(bits(qi.cpu().numpy()), bits(wi))
    c, t = (q + 1) % nq, q
    wc, wt = orc.widths_ct(c, t)
    ex.cu_q().select().launch([n, wc, wt] + m + [dev(re, cuda), dev(im, cuda), qr, qi])
    wr, wi = orc.cu_q(wc, wt, m, re, im)
    assert np.array_equal(bits(qr.cpu().numpy()), bits(wr)) and np.array_equal(bits(qi.cpu().numpy()), bits(wi))
    ex.swap_q().select().launch([n, wc, wt, dev(re, cuda), dev(im, cuda), qr, qi])
    wr, wi = orc.swap_q(wc, wt, re, im)
    assert np.array_equal(bits(qr.cpu().numpy()), bits(wr)) and np.array_equal(bits(qi.cpu().numpy()), bits(wi))
    ex.hadamard_q().select().launch([n, 1 << q, float(np.float32(cc.S)), dev(re, cuda), dev(im, cuda), qr, qi])
    wr, wi = orc.hadamard_q(1 << q, float(np.float32(cc.S)), re, im)
    assert np.array_equal(bits(qr.cpu().numpy()), bits(wr)) and np.array_equal(bits(qi.cpu().numpy()), bits(wi))


def test_a_refused_width_runs_nothing(cuda):
    n = 96
    re = torch.zeros(n, device=cuda)
    qr = torch.full((n,), 7.0, device=cuda)
    with pytest.raises(lb.LythError):
        ex.gate_q().select().launch([n, 64] + [0.0] * 8 + [re, re, qr, qr])  # 2w = 128 does not divide 96
    torch.cuda.synchronize()
    assert float(qr.min()) == 7.0


def test_matmul_through_select(cuda):
    m = n = k = 256
    a, b = orc.uniform(6, m * k), orc.uniform(7, k * n)
    c = torch.empty(m * n, device=cuda)
    ex.matmul(False).select().launch([m, n, k, dev(a, cuda), dev(b, cuda), c])
    assert np.array_equal(bits(c.cpu().numpy()), bits(orc.matmul(m, n, k, a, b)))
