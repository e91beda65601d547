"""Parity of the streamed elementwise bodies and the rank-2 walks with the host evaluator:
bit for bit (the north star's bar for elementwise, copy and transpose)."""
import numpy as np
import pytest
import torch

import lyth_b200 as lb
from oracle import oracle as orc
from tests import adr16
from tests.conftest import bits

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 3, 4, 5, 1023, 4096, (1 << 20) + 3]


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("n", SIZES)
def test_saxpy_axpby_lerp_horner(cuda, n):
    x, y = orc.uniform(1, n), orc.uniform(2, n)
    yd = dev(y, cuda)
    lb.saxpy(2.5, dev(x, cuda), yd)
    assert np.array_equal(bits(yd.cpu().numpy()), bits(orc.saxpy(2.5, x, y)))
    yd = dev(y, cuda)
    lb.axpby(1.25, -0.75, dev(x, cuda), yd)
    assert np.array_equal(bits(yd.cpu().numpy()), bits(orc.axpby(1.25, -0.75, x, y)))
    zd = torch.empty(n, device=cuda)
    lb.lerp(0.3, dev(x, cuda), dev(y, cuda), zd)
    assert np.array_equal(bits(zd.cpu().numpy()), bits(orc.lerp(0.3, x, y)))
    yd = torch.empty(n, device=cuda)
    lb.horner(0.5, -1.5, 2.25, 0.125, dev(x, cuda), yd)
    assert np.array_equal(bits(yd.cpu().numpy()), bits(orc.horner(0.5, -1.5, 2.25, 0.125, x)))


def test_unaligned_buffers_take_the_scalar_path(cuda):
    n = 10001
    x, y = orc.uniform(3, n + 1), orc.uniform(4, n + 1)
    xd, yd = dev(x, cuda), dev(y, cuda)
    lb.saxpy(-3.0, xd[1:], yd[1:])  # 4-byte offset: not 16-byte aligned
    want = y.copy()
    want[1:] = orc.saxpy(-3.0, x[1:], y[1:])
    assert np.array_equal(bits(yd.cpu().numpy()), bits(want))


def test_lyth_run_inputs_through_the_adr16_launch(cuda):
    # The inputs `lyth run` generates (inputs.rs), launched as a generated C binding would.
    n = 1 << 16
    x, y = orc.buffer("x", orc.TY_F32, n), orc.buffer("y", orc.TY_F32, n)
    xd, yd = dev(x, cuda), dev(y, cuda)
    fn = adr16.load("saxpy")
    assert adr16.launch("saxpy", fn, n, 2.0, xd.data_ptr(), yd.data_ptr()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(bits(yd.cpu().numpy()), bits(orc.saxpy(2.0, x, y)))
    # launch_with: any grid the caller picks gives the same bits (grid-stride).
    yd = dev(y, cuda)
    assert adr16.launch("saxpy", fn, n, 2.0, xd.data_ptr(), yd.data_ptr(), grid=7) == 0
    torch.cuda.synchronize()
    assert np.array_equal(bits(yd.cpu().numpy()), bits(orc.saxpy(2.0, x, y)))


def test_adr16_family_elementwise(cuda):
    n = 70001
    x, y = orc.uniform(5, n), orc.uniform(6, n)
    xd, yd, zd = dev(x, cuda), dev(y, cuda), torch.empty(n, device=cuda)
    assert adr16.launch("axpby", adr16.load("axpby"), n, 0.5, 2.0, xd.data_ptr(), yd.data_ptr()) == 0
    assert adr16.launch("lerp", adr16.load("lerp"), n, 0.25, xd.data_ptr(), yd.data_ptr(), zd.data_ptr()) == 0
    torch.cuda.synchronize()
    want_y = orc.axpby(0.5, 2.0, x, y)
    assert np.array_equal(bits(yd.cpu().numpy()), bits(want_y))
    assert np.array_equal(bits(zd.cpu().numpy()), bits(orc.lerp(0.25, x, want_y)))
    hd = torch.empty(n, device=cuda)
    assert adr16.launch("horner", adr16.load("horner"), n, 1.0, 2.0, 3.0, 4.0, xd.data_ptr(), hd.data_ptr()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(bits(hd.cpu().numpy()), bits(orc.horner(1.0, 2.0, 3.0, 4.0, x)))


# ADR-0017's ragged shapes, plus the headline 4096^2.
SHAPES = [(1, 1), (33, 17), (31, 129), (1024, 33), (64, 64), (257, 300), (4095, 4095), (4097, 4097), (4096, 4096),
          (4, 4), (36, 100), (100, 68), (1028, 516), (8, 4096)]  # multiples of 4: the TMA path, edges clipped


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_transposes_and_copy2d(cuda, rows, cols):
    a = orc.uniform(3, rows * cols)
    ad = dev(a, cuda).view(rows, cols)
    want_t = orc.transpose(rows, cols, a)
    for f in (lb.transpose_tiled, lb.transpose_naive):
        bd = torch.full((cols, rows), float("nan"), device=cuda)
        f(ad, bd)
        assert np.array_equal(bits(bd.cpu().numpy().ravel()), bits(want_t)), f.__name__
    cd = torch.empty(rows, cols, device=cuda)
    lb.copy2d(ad, cd)
    assert np.array_equal(bits(cd.cpu().numpy().ravel()), bits(orc.copy2d(rows, cols, a)))


def test_adr16_transposes(cuda):
    rows, cols = 1000, 777
    a = orc.uniform(8, rows * cols)
    ad = dev(a, cuda)
    for k in ("transpose", "transpose_tiled"):
        bd = torch.empty(rows * cols, device=cuda)
        assert adr16.launch(k, adr16.load(k), rows, cols, ad.data_ptr(), bd.data_ptr()) == 0
        torch.cuda.synchronize()
        assert np.array_equal(bits(bd.cpu().numpy()), bits(orc.transpose(rows, cols, a))), k
    bd = torch.empty(rows * cols, device=cuda)
    assert adr16.launch("copy2d", adr16.load("copy2d"), rows, cols, ad.data_ptr(), bd.data_ptr()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(bits(bd.cpu().numpy()), bits(a))
