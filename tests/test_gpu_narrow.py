"""Narrow storage (ADR-0024, crates/lyth-ptx/src/lib.rs:607-732): f16 and bf16 buffers, f32
arithmetic, each drained value rounded once at the store. Bit for bit against the evaluator: the
widened inputs through the f32 chain, then the RNE rounding of half.rs (pinned on the reference's
device-measured vectors)."""
import numpy as np
import pytest
import torch

import lyth_b200 as lb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TYPES = {"f16": (torch.float16, orc.to_f16_bits), "bf16": (torch.bfloat16, orc.to_bf16_bits)}


def widen(bits, ty):
    if ty == "f16":
        return orc.f16_bits_to_f32_array(bits)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def narrow_input(seed, n, ty):
    return TYPES[ty][1](orc.uniform(seed, n))


def to_dev(bits, ty, cuda):
    return torch.from_numpy(bits.view(np.int16)).to(cuda).view(TYPES[ty][0])


def dev_bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("ty", ["f16", "bf16"])
@pytest.mark.parametrize("n", [0, 1, 7, 8, 1000, (1 << 20) + 5])
def test_streams_bit_exact(cuda, ty, n):
    xb, yb = narrow_input(11, n, ty), narrow_input(12, n, ty)
    x, y = widen(xb, ty), widen(yb, ty)
    rnd = TYPES[ty][1]
    cases = [
        (lb.STREAM_SAXPY, [2.5], True, lambda: orc.saxpy(2.5, x, y)),
        (lb.STREAM_AXPBY, [1.5, 0.5], True, lambda: orc.axpby(1.5, 0.5, x, y)),
        (lb.STREAM_LERP, [0.3], True, lambda: orc.lerp(0.3, x, y)),
        (lb.STREAM_HORNER, [0.1, 0.2, 0.3, 0.4], False, lambda: orc.horner(0.1, 0.2, 0.3, 0.4, x)),
        (lb.STREAM_COPY, [], False, lambda: x.copy()),
    ]
    for op, sc, two, want in cases:
        xd, yd = to_dev(xb, ty, cuda), to_dev(yb, ty, cuda)
        out = torch.empty(n, dtype=TYPES[ty][0], device=cuda)
        lb.stream_narrow(op, sc, xd, yd if two else None, out)
        assert np.array_equal(dev_bits(out), rnd(want())), (ty, op)


@pytest.mark.parametrize("ty", ["f16", "bf16"])
def test_saxpy_in_place(cuda, ty):
    n = 4099
    xb, yb = narrow_input(13, n, ty), narrow_input(14, n, ty)
    xd, yd = to_dev(xb, ty, cuda), to_dev(yb, ty, cuda)
    lb.stream_narrow(lb.STREAM_SAXPY, [2.5], xd, yd, yd)
    assert np.array_equal(dev_bits(yd), TYPES[ty][1](orc.saxpy(2.5, widen(xb, ty), widen(yb, ty))))


@pytest.mark.parametrize("ty", ["f16", "bf16"])
# rows and cols multiples of 8 take the TMA tiles (64 x 64, edges clipped); the rest the plain tile
@pytest.mark.parametrize("rows,cols", [(1, 1), (33, 17), (257, 300), (4096, 4096), (31, 129), (8, 8), (64, 200),
                                       (136, 72), (1024, 8), (8, 1032)])
def test_transpose_bit_exact(cuda, ty, rows, cols):
    ab = narrow_input(15, rows * cols, ty)
    ad = to_dev(ab, ty, cuda).view(rows, cols)
    bd = torch.empty(cols, rows, dtype=TYPES[ty][0], device=cuda)
    lb.transpose_narrow(ad, bd)
    assert np.array_equal(dev_bits(bd).ravel(), ab.reshape(rows, cols).T.ravel())


# n = 2^22 fills every batch of reference blocks exactly (the paired 32-bit loads throughout);
# offset = 1 starts both buffers on an odd element (2-byte aligned: the 16-bit loads).
@pytest.mark.parametrize("ty", ["f16", "bf16"])
@pytest.mark.parametrize("n,offset", [(1, 0), (2049, 0), (1_000_003, 0), (1 << 22, 0), (1_000_003, 1)])
def test_reduction_partials_bit_exact(cuda, ty, n, offset):
    xb, yb = narrow_input(16, n, ty), narrow_input(17, n, ty)
    x, y = widen(xb, ty), widen(yb, ty)
    grid = int(lb.lib.lyth_b200_reduce_grid(n))
    pad = np.zeros(offset, np.uint16)
    xd = to_dev(np.concatenate([pad, xb]), ty, cuda)[offset:]
    yd = to_dev(np.concatenate([pad, yb]), ty, cuda)[offset:]
    for op, yy, want in ((lb.SUM, None, orc.reduce(orc.SUM, x, grid=grid)),
                         (lb.SUM, yd, orc.reduce(orc.SUM, x, y, grid=grid)),
                         (lb.MAX, None, orc.reduce(orc.MAX, x, grid=grid)),
                         (lb.MIN, None, orc.reduce(orc.MIN, x, grid=grid))):
        got = lb.reduce_partials_narrow(op, xd, yy).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (ty, op, yy is None)


def test_narrow_through_select(cuda):
    from lyth_b200 import examples as ex
    from lyth_b200 import ir

    k = ex.saxpy()
    k.params = [(nm, ir.TY["bf16[]"] if t == ir.TY["f32[]"] else t) for nm, t in k.params]
    sel = k.select()
    n = 10_001
    xb, yb = narrow_input(18, n, "bf16"), narrow_input(19, n, "bf16")
    xd, yd = to_dev(xb, "bf16", cuda), to_dev(yb, "bf16", cuda)
    sel.launch([n, 2.5, xd, yd])
    assert np.array_equal(dev_bits(yd), orc.to_bf16_bits(orc.saxpy(2.5, widen(xb, "bf16"), widen(yb, "bf16"))))
