"""Reductions: per-block partials bit for bit with the evaluator's two-stage order; the whole
reduction equal to the oracle's partials folded in the documented cluster order, and within
1e-5 relative of the f64 sum."""
import numpy as np
import pytest
import torch

import lyth_b200 as lb
from oracle import oracle as orc
from tests import adr16
from tests.conftest import bits

pytestmark = pytest.mark.gpu


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("n", [1, 10, 255, 256, 2049, 100_000, (1 << 22) + 5])
@pytest.mark.parametrize("op", [lb.SUM, lb.MAX, lb.MIN, "dot"])
def test_partials_bit_exact(cuda, n, op):
    x, y = orc.uniform(21, n), orc.uniform(22, n)
    grid = lb.reduce_grid(n)
    if op == "dot":
        got = lb.reduce_partials(lb.SUM, dev(x, cuda), dev(y, cuda))
        want = orc.reduce(orc.SUM, x, y, grid=grid)
    else:
        got = lb.reduce_partials(op, dev(x, cuda))
        want = orc.reduce(op, x, grid=grid)
    assert np.array_equal(bits(got.cpu().numpy()), bits(want))


@pytest.mark.parametrize("grid", [1, 3, 1000])
def test_partials_at_any_grid(cuda, grid):
    n = 123_457
    x = orc.uniform(23, n)
    got = lb.reduce_partials(lb.SUM, dev(x, cuda), grid=grid)
    assert np.array_equal(bits(got.cpu().numpy()), bits(orc.reduce(orc.SUM, x, grid=grid)))


def test_signed_zeros_and_nan_in_max_min(cuda):
    # ADR-0013: the device and the oracle must agree on (-0, +0) and on a NaN operand.
    n = 4096
    x = np.zeros(n, np.float32)
    x[::2] = -0.0
    x[7] = np.nan
    for op in (lb.MAX, lb.MIN):
        got = lb.reduce_partials(op, dev(x, cuda), grid=4).cpu().numpy()
        want = orc.reduce(op, x, grid=4)
        assert np.array_equal(bits(got), bits(want)), op


@pytest.mark.parametrize("pair", [(-0.0, 0.0), (0.0, -0.0), (-0.0, -0.0), (0.0, 0.0), (float("nan"), -0.0),
                                  (-0.0, float("nan")), (-1.5, float("nan"))])
def test_combine_both_operand_orders(cuda, pair):
    # ast.rs:594-621: max(-0, +0) = +0 and min(-0, +0) = -0 whichever comes first; NaN loses.
    # With two elements in one block, slot 0 = x[0], slot 1 = x[1], and the tree's last level
    # combines them in that order.
    x = np.array(pair, np.float32)
    for op in (lb.MAX, lb.MIN):
        got = lb.reduce_partials(op, dev(x, cuda), grid=1).cpu().numpy()
        want = orc.reduce(op, x, grid=1)
        assert np.array_equal(bits(got), bits(want)), (op, pair, got, want)


def _cluster_fold(op, partials):
    # lyth_b200_reduce's order: partials in groups of 8 (clusters), folded left to right within
    # each group, then the group results left to right. Blocks past the grid add the identity.
    p = list(partials) + [orc.identity(op)] * ((-len(partials)) % 8)
    groups = []
    for g in range(0, len(p), 8):
        acc = p[g]
        for v in p[g + 1:g + 8]:
            acc = orc.combine(op, acc, v)
        groups.append(acc)
    acc = groups[0]
    for v in groups[1:]:
        acc = orc.combine(op, acc, v)
    return np.float32(acc)


@pytest.mark.parametrize("n", [5, 5000, (1 << 24) + 11])
@pytest.mark.parametrize("op", [lb.SUM, lb.MAX, lb.MIN, "dot"])
def test_full_reduction(cuda, n, op):
    x, y = orc.uniform(31, n), orc.uniform(32, n)
    grid = lb.reduce_grid(n)
    if op == "dot":
        got = float(lb.reduce(lb.SUM, dev(x, cuda), dev(y, cuda)).cpu()[0])
        partials = orc.reduce(orc.SUM, x, y, grid=grid)
        want = _cluster_fold(orc.SUM, partials)
        ref64 = orc.sum_f64(x, y)
    else:
        got = float(lb.reduce(op, dev(x, cuda)).cpu()[0])
        partials = orc.reduce(op, x, grid=grid)
        want = _cluster_fold(op, partials)
        ref64 = orc.sum_f64(x) if op == lb.SUM else (float(x.max()) if op == lb.MAX else float(x.min()))
    assert np.float32(got).view(np.uint32) == want.view(np.uint32)
    if op in (lb.SUM, "dot"):
        scale = orc.sum_f64(np.abs(x)) if op == lb.SUM else orc.sum_f64(np.abs(x * y))
        assert abs(got - ref64) <= 1e-5 * scale  # relative to the sum of magnitudes
    else:
        assert got == ref64


@pytest.mark.parametrize("k,op", [("sum", orc.SUM), ("max_of", orc.MAX), ("min_of", orc.MIN)])
def test_adr16_reductions(cuda, k, op):
    n = 1_000_003
    x = orc.uniform(41, n)
    grid = int(getattr(lb.lib, f"lyth_{k}_grid")(n))
    part = torch.empty(grid, device=cuda)
    xd = dev(x, cuda)
    assert adr16.launch(k, adr16.load(k), n, xd.data_ptr(), part.data_ptr()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(bits(part.cpu().numpy()), bits(orc.reduce(op, x, grid=grid)))


def test_adr16_dot(cuda):
    n = 777_777
    x, y = orc.uniform(42, n), orc.uniform(43, n)
    grid = int(lb.lib.lyth_dot_grid(n))
    part = torch.empty(grid, device=cuda)
    xd, yd = dev(x, cuda), dev(y, cuda)
    assert adr16.launch("dot", adr16.load("dot"), n, xd.data_ptr(), yd.data_ptr(), part.data_ptr()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(bits(part.cpu().numpy()), bits(orc.reduce(orc.SUM, x, y, grid=grid)))
