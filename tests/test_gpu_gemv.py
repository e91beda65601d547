"""gate_proj GEMV (INT4 / NF4, group 64, fp16 scales): dequantisation bit for bit with the
oracle; y within 1e-3 relative (||y - ref|| / ||ref||, ref in f64). Parity unpinned: the
reference has no kernel for this class, so the format and the oracle are this project's."""
import numpy as np
import pytest
import torch

import lyth_b200 as lb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def problem(rows, k, group, seed=60):
    """W nibbles uniform over 0..15 (INT4: -8..7; NF4: a codebook index), scales |N(0, 0.02)|
    as fp16, x ~ N(0, 1) as fp16."""
    raw = orc.uniform(seed, rows * k // 2)
    w = ((raw + 1.0) * 128.0).astype(np.int64).clip(0, 255).astype(np.uint8)
    scales = orc.to_f16_bits(np.abs(orc.normal(seed + 1, rows * (k // group), 0.0, 0.02)))
    x = orc.to_f16_bits(orc.normal(seed + 2, k, 0.0, 1.0))
    return w, scales, x


def to_dev(w, scales, x, rows, k, group, cuda):
    wd = torch.from_numpy(w).to(cuda).view(rows, k // 2)
    sd = torch.from_numpy(scales.view(np.float16)).to(cuda)
    xd = torch.from_numpy(x.view(np.float16)).to(cuda)
    return wd, sd, xd


@pytest.mark.parametrize("fmt", [lb.GEMV_INT4, lb.GEMV_NF4])
@pytest.mark.parametrize("rows,k,group", [(64, 1024, 64), (14336, 4096, 64), (3, 24, 8)])
def test_dequant_bit_exact(cuda, fmt, rows, k, group):
    # lyth_b200_gemv_dequant decodes W with the GEMV kernels' own decode (decode_word): a change
    # to the hot decode (nibble order, the PRMT selectors, the INT4 offset) breaks this test.
    w, scales, x = problem(rows, k, group)
    wd, sd, _ = to_dev(w, scales, x, rows, k, group, cuda)
    out = torch.empty(rows * k, device=cuda)
    lb.gemv_dequant(fmt, wd, sd, out, group=group)
    want = orc.gemv_dequant(fmt, rows, k, group, w, scales)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("fmt", [lb.GEMV_INT4, lb.GEMV_NF4])
# the ring kernel streams 8-row stages (1001 and 5 rows end in a partial stage); 37 x 3072 with
# group 1024 runs the row kernel
@pytest.mark.parametrize("rows,k,group", [(64, 1024, 64), (14336, 4096, 64), (1000, 2048, 128), (37, 3072, 1024),
                                          (1001, 2048, 64), (5, 4096, 64)])
def test_gemv_within_tolerance(cuda, fmt, rows, k, group):
    w, scales, x = problem(rows, k, group)
    wd, sd, xd = to_dev(w, scales, x, rows, k, group, cuda)
    y = torch.empty(rows, dtype=torch.float16, device=cuda)
    lb.gemv_q4(fmt, wd, sd, xd, y, group=group)
    got = y.cpu().numpy().astype(np.float64)
    ref = orc.gemv_f64(fmt, rows, k, group, w, scales, x)
    rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert rel <= 1e-3, rel


@pytest.mark.parametrize("fmt", [lb.GEMV_INT4, lb.GEMV_NF4])
def test_gemv_is_the_dequantised_product(cuda, fmt):
    # y against the f64 product of the DEVICE's dequantised matrix (the values the kernel's
    # decode produces) with x: the same 1e-3 bar, so the GEMV multiplies what the dequant shows.
    rows, k, group = 14336, 4096, 64
    w, scales, x = problem(rows, k, group, seed=61)
    wd, sd, xd = to_dev(w, scales, x, rows, k, group, cuda)
    deq = torch.empty(rows * k, device=cuda)
    lb.gemv_dequant(fmt, wd, sd, deq, group=group)
    y = torch.empty(rows, dtype=torch.float16, device=cuda)
    lb.gemv_q4(fmt, wd, sd, xd, y, group=group)
    ref = deq.view(rows, k).double() @ xd.double()
    got = y.double()
    rel = float(torch.linalg.norm(got - ref) / torch.linalg.norm(ref))
    assert rel <= 1e-3, rel
