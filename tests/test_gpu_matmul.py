"""The f32 contraction: exact mode bit for bit with eval_contraction (p ascending, mul.rn then
add.rn); the FFMA mode within the north star's 1e-5 relative (||C - ref|| / ||ref||)."""
import numpy as np
import pytest
import torch

import lyth_b200 as lb
from oracle import oracle as orc
from tests import adr16
from tests.conftest import bits

pytestmark = pytest.mark.gpu


def operands(m, n, k, seed=4):
    s = 1.0 / np.sqrt(k)
    return orc.normal(seed, m * k, 0.0, s), orc.normal(seed + 1, k * n, 0.0, s)


def rel(got, want):
    got64, want64 = got.astype(np.float64), want.astype(np.float64)
    return float(np.linalg.norm(got64 - want64) / np.linalg.norm(want64))


@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (128, 384, 64), (100, 70, 33), (1, 1, 1), (5, 300, 17)])
def test_exact_mode_bit_for_bit(cuda, m, n, k):
    a, b = operands(m, n, k)
    ad = torch.from_numpy(a).to(cuda).view(m, k)
    bd = torch.from_numpy(b).to(cuda).view(k, n)
    cd = torch.empty(m, n, device=cuda)
    lb.matmul_f32(ad, bd, cd, exact=True)
    assert np.array_equal(bits(cd.cpu().numpy().ravel()), bits(orc.matmul(m, n, k, a, b)))


@pytest.mark.parametrize("m,n,k", [(512, 512, 512), (384, 256, 1024), (100, 70, 33)])
def test_ffma_mode_within_tolerance(cuda, m, n, k):
    a, b = operands(m, n, k, seed=9)
    ad = torch.from_numpy(a).to(cuda).view(m, k)
    bd = torch.from_numpy(b).to(cuda).view(k, n)
    cd = torch.empty(m, n, device=cuda)
    lb.matmul_f32(ad, bd, cd, exact=False)
    assert rel(cd.cpu().numpy().ravel(), orc.matmul(m, n, k, a, b)) <= 1e-5


def test_full_size_rows_sampled(cuda):
    # 4096^3: the evaluator on a block of rows (the full product is 1.4e11 mul+add on the host).
    m = n = k = 4096
    a, b = operands(m, n, k, seed=4)
    ad = torch.from_numpy(a).to(cuda).view(m, k)
    bd = torch.from_numpy(b).to(cuda).view(k, n)
    for exact in (True, False):
        cd = torch.empty(m, n, device=cuda)
        lb.matmul_f32(ad, bd, cd, exact=exact)
        got = cd.cpu().numpy().ravel()
        rows = [(0, 8), (2048, 2056), (4088, 4096)]
        for r0, r1 in rows:
            want = orc.matmul(m, n, k, a, b, rows=(r0, r1))[r0 * n:r1 * n]
            g = got[r0 * n:r1 * n]
            if exact:
                assert np.array_equal(bits(g), bits(want)), (r0, r1)
            else:
                assert rel(g, want) <= 1e-5


def test_adr16_matmul_is_the_reference_order(cuda):
    for (m, n, k) in [(256, 128, 64), (33, 65, 17)]:
        a, b = operands(m, n, k, seed=12)
        ad, bd = torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)
        cd = torch.empty(m * n, device=cuda)
        assert adr16.launch("matmul", adr16.load("matmul"), m, n, k, ad.data_ptr(), bd.data_ptr(), cd.data_ptr()) == 0
        torch.cuda.synchronize()
        assert np.array_equal(bits(cd.cpu().numpy()), bits(orc.matmul(m, n, k, a, b))), (m, n, k)
