"""The bf16 tensor-core contraction (tcgen05): within the north star's 1e-2 relative of the host
evaluator's contraction on the bf16-rounded inputs (eval_contraction, p ascending), and of a
plain PyTorch fp32 product of the same rounded inputs. Relative = ||C - ref|| / ||ref||."""
import numpy as np
import pytest
import torch

import lyth_b200 as lb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TOL = 1e-2


def operands(m, n, k, seed):
    s = 1.0 / np.sqrt(k)
    a = orc.round_bf16(orc.normal(seed, m * k, 0.0, s))
    b = orc.round_bf16(orc.normal(seed + 1, k * n, 0.0, s))
    return a, b


def rel(got, want):
    got64, want64 = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.linalg.norm(got64 - want64) / np.linalg.norm(want64))


def run(m, n, k, a, b, cuda, pair=None):
    ad = torch.from_numpy(a).to(cuda).view(m, k).bfloat16()
    bd = torch.from_numpy(b).to(cuda).view(k, n).bfloat16()
    cd = torch.full((m, n), float("nan"), device=cuda)
    lb.matmul_bf16(ad, bd, cd, pair=pair)
    torch.cuda.synchronize()
    assert lb.lib.lyth_b200_device_error() == 0
    return ad, bd, cd


# Both forms: the single-SM kernel (any m multiple of 128) and the CTA-pair kernel (m multiple of
# 256), including more tiles than CTA pairs (4096 x 2048: 128 tiles of 256 x 256 on 74 pairs).
@pytest.mark.parametrize("m,n,k,pair", [(128, 256, 64, False), (256, 512, 128, False), (128, 256, 1024, False),
                                        (512, 768, 320, False), (256, 256, 64, True), (256, 512, 128, True),
                                        (512, 768, 320, True), (768, 256, 1024, True), (4096, 2048, 192, True)])
def test_small_shapes_against_the_evaluator(cuda, m, n, k, pair):
    a, b = operands(m, n, k, 70)
    ad, bd, cd = run(m, n, k, a, b, cuda, pair)
    got = cd.cpu().numpy().ravel()
    assert np.isfinite(got).all()
    if m * n * k <= 512 * 768 * 1024:
        assert rel(got, orc.matmul(m, n, k, a, b)) <= TOL
    ref = (ad.float() @ bd.float()).cpu().numpy().ravel()
    assert rel(got, ref) <= TOL


def test_pair_form_refuses_m_not_multiple_of_256(cuda):
    a = torch.zeros(128, 64, dtype=torch.bfloat16, device=cuda)
    b = torch.zeros(64, 256, dtype=torch.bfloat16, device=cuda)
    c = torch.zeros(128, 256, device=cuda)
    with pytest.raises(lb.LythError) as e:
        lb.matmul_bf16(a, b, c, pair=True)
    assert e.value.status == lb.E_UNSUPPORTED


@pytest.mark.parametrize("pair", [False, True])
def test_full_size_4096(cuda, pair):
    m = n = k = 4096
    a, b = operands(m, n, k, 4)
    ad, bd, cd = run(m, n, k, a, b, cuda, pair)
    got = cd.cpu().numpy().ravel()
    assert np.isfinite(got).all()
    ref = (ad.float() @ bd.float()).cpu().numpy().ravel()
    assert rel(got, ref) <= TOL
    for r0, r1 in [(0, 4), (1000, 1004), (4092, 4096)]:
        want = orc.matmul(m, n, k, a, b, rows=(r0, r1))[r0 * n:r1 * n]
        assert rel(got[r0 * n:r1 * n], want) <= TOL, (r0, r1)


def test_unsupported_shapes_are_refused(cuda):
    a = torch.zeros(100, 64, dtype=torch.bfloat16, device=cuda)
    b = torch.zeros(64, 256, dtype=torch.bfloat16, device=cuda)
    c = torch.zeros(100, 256, device=cuda)
    with pytest.raises(lb.LythError) as e:
        lb.matmul_bf16(a, b, c)
    assert e.value.status == lb.E_UNSUPPORTED


def test_pair_count_is_the_resident_clusters(cuda):
    # the pair form runs as many CTA pairs as fit at once: at most half the SMs, at least one
    p = int(lb.lib.lyth_b200_matmul_bf16_pairs())
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    assert 1 <= p <= sms // 2
