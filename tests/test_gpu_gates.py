"""State-vector gate passes vs the evaluator's lowered bodies, bit for bit, at every qubit
position and every ordered pair of a 10-qubit register, in and out of place; plus widths that
are not powers of two (the reference's general view_index) and the ADR-0016 launches."""
import numpy as np
import pytest
import torch

import lyth_b200 as lb
from lyth_b200 import circuit as cc
from oracle import oracle as orc
from tests import adr16
from tests.conftest import bits

pytestmark = pytest.mark.gpu

Q = 10
N = 1 << Q
ZYZ = cc.f32s(cc.zyz(0.7, 1.9, -2.3))


def state(seed, n=N):
    return orc.uniform(seed, n), orc.uniform(seed + 1, n)


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("inplace", [True, False])
def test_gate_q_every_qubit(cuda, inplace):
    re, im = state(1)
    for q in range(Q):
        w = 1 << q
        wr, wi = orc.gate_q(w, ZYZ, re, im)
        rd, idd = dev(re, cuda), dev(im, cuda)
        if inplace:
            lb.gate(w, ZYZ, rd, idd)
            gr, gi = rd, idd
        else:
            gr, gi = torch.empty_like(rd), torch.empty_like(idd)
            lb.gate(w, ZYZ, rd, idd, gr, gi)
        assert np.array_equal(bits(gr.cpu().numpy()), bits(wr)), q
        assert np.array_equal(bits(gi.cpu().numpy()), bits(wi)), q


def test_hadamard_every_qubit(cuda):
    re, im = state(3)
    s = float(np.float32(cc.S))
    for q in range(Q):
        wr, wi = orc.hadamard_q(1 << q, s, re, im)
        rd, idd = dev(re, cuda), dev(im, cuda)
        lb.hadamard(1 << q, s, rd, idd)
        assert np.array_equal(bits(rd.cpu().numpy()), bits(wr)), q
        assert np.array_equal(bits(idd.cpu().numpy()), bits(wi)), q


@pytest.mark.parametrize("inplace", [True, False])
@pytest.mark.parametrize("kind", ["cu", "swap"])
def test_two_qubit_every_ordered_pair(cuda, kind, inplace):
    re, im = state(5)
    for c in range(Q):
        for t in range(Q):
            if c == t:
                continue
            wc, wt = orc.widths_ct(c, t)
            rd, idd = dev(re, cuda), dev(im, cuda)
            gr, gi = (rd, idd) if inplace else (torch.empty_like(rd), torch.empty_like(idd))
            if kind == "cu":
                wr, wi = orc.cu_q(wc, wt, ZYZ, re, im)
                lb.cu(wc, wt, ZYZ, rd, idd, gr, gi)
            else:
                wr, wi = orc.swap_q(wc, wt, re, im)
                lb.swap(wc, wt, rd, idd, gr, gi)
            assert np.array_equal(bits(gr.cpu().numpy()), bits(wr)), (c, t)
            assert np.array_equal(bits(gi.cpu().numpy()), bits(wi)), (c, t)


def test_widths_that_are_not_powers_of_two(cuda):
    # hadamard_q at n = 96, w = 3 (split_view.rs depth_one_is_unchanged), cu/swap at (6, 4) on 96.
    n = 96
    re, im = state(7, n)
    wr, wi = orc.gate_q(3, ZYZ, re, im)
    rd, idd = dev(re, cuda), dev(im, cuda)
    lb.gate(3, ZYZ, rd, idd)
    assert np.array_equal(bits(rd.cpu().numpy()), bits(wr))
    assert np.array_equal(bits(idd.cpu().numpy()), bits(wi))
    for kind in ("cu", "swap"):
        rd, idd = dev(re, cuda), dev(im, cuda)
        gr, gi = torch.empty_like(rd), torch.empty_like(idd)
        if kind == "cu":
            wr, wi = orc.cu_q(6, 4, ZYZ, re, im)
            lb.cu(6, 4, ZYZ, rd, idd, gr, gi)
        else:
            wr, wi = orc.swap_q(6, 4, re, im)
            lb.swap(6, 4, rd, idd, gr, gi)
        assert np.array_equal(bits(gr.cpu().numpy()), bits(wr)), kind
        assert np.array_equal(bits(gi.cpu().numpy()), bits(wi)), kind


def test_refused_split_runs_nothing(cuda):
    rd = torch.full((12,), 5.0, device=cuda)
    idd = torch.full((12,), 5.0, device=cuda)
    with pytest.raises(lb.LythError) as e:
        lb.gate(4, ZYZ, rd, idd)
    assert e.value.status == lb.E_SPLIT
    assert torch.all(rd == 5.0)


def test_adr16_gate_launches(cuda):
    n = 1 << 12
    re, im = state(9, n)
    rd, idd = dev(re, cuda), dev(im, cuda)
    qr, qi = torch.empty_like(rd), torch.empty_like(idd)
    fn = adr16.load("gate_q")
    assert adr16.launch("gate_q", fn, n, 8, *ZYZ, rd.data_ptr(), idd.data_ptr(), qr.data_ptr(), qi.data_ptr()) == 0
    torch.cuda.synchronize()
    wr, wi = orc.gate_q(8, ZYZ, re, im)
    assert np.array_equal(bits(qr.cpu().numpy()), bits(wr)) and np.array_equal(bits(qi.cpu().numpy()), bits(wi))
    # A refused width returns CUDA_ERROR_INVALID_VALUE (1) and writes nothing.
    qr.fill_(7.0)
    assert adr16.launch("gate_q", fn, n, 3, *ZYZ, rd.data_ptr(), idd.data_ptr(), qr.data_ptr(), qi.data_ptr()) == 1
    torch.cuda.synchronize()
    assert torch.all(qr == 7.0)
    wc, wt = orc.widths_ct(2, 9)
    assert adr16.launch("cu_q", adr16.load("cu_q"), n, wc, wt, *ZYZ, rd.data_ptr(), idd.data_ptr(), qr.data_ptr(),
                        qi.data_ptr()) == 0
    torch.cuda.synchronize()
    wr, wi = orc.cu_q(wc, wt, ZYZ, re, im)
    assert np.array_equal(bits(qr.cpu().numpy()), bits(wr)) and np.array_equal(bits(qi.cpu().numpy()), bits(wi))
    assert adr16.launch("swap_q", adr16.load("swap_q"), n, wc, wt, rd.data_ptr(), idd.data_ptr(), qr.data_ptr(),
                        qi.data_ptr()) == 0
    s = float(np.float32(cc.S))
    torch.cuda.synchronize()
    wr, wi = orc.swap_q(wc, wt, re, im)
    assert np.array_equal(bits(qr.cpu().numpy()), bits(wr)) and np.array_equal(bits(qi.cpu().numpy()), bits(wi))
    assert adr16.launch("hadamard_q", adr16.load("hadamard_q"), n, 1, s, rd.data_ptr(), idd.data_ptr(),
                        qr.data_ptr(), qi.data_ptr()) == 0
    torch.cuda.synchronize()
    wr, wi = orc.hadamard_q(1, s, re, im)
    assert np.array_equal(bits(qr.cpu().numpy()), bits(wr)) and np.array_equal(bits(qi.cpu().numpy()), bits(wi))
