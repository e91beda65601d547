"""The state-vector engine (one GPU): whole circuits from seeded states, bit for bit against
the evaluator applying the same gates unfused (lyth-circuit's execute / run_fused_host)."""
import numpy as np
import pytest

import lyth_b200 as lb
from lyth_b200 import circuit as cc
from oracle import oracle as orc
from tests.conftest import bits

pytestmark = pytest.mark.gpu


as_tuples = cc.as_tuples


def run_engine(q, gates, re0, im0, fuse=6):
    with lb.StateVector(q, device=0) as sv:
        sv.set_fusion(fuse)
        sv.set_local(re0, im0)
        sv.apply(gates)
        sv.sync()
        gr, gi = np.empty_like(re0), np.empty_like(im0)
        sv.get_local(gr, gi)
        return gr, gi, sv.stats()


def suite():
    rng = cc.Rng(20_260_930)
    return [
        ("GHZ(12)", 12, cc.ghz(12)),
        ("QFT(10)", 10, cc.qft(10, rng)),
        ("random(10, depth 20)", 10, cc.random(10, 20, rng)),
        ("random(20, depth 10)", 20, cc.random(20, 10, cc.Rng(20_260_931))),
        ("layered(16, 4)", 16, cc.layered(16, 4, cc.Rng(cc.BENCH_SEED))),
        ("layered(22, 2)", 22, cc.layered(22, 2, cc.Rng(cc.BENCH_SEED))),
    ]


@pytest.mark.parametrize("case", range(6))
def test_circuits_bit_exact(cuda, case):
    name, q, gates = suite()[case]
    re0, im0 = orc.random_state(100 + case, q)
    wr, wi = orc.run_gates(as_tuples(gates), re0, im0)
    gr, gi, st = run_engine(q, gates, re0, im0)
    assert np.array_equal(bits(gr), bits(wr)), name
    assert np.array_equal(bits(gi), bits(wi)), name
    swaps = sum(isinstance(g, cc.Swap) for g in gates)
    assert st["passes"] <= len(gates) - swaps  # swaps are relabels; fused groups take one pass


@pytest.mark.parametrize("case", [1, 2, 3, 4, 5])
def test_fused_equals_unfused_at_every_k(cuda, case):
    # ADR-0030 Q1: a fused circuit is the unfused circuit, bit for bit, for every group size: the
    # register pass (k <= 6, states below 2^14) and the tile pass (k up to 13, 16 qubits and up).
    name, q, gates = suite()[case]
    re0, im0 = orc.random_state(200 + case, q)
    ur, ui, ust = run_engine(q, gates, re0, im0, fuse=1)
    passes = []
    for k in (2, 3, 4, 5, 6, 8, 10, 13):
        fr, fi, fst = run_engine(q, gates, re0, im0, fuse=k)
        assert np.array_equal(bits(fr), bits(ur)), (name, k)
        assert np.array_equal(bits(fi), bits(ui)), (name, k)
        passes.append(fst["passes"])
    assert passes == sorted(passes, reverse=True) and passes[-1] < ust["passes"], passes


def test_from_basis_zero_like_lyth_circuit(cuda):
    q = 12
    gates = cc.ghz(q)
    with lb.StateVector(q, device=0) as sv:
        sv.init_basis(0)
        sv.apply(gates)
        gr, gi = np.empty(1 << q, np.float32), np.empty(1 << q, np.float32)
        sv.get_local(gr, gi)
    re0 = np.zeros(1 << q, np.float32)
    re0[0] = 1.0
    wr, wi = orc.run_gates(as_tuples(gates), re0, np.zeros_like(re0))
    assert np.array_equal(bits(gr), bits(wr)) and np.array_equal(bits(gi), bits(wi))
    assert gr[0] == gr[-1] == np.float32(cc.S)


def test_init_random_matches_the_definition(cuda):
    q = 18
    with lb.StateVector(q, device=0) as sv:
        sv.init_random(77)
        gr, gi = np.empty(1 << q, np.float32), np.empty(1 << q, np.float32)
        sv.get_local(gr, gi)
    wr, wi = orc.random_state(77, q)
    assert np.array_equal(bits(gr), bits(wr)) and np.array_equal(bits(gi), bits(wi))
    norm = float(np.sum(gr.astype(np.float64) ** 2 + gi.astype(np.float64) ** 2))
    assert abs(norm - 1.0) < 1e-5


def test_unitarity_physics_check(cuda):
    # The check bit-exactness cannot see (unitary_gate.rs): U then U-dagger returns the state.
    q = 14
    m = cc.zyz(0.4, -1.1, 2.0)
    mdag = ((m[0][0], -m[0][1]), (m[2][0], -m[2][1]), (m[1][0], -m[1][1]), (m[3][0], -m[3][1]))
    gates = [cc.U(3, m), cc.CU(5, 9, m), cc.CU(5, 9, mdag), cc.U(3, mdag)]
    re0, im0 = orc.random_state(5, q)
    gr, gi, _ = run_engine(q, gates, re0, im0)
    assert np.max(np.abs(gr - re0)) < 1e-6 and np.max(np.abs(gi - im0)) < 1e-6


def on_bits(bits, n, rng):
    """n random U / CU gates whose qubits all lie in `bits` (so fusion makes one group of them)."""
    g = []
    for _ in range(n):
        t = bits[rng.below(len(bits))]
        m = cc.zyz(rng.angle(), rng.angle(), rng.angle())
        if len(bits) > 1 and rng.below(3):
            c = bits[rng.below(len(bits))]
            while c == t:
                c = bits[rng.below(len(bits))]
            g.append(cc.CU(c, t, m))
        else:
            g.append(cc.U(t, m))
    return g


# The tile pass (2^14 amplitudes and more): a group's bits are tile bits, its gates run in segments
# of at most five register levels (address bits 0 and 1 always among them), controls on register
# levels or as lane / warp predicates; up to 13 bits, at most 8 of them above bit 4, which makes
# the tile's boxes (ranges of consecutive bits, iterated beyond four ranges).
STAGED_BITS = [
    (0, 1, 2, 3, 4, 5), (10, 11, 12, 13, 14, 15), (5, 6, 7, 8, 9, 10), (1, 3, 7, 9, 12, 14),
    (0, 5, 6, 7, 8, 9), (2, 3, 4), (4, 13), (0,), (15,), (3, 4, 5, 6, 7),
    (0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12), (5, 6, 7, 8, 9, 10, 11, 12), (1, 2, 5, 7, 9, 11, 13, 15),
    (0, 2, 4, 6, 8, 10, 12, 14, 16, 18, 19), (3, 4, 6, 7, 17, 18, 19, 20, 21, 23),
]


@pytest.mark.parametrize("bits_", STAGED_BITS, ids=[",".join(map(str, b)) for b in STAGED_BITS])
def test_staged_groups_bit_exact(cuda, bits_):
    q = 16 if max(bits_) < 16 else 24
    gates = on_bits(bits_, 40, cc.Rng(hash(bits_) & 0xFFFF))
    re0, im0 = orc.random_state(500 + len(bits_), q)
    wr, wi = orc.run_gates(as_tuples(gates), re0, im0)
    gr, gi, st = run_engine(q, gates, re0, im0, fuse=13)
    assert np.array_equal(bits(gr), bits(wr)) and np.array_equal(bits(gi), bits(wi))
    assert st["passes"] == 1  # one fused group


def test_staged_ring_wraps_bit_exact(cuda):
    # 2^24 amplitudes: 2^11 tiles over at most 148 CTAs, so every CTA's 3-stage ring wraps.
    q = 24
    gates = cc.layered(q, 1, cc.Rng(cc.BENCH_SEED)) + on_bits((0, 1, 2, 20, 21, 22), 30, cc.Rng(9))
    re0, im0 = orc.random_state(600, q)
    wr, wi = orc.run_gates(as_tuples(gates), re0, im0)
    gr, gi, _ = run_engine(q, gates, re0, im0)
    assert np.array_equal(bits(gr), bits(wr)) and np.array_equal(bits(gi), bits(wi))
