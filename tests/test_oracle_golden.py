"""The oracle pinned against the reference's own golden vectors and known answers.

Every case here restates a reference test: half_rounding.rs (the device-measured vectors),
half.rs, eval.rs, ast.rs, inputs.rs unit tests, split_view.rs / two_qubit_gate.rs addressing,
and manifest.rs launch figures. No GPU.
"""
import json
import math
import os

import numpy as np
import pytest

from oracle import oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "half_vectors.json")


def _u2f(u):
    return float(np.array([u], np.uint32).view(np.float32)[0])


# ------------------------------------------------------------------ half_rounding.rs
def _nan_class(bits, exp_mask, mant_mask):
    return (bits & exp_mask) == exp_mask and (bits & mant_mask) != 0


def test_half_vectors_f16_bit_for_bit():
    vecs = json.load(open(GOLDEN))["vectors"]
    assert len(vecs) == 138
    for v in vecs:
        x = _u2f(v["f32"])
        got = orc.f32_to_f16_bits(x)
        if math.isnan(x):
            assert _nan_class(got, 0x7C00, 0x03FF) and _nan_class(v["f16"], 0x7C00, 0x03FF)
        else:
            assert got == v["f16"], f"f32 0x{v['f32']:08x}: oracle 0x{got:04x}, device 0x{v['f16']:04x}"


def test_half_vectors_bf16_bit_for_bit():
    for v in json.load(open(GOLDEN))["vectors"]:
        x = _u2f(v["f32"])
        got = orc.f32_to_bf16_bits(x)
        if math.isnan(x):
            assert _nan_class(got, 0x7F80, 0x007F) and _nan_class(v["bf16"], 0x7F80, 0x007F)
        else:
            assert got == v["bf16"], f"f32 0x{v['f32']:08x}: oracle 0x{got:04x}, device 0x{v['bf16']:04x}"


# ------------------------------------------------------------------ half.rs unit tests
def round_f16(x):
    return orc.f16_bits_to_f32(orc.f32_to_f16_bits(x))


def test_ties_round_to_even():
    assert round_f16(2049.0) == 2048.0
    assert round_f16(2051.0) == 2052.0
    assert round_f16(2050.0) == 2050.0


def test_overflow_goes_to_infinity():
    assert round_f16(65504.0) == 65504.0
    assert math.isinf(round_f16(65520.0))
    assert math.isinf(round_f16(70000.0))
    assert math.isfinite(float(orc.round_bf16(np.float32([70000.0]))[0]))


def test_subnormals_not_flushed():
    tiny = 2.0 ** -24
    assert round_f16(tiny) == tiny
    assert round_f16(tiny * 0.4) == 0.0
    assert round_f16(tiny * 0.6) == tiny


def test_sign_survives_zero():
    assert math.copysign(1.0, round_f16(-0.0)) < 0
    assert math.copysign(1.0, float(orc.round_bf16(np.float32([-0.0]))[0])) < 0


# ------------------------------------------------------------------ eval.rs known answers
def test_saxpy_computes_saxpy():
    y = orc.saxpy(2.0, [1.0, 2.0, 3.0], [10.0, 20.0, 30.0])
    assert y.tolist() == [12.0, 24.0, 36.0]


def test_the_reference_fuses_exactly_as_the_generated_code_does():
    # The reference's case (eval.rs:596-608): y must be a.mul_add(x, y).
    eps = float(np.finfo(np.float32).eps)
    a = x = np.float32(1.0 + eps)
    y = orc.saxpy(float(a), [float(x)], [-1.0])[0]
    assert y == float(np.float32(float(a) * float(x) + -1.0))  # exact product, one rounding
    # And one where one rounding and two differ: (1 + 2^-12)^2 - (1 + 2^-11) = 2^-24 fused, 0 unfused.
    a = x = np.float32(1.0 + 2.0 ** -12)
    c = np.float32(-(1.0 + 2.0 ** -11))
    y = orc.saxpy(float(a), [float(x)], [float(c)])[0]
    fused = float(np.float32(float(a) * float(x) + float(c)))
    unfused = float(np.float32(np.float32(a * x) + c))
    assert fused == 2.0 ** -24 and unfused == 0.0
    assert y == fused


def test_tree_computes_the_dot_product():
    x = np.array([float(1 << i) for i in range(8)], np.float32)
    p = orc.reduce(orc.SUM, x, np.ones(8, np.float32), grid=1, block=8)
    assert p[0] == 255.0


def test_ragged_tail_contributes_identity():
    p = orc.reduce(orc.SUM, np.ones(10, np.float32), np.ones(10, np.float32), grid=3, block=4)
    assert p.tolist() == [4.0, 4.0, 2.0]


def test_tree_order_not_left_fold():
    big = 1.0e8
    x = np.array([big, 1.0, -big, 1.0], np.float32)
    p = orc.reduce(orc.SUM, x, np.ones(4, np.float32), grid=1, block=4)
    assert p[0] == 2.0  # (x0 + x2) + (x1 + x3); the left fold gives 1.0


def test_two_stage_order_depends_on_grid_and_block():
    x = orc.uniform(11, 5000) * np.float32(1e4)
    a = orc.reduce(orc.SUM, x, grid=3, block=256)
    b = orc.reduce(orc.SUM, x, grid=3, block=128)
    assert a.shape == (3,) and b.shape == (3,)
    assert float(np.sum(a.astype(np.float64))) == pytest.approx(orc.sum_f64(x), rel=1e-5)


def test_zero_block_is_refused():
    with pytest.raises(ValueError):
        orc.reduce(orc.SUM, np.ones(4, np.float32), grid=1, block=0)


# ------------------------------------------------------------------ ast.rs
def test_combine_orders_signed_zeros_the_way_the_hardware_does():
    def neg(v):
        return math.copysign(1.0, v) < 0

    assert not neg(orc.combine(orc.MAX, -0.0, 0.0))
    assert not neg(orc.combine(orc.MAX, 0.0, -0.0))
    assert neg(orc.combine(orc.MIN, -0.0, 0.0))
    assert neg(orc.combine(orc.MIN, 0.0, -0.0))
    assert neg(orc.combine(orc.MAX, -0.0, -0.0))
    assert not neg(orc.combine(orc.MIN, 0.0, 0.0))


def test_combine_returns_the_non_nan_operand():
    assert orc.combine(orc.MAX, float("nan"), 3.0) == 3.0
    assert orc.combine(orc.MAX, 3.0, float("nan")) == 3.0
    assert math.isnan(orc.combine(orc.MAX, float("nan"), float("nan")))


def test_identity_cannot_win():
    assert orc.combine(orc.MAX, orc.identity(orc.MAX), -1e30) == np.float32(-1e30)
    assert orc.combine(orc.MIN, orc.identity(orc.MIN), 1e30) == np.float32(1e30)
    assert orc.combine(orc.SUM, orc.identity(orc.SUM), 7.0) == 7.0


# ------------------------------------------------------------------ inputs.rs
def test_two_buffers_get_different_data():
    for a, b in [("x", "y"), ("a", "b"), ("b", "c")]:
        same = int(np.sum(orc.buffer(a, orc.TY_F32, 4096) == orc.buffer(b, orc.TY_F32, 4096)))
        assert same < 4096 // 100


def test_seed_of_and_range():
    assert orc.seed_of("x") == 31 + ord("x")
    v = orc.buffer("x", orc.TY_F32, 1024)
    assert np.all((v >= -4.0) & (v < 4.0))
    h = orc.buffer("x", orc.TY_F16, 64)
    assert np.array_equal(h, np.array([round_f16(float(t)) for t in h], np.float32))


# ------------------------------------------------------------------ SplitMix64 (lib.rs:418-433)
def test_splitmix64_known_outputs():
    # SplitMix64 from state 0: the published first outputs of the generator.
    assert orc.splitmix_at(0, 0) == 0xE220A8397B1DCDAF
    assert orc.splitmix_at(0, 1) == 0x6E789E6AA1B965F4
    assert orc.splitmix_at(0, 2) == 0x06C45D188009454F


def test_uniform_range():
    u = orc.uniform(20260930, 100000)
    assert u.min() >= -1.0 and u.max() < 1.0
    assert abs(float(u.mean())) < 0.01


# ------------------------------------------------------------------ split addressing
def _insert_zero(k, b):
    low = k & ((1 << b) - 1)
    return ((k >> b) << (b + 1)) | low


def test_every_leaf_holds_exactly_the_amplitudes_its_two_bits_name():
    q = 7
    n = 1 << q
    pairs = 0
    for c in range(q):
        for t in range(q):
            if c == t:
                continue
            wc, wt = orc.widths_ct(c, t)
            lo, hi = min(c, t), max(c, t)
            seen = np.zeros(n, bool)
            for x, y in [(0, 0), (0, 1), (1, 0), (1, 1)]:
                for kk in range(n // 4):
                    got = orc.view_index(wc, x, orc.view_index(wt, y, kk))
                    want = _insert_zero(_insert_zero(kk, lo), hi) | (x << c) | (y << t)
                    assert got == want
                    assert not seen[got]
                    seen[got] = True
            assert seen.all()
            pairs += 1
    assert pairs == 42


def test_depth_one_view_index_any_width():
    # hadamard_q at n = 96, w = 3 walks 48 pairs covering every element once.
    seen = sorted(orc.view_index(3, p, k) for p in (0, 1) for k in range(48))
    assert seen == list(range(96))


def test_gate_chains_against_a_dense_reference():
    # two_qubit_gate.rs: leaves built from the physics (bits), the formula in fma order.
    rng = np.random.default_rng(5)
    n, c, t = 64, 4, 1
    re = rng.standard_normal(n).astype(np.float32)
    im = rng.standard_normal(n).astype(np.float32)
    m = np.array([0.3, -0.2, 0.9, 0.1, -0.4, 0.7, 0.2, -0.5], np.float32)
    wc, wt = orc.widths_ct(c, t)
    qr, qi = orc.cu_q(wc, wt, m, re, im)
    ar, ai, br, bi, cr, ci, dr, di = [np.float32(v) for v in m]

    def fma(a, b, cc):
        return np.float32(float(a) * float(b) + float(cc))  # exact in f64 for these f32 values

    for i in range(n):
        if (i >> c) & 1 == 0:
            assert qr[i] == re[i] and qi[i] == im[i]
        elif (i >> t) & 1 == 0:
            j = i | (1 << t)
            p0r, p0i, p1r, p1i = re[i], im[i], re[j], im[j]
            assert qr[i] == fma(ar, p0r, fma(-ai, p0i, fma(br, p1r, np.float32(-bi * p1i))))
            assert qi[i] == fma(ar, p0i, fma(ai, p0r, fma(br, p1i, np.float32(bi * p1r))))
            assert qr[j] == fma(cr, p0r, fma(-ci, p0i, fma(dr, p1r, np.float32(-di * p1i))))
            assert qi[j] == fma(cr, p0i, fma(ci, p0r, fma(dr, p1i, np.float32(di * p1r))))


def test_split_refusals():
    with pytest.raises(ValueError):
        orc.gate_q(0, np.zeros(8, np.float32), np.zeros(12, np.float32), np.zeros(12, np.float32))
    with pytest.raises(ValueError):
        orc.gate_q(4, np.zeros(8, np.float32), np.zeros(12, np.float32), np.zeros(12, np.float32))


# ------------------------------------------------------------------ contraction order
def test_contraction_is_ascending_mul_then_add():
    a = np.array([[1e8, 1.0, -1e8, 1.0]], np.float32)
    b = np.ones((4, 1), np.float32)
    c = orc.matmul(1, 1, 4, a, b)
    assert c[0] == 1.0  # ((1e8 + 1) - 1e8) + 1, not the tree's 2.0


# ------------------------------------------------------------------ NF4 (format of this project)
def test_nf4_codebook_is_the_published_construction():
    from scipy.stats import norm

    offset = 0.9677083
    v1 = norm.ppf(np.linspace(offset, 0.5, 9)[:-1]).tolist()
    v3 = (-norm.ppf(np.linspace(offset, 0.5, 8)[:-1])).tolist()
    v = np.array(sorted(v1 + [0.0] + v3))
    v /= v.max()
    assert np.array_equal(orc.nf4_codebook(), v.astype(np.float32))


def test_int4_dequant_is_exact_and_signed():
    rows, k, group = 2, 64, 64
    w = np.arange(rows * k // 2, dtype=np.uint8)  # every nibble pattern appears
    scales = orc.to_f16_bits(np.array([0.5, 0.25], np.float32))
    d = orc.gemv_dequant(0, rows, k, group, w, scales).reshape(rows, k)
    nib = np.empty(rows * k, np.int32)
    nib[0::2] = w & 0xF
    nib[1::2] = w >> 4
    q = np.where(nib >= 8, nib - 16, nib).reshape(rows, k)
    assert np.array_equal(d, (q * np.array([[0.5], [0.25]])).astype(np.float32))
