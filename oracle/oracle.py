"""ctypes wrapper over liblythref.so, the CPU restatement of LYTH's host IR evaluator.

TEST INFRASTRUCTURE ONLY. This module is the checker: tests/, ``__graft_entry__.smoke()``
and bench.py's CPU-baseline leg import it, and nothing in the ``lyth_b200`` package may.
Each function names the reference routine it restates (paths inside QuantumDrizzy/LYTH).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "liblythref.so")

_F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_F64P = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_U16P = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_U8P = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")

SUM, MAX, MIN = 0, 1, 2
TY_F32, TY_F16, TY_BF16 = 0, 1, 2


def build() -> str:
    """Compile liblythref.so with oracle/Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def _load() -> C.CDLL:
    if not os.path.exists(_SO):
        build()
    lib = C.CDLL(_SO)
    u64, u32, f32, i32 = C.c_uint64, C.c_uint32, C.c_float, C.c_int
    sig = {
        "lr_f32_to_f16_bits": (C.c_uint16, [f32]),
        "lr_f16_bits_to_f32": (f32, [C.c_uint16]),
        "lr_f32_to_bf16_bits": (C.c_uint16, [f32]),
        "lr_bf16_bits_to_f32": (f32, [C.c_uint16]),
        "lr_round_bf16_array": (None, [u64, _F32P, _F32P]),
        "lr_f32_to_f16_array": (None, [u64, _F32P, _U16P]),
        "lr_f32_to_bf16_array": (None, [u64, _F32P, _U16P]),
        "lr_seed_of": (u32, [C.c_char_p]),
        "lr_element": (f32, [C.c_char_p, i32, u32]),
        "lr_buffer": (None, [C.c_char_p, i32, u32, _F32P]),
        "lr_splitmix_next": (u64, [C.POINTER(u64)]),
        "lr_splitmix_at": (u64, [u64, u64]),
        "lr_uniform": (None, [u64, u64, _F32P]),
        "lr_normal": (None, [u64, u64, C.c_double, C.c_double, _F32P]),
        "lr_identity": (f32, [i32]),
        "lr_combine": (f32, [i32, f32, f32]),
        "lr_saxpy": (None, [u64, f32, _F32P, _F32P]),
        "lr_axpby": (None, [u64, f32, f32, _F32P, _F32P]),
        "lr_lerp": (None, [u64, f32, _F32P, _F32P, _F32P]),
        "lr_horner": (None, [u64, f32, f32, f32, f32, _F32P, _F32P]),
        "lr_copy2d": (None, [u32, u32, _F32P, _F32P]),
        "lr_transpose": (None, [u32, u32, _F32P, _F32P]),
        "lr_reduce": (i32, [i32, u64, _F32P, C.c_void_p, u32, u32, _F32P]),
        "lr_sum_f64": (C.c_double, [u64, _F32P, C.c_void_p]),
        "lr_matmul": (None, [u32, u32, u32, _F32P, _F32P, _F32P, u32, u32]),
        "lr_view_index": (u64, [u64, u32, u64]),
        "lr_hadamard_q": (i32, [u64, u64, f32, _F32P, _F32P, _F32P, _F32P]),
        "lr_gate_q": (i32, [u64, u64, _F32P, _F32P, _F32P, _F32P, _F32P]),
        "lr_cu_q": (i32, [u64, u64, u64, _F32P, _F32P, _F32P, _F32P, _F32P]),
        "lr_swap_q": (i32, [u64, u64, u64, _F32P, _F32P, _F32P, _F32P]),
        "lr_nf4_codebook": (None, [_F32P]),
        "lr_gemv_dequant": (None, [i32, u32, u32, u32, _U8P, _U16P, _F32P]),
        "lr_gemv_f64": (None, [i32, u32, u32, u32, _U8P, _U16P, _U16P, _F64P]),
        "lr_threads": (i32, []),
        "lr_set_threads": (None, [i32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- half.rs
def f32_to_f16_bits(x: float) -> int:
    return int(LIB.lr_f32_to_f16_bits(x))


def f32_to_bf16_bits(x: float) -> int:
    return int(LIB.lr_f32_to_bf16_bits(x))


def f16_bits_to_f32(h: int) -> float:
    return float(LIB.lr_f16_bits_to_f32(h))


def to_f16_bits(a) -> np.ndarray:
    a = _f32(a)
    out = np.empty(a.shape, np.uint16)
    LIB.lr_f32_to_f16_array(a.size, a.ravel(), out.ravel())
    return out


def to_bf16_bits(a) -> np.ndarray:
    a = _f32(a)
    out = np.empty(a.shape, np.uint16)
    LIB.lr_f32_to_bf16_array(a.size, a.ravel(), out.ravel())
    return out


def round_bf16(a) -> np.ndarray:
    a = _f32(a)
    out = np.empty_like(a)
    LIB.lr_round_bf16_array(a.size, a.ravel(), out.ravel())
    return out


def f16_bits_to_f32_array(h) -> np.ndarray:
    """Exact widening (every binary16 is an f32); numpy's float16 agrees with half.rs here."""
    return np.asarray(h, np.uint16).view(np.float16).astype(np.float32)


# ---------------------------------------------------------------- inputs.rs / Rng
def seed_of(name: str) -> int:
    return int(LIB.lr_seed_of(name.encode()))


def buffer(name: str, ty: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    LIB.lr_buffer(name.encode(), ty, n, out)
    return out


def splitmix_at(seed: int, i: int) -> int:
    return int(LIB.lr_splitmix_at(seed, i))


def uniform(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    LIB.lr_uniform(seed, n, out)
    return out


def normal(seed: int, n: int, mu: float, sigma: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    LIB.lr_normal(seed, n, mu, sigma, out)
    return out


# ---------------------------------------------------------------- ast.rs
def identity(op: int) -> float:
    return float(LIB.lr_identity(op))


def combine(op: int, a: float, b: float) -> float:
    return float(LIB.lr_combine(op, a, b))


# ---------------------------------------------------------------- elementwise (eval.rs)
def saxpy(a: float, x, y) -> np.ndarray:
    y = _f32(y).copy()
    LIB.lr_saxpy(y.size, a, _f32(x), y)
    return y


def axpby(a: float, b: float, x, y) -> np.ndarray:
    y = _f32(y).copy()
    LIB.lr_axpby(y.size, a, b, _f32(x), y)
    return y


def lerp(t: float, x, y) -> np.ndarray:
    x = _f32(x)
    z = np.empty_like(x)
    LIB.lr_lerp(x.size, t, x, _f32(y), z)
    return z


def horner(c0, c1, c2, c3, x) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    LIB.lr_horner(x.size, c0, c1, c2, c3, x, y)
    return y


def copy2d(rows: int, cols: int, a) -> np.ndarray:
    b = np.empty(rows * cols, np.float32)
    LIB.lr_copy2d(rows, cols, _f32(a).ravel(), b)
    return b


def transpose(rows: int, cols: int, a) -> np.ndarray:
    b = np.empty(rows * cols, np.float32)
    LIB.lr_transpose(rows, cols, _f32(a).ravel(), b)
    return b


# ---------------------------------------------------------------- reductions
def reduce(op: int, x, y=None, *, grid: int, block: int = 256) -> np.ndarray:
    x = _f32(x)
    yv = None if y is None else _f32(y)
    out = np.empty(grid, np.float32)
    rc = LIB.lr_reduce(op, x.size, x, None if yv is None else yv.ctypes.data, grid, block, out)
    if rc != 0:
        raise ValueError("a block of zero threads reduces nothing")
    return out


def sum_f64(x, y=None) -> float:
    x = _f32(x)
    yv = None if y is None else _f32(y)
    return float(LIB.lr_sum_f64(x.size, x, None if yv is None else yv.ctypes.data))


# ---------------------------------------------------------------- contraction
def matmul(m: int, n: int, k: int, a, b, rows: tuple[int, int] | None = None) -> np.ndarray:
    r0, r1 = rows if rows else (0, m)
    c = np.zeros(m * n, np.float32)
    LIB.lr_matmul(m, n, k, _f32(a).ravel(), _f32(b).ravel(), c, r0, r1)
    return c


# ---------------------------------------------------------------- split views + gates
def view_index(w: int, part: int, k: int) -> int:
    return int(LIB.lr_view_index(w, part, k))


def widths_ct(c: int, t: int) -> tuple[int, int]:
    """lyth-circuit/src/lib.rs:387-389."""
    return 1 << c, (1 << t) if t < c else (1 << (t - 1))


def _gate_io(re, im, inplace):
    re, im = _f32(re), _f32(im)
    if inplace:
        return re, im, re, im
    return re, im, np.empty_like(re), np.empty_like(im)


def hadamard_q(w: int, s: float, re, im, inplace=False):
    re, im, qr, qi = _gate_io(re, im, inplace)
    if LIB.lr_hadamard_q(re.size, w, s, re, im, qr, qi):
        raise ValueError(f"split refused: 2*w={2 * w} must divide n={re.size}")
    return qr, qi


def gate_q(w: int, m8, re, im, inplace=False):
    re, im, qr, qi = _gate_io(re, im, inplace)
    if LIB.lr_gate_q(re.size, w, _f32(m8), re, im, qr, qi):
        raise ValueError(f"split refused: 2*w={2 * w} must divide n={re.size}")
    return qr, qi


def cu_q(wc: int, wt: int, m8, re, im, inplace=False):
    re, im, qr, qi = _gate_io(re, im, inplace)
    if LIB.lr_cu_q(re.size, wc, wt, _f32(m8), re, im, qr, qi):
        raise ValueError("split refused")
    return qr, qi


def swap_q(wc: int, wt: int, re, im, inplace=False):
    re, im, qr, qi = _gate_io(re, im, inplace)
    if LIB.lr_swap_q(re.size, wc, wt, re, im, qr, qi):
        raise ValueError("split refused")
    return qr, qi


# ---------------------------------------------------------------- GEMV (unpinned)
def nf4_codebook() -> np.ndarray:
    out = np.empty(16, np.float32)
    LIB.lr_nf4_codebook(out)
    return out


def gemv_dequant(fmt: int, rows: int, k: int, group: int, w, scales) -> np.ndarray:
    out = np.empty(rows * k, np.float32)
    LIB.lr_gemv_dequant(fmt, rows, k, group, np.ascontiguousarray(w, np.uint8),
                        np.ascontiguousarray(scales, np.uint16), out)
    return out


def gemv_f64(fmt: int, rows: int, k: int, group: int, w, scales, x16) -> np.ndarray:
    out = np.empty(rows, np.float64)
    LIB.lr_gemv_f64(fmt, rows, k, group, np.ascontiguousarray(w, np.uint8),
                    np.ascontiguousarray(scales, np.uint16), np.ascontiguousarray(x16, np.uint16), out)
    return out


def threads() -> int:
    return int(LIB.lr_threads())


def set_threads(n: int) -> None:
    LIB.lr_set_threads(n)


# ---------------------------------------------------------------- circuits (unfused, in order)
def run_gates(gates, re, im, inplace=False):
    """Apply (kind, q0, q1, m8) gates in order, the unfused way lyth-circuit's execute does:
    kind 0 = gate_q on width 2^q0; 1 = cu_q with widths_ct(q0, q1); 2 = swap_q likewise.
    Returns new (re, im); the inputs are not modified unless `inplace` (then they must be
    contiguous f32 arrays, and are returned)."""
    if inplace:
        if not (isinstance(re, np.ndarray) and re.dtype == np.float32 and re.flags.c_contiguous
                and isinstance(im, np.ndarray) and im.dtype == np.float32 and im.flags.c_contiguous):
            raise ValueError("run_gates(inplace=True) needs contiguous float32 arrays")
    else:
        re = _f32(re).copy()
        im = _f32(im).copy()
    for kind, q0, q1, m8 in gates:
        if kind == 0:
            re, im = gate_q(1 << q0, m8, re, im, inplace=True)
        elif kind == 1:
            wc, wt = widths_ct(q0, q1)
            re, im = cu_q(wc, wt, m8, re, im, inplace=True)
        elif kind == 2:
            wc, wt = widths_ct(q0, q1)
            re, im = swap_q(wc, wt, re, im, inplace=True)
        else:
            raise ValueError(f"gate kind {kind}")
    return re, im


def random_state(seed: int, qubits: int):
    """re/im from the SplitMix64 stream (re: output 2i, im: 2i+1), U[-1, 1), scaled by
    1/sqrt(sum |a|^2) computed in f64 and applied in f32."""
    n = 1 << qubits
    both = uniform(seed, 2 * n)
    re = np.ascontiguousarray(both[0::2])
    im = np.ascontiguousarray(both[1::2])
    norm2 = float(np.sum(re.astype(np.float64) ** 2) + np.sum(im.astype(np.float64) ** 2))
    f = np.float32(1.0 / np.sqrt(norm2))
    return (re * f).astype(np.float32), (im * f).astype(np.float32)
