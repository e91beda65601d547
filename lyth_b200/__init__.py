"""lyth_b200: a B200 (sm_100a) execution back end for the kernel classes LYTH lowers to.

The product is ``liblyth_b200.so`` (CUDA kernels + C ABI, ``include/lyth_b200.h``). This
module is the Python host side over that ABI, mirroring how LYTH's generated ctypes bindings
(crates/lyth/src/bind_py.rs) and the ``lyth run`` launcher (crates/lyth/src/main.rs:1320-1499)
call a kernel: the caller owns device memory (here: torch CUDA tensors or raw device
pointers), the call launches on a stream, and a refused launch raises with the reason.

There is no CPU fallback. If the library is missing the import fails; without a GPU every call
raises the CUDA error the library returns.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblyth_b200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is not built: run `python lyth_b200/build.py` (nvcc, sm_100a). "
        "lyth_b200 has no CPU fallback."
    )

lib = C.CDLL(LIB_PATH)

# Status codes (include/lyth_b200.h).
OK = 0
E_SPLIT = -1
E_UNSUPPORTED = -2
E_INVALID = -3
E_TIMEOUT = -4
E_NCCL = -5
E_NO_NCCL = -6
E_OOM = -7

SUM, MAX, MIN = 0, 1, 2
GEMV_INT4, GEMV_NF4 = 0, 1
GATE_U, GATE_CU, GATE_SWAP = 0, 1, 2


class LythError(RuntimeError):
    """A refused or failed launch: ``status`` is the library's code (see include/lyth_b200.h)."""

    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = lib.lyth_b200_error_string(status).decode()
        super().__init__(f"{what}: {msg} (status {status})" if what else f"{msg} (status {status})")


_u32, _u64, _f32, _i32, _vp = C.c_uint32, C.c_uint64, C.c_float, C.c_int, C.c_void_p


class Gate(C.Structure):
    """``lyth_gate``: kind (U / CU / SWAP), q0, q1, m = ar ai br bi cr ci dr di."""

    _fields_ = [("kind", _u32), ("q0", _u32), ("q1", _u32), ("m", _f32 * 8)]


SV_OP_U, SV_OP_CU, SV_OP_FUSED, SV_OP_EXCHANGE = 0, 1, 2, 3
SV_OP_SWAP_LOCAL, SV_OP_SWAP_LR, SV_OP_SWAP_RR, SV_OP_SWAP_MULTI, SV_OP_PERMUTE = 4, 5, 6, 7, 8


class SvOp(C.Structure):
    """``lyth_sv_op``: one step a plan handle recorded (include/lyth_b200.h)."""

    _fields_ = [("kind", C.c_int32), ("a", C.c_int32), ("b", C.c_int32), ("c", C.c_int32),
                ("m", _f32 * 8), ("k", C.c_int32), ("bits", _u32 * 13), ("rbits", _u32 * 13), ("ngates", _u32),
                ("gt", C.c_int8 * 48), ("gc", C.c_int8 * 48), ("gm", (_f32 * 8) * 48)]


def _sig(name, res, args):
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = args
    return fn


_sig("lyth_b200_error_string", C.c_char_p, [_i32])
_sig("lyth_b200_version", _i32, [])
_sig("lyth_b200_saxpy", _i32, [_u64, _f32, _vp, _vp, _vp])
_sig("lyth_b200_axpby", _i32, [_u64, _f32, _f32, _vp, _vp, _vp])
_sig("lyth_b200_lerp", _i32, [_u64, _f32, _vp, _vp, _vp, _vp])
_sig("lyth_b200_horner", _i32, [_u64, _f32, _f32, _f32, _f32, _vp, _vp, _vp])
_sig("lyth_b200_copy2d", _i32, [_u32, _u32, _vp, _vp, _vp])
_sig("lyth_b200_transpose_naive", _i32, [_u32, _u32, _vp, _vp, _vp])
_sig("lyth_b200_transpose_tiled", _i32, [_u32, _u32, _vp, _vp, _vp])
_sig("lyth_b200_reduce_grid", _u32, [_u64])
_sig("lyth_b200_reduce_partials", _i32, [_i32, _u64, _vp, _vp, _u32, _vp, _vp])
_sig("lyth_b200_reduce_workspace_bytes", C.c_size_t, [_u64])
_sig("lyth_b200_reduce", _i32, [_i32, _u64, _vp, _vp, _vp, _vp, C.c_size_t, _vp])
_sig("lyth_b200_matmul_f32", _i32, [_u32, _u32, _u32, _vp, _vp, _vp, _i32, _vp])
_sig("lyth_b200_matmul_bf16", _i32, [_u32, _u32, _u32, _vp, _vp, _vp, _vp])
_sig("lyth_b200_matmul_bf16_form", _i32, [_i32, _u32, _u32, _u32, _vp, _vp, _vp, _vp])
_sig("lyth_b200_matmul_bf16_pairs", _i32, [])
_sig("lyth_b200_gemv_q4", _i32, [_i32, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp])
_sig("lyth_b200_gemv_dequant", _i32, [_i32, _u32, _u32, _u32, _vp, _vp, _vp, _vp])
_sig("lyth_b200_nf4_codebook", None, [C.POINTER(_f32)])
_sig("lyth_b200_hadamard", _i32, [_u64, _u64, _f32, _vp, _vp, _vp, _vp, _vp])
_sig("lyth_b200_gate", _i32, [_u64, _u64, C.POINTER(_f32), _vp, _vp, _vp, _vp, _vp])
_sig("lyth_b200_cu", _i32, [_u64, _u64, _u64, C.POINTER(_f32), _vp, _vp, _vp, _vp, _vp])
_sig("lyth_b200_swap", _i32, [_u64, _u64, _u64, _vp, _vp, _vp, _vp, _vp])
_sig("lyth_sv_unique_id", _i32, [C.c_char_p])
_sig("lyth_sv_create", _i32, [C.POINTER(_vp), _u32, _i32, _i32, _i32, C.c_char_p])
_sig("lyth_sv_destroy", _i32, [_vp])
_sig("lyth_sv_local_len", _u64, [_vp])
_sig("lyth_sv_stream", _vp, [_vp])
_sig("lyth_sv_init_basis", _i32, [_vp, _u64])
_sig("lyth_sv_init_random", _i32, [_vp, _u64])
_sig("lyth_sv_set_local", _i32, [_vp, _vp, _vp])
_sig("lyth_sv_get_local", _i32, [_vp, _vp, _vp])
_sig("lyth_sv_apply", _i32, [_vp, C.POINTER(Gate), _u64])
_sig("lyth_sv_sync", _i32, [_vp])
_sig("lyth_sv_set_deadline", _i32, [_vp, C.c_double])
_sig("lyth_sv_set_pull_queues", _i32, [_vp, _i32])
_sig("lyth_sv_deadline_selftest", _i32, [_i32, C.c_double, C.POINTER(_i32), C.POINTER(_u64)])
_sig("lyth_sv_stats", _i32, [_vp, C.POINTER(_u64), C.POINTER(_u64), C.POINTER(_u64)])
_sig("lyth_sv_launches", _u64, [_vp])
_sig("lyth_sv_set_timing", _i32, [_vp, _i32])
_sig("lyth_sv_timing", _i32, [_vp, _i32, C.POINTER(_u64), C.POINTER(C.c_double)])
_sig("lyth_sv_reset_timing", _i32, [_vp])
_sig("lyth_sv_set_fusion", _i32, [_vp, _i32])
_sig("lyth_sv_set_remap", _i32, [_vp, _i32])
_sig("lyth_sv_set_diagonal", _i32, [_vp, _i32])
_sig("lyth_sv_set_swap_batch", _i32, [_vp, _i32])
_sig("lyth_sv_set_transport", _i32, [_vp, _i32])
_sig("lyth_sv_transport", _i32, [_vp])
_sig("lyth_sv_set_chunk", _i32, [_vp, _u64])
_sig("lyth_sv_plan_create", _i32, [C.POINTER(_vp), _u32, _i32, _i32])
_sig("lyth_sv_plan_count", _u64, [_vp])
_sig("lyth_sv_plan_op", _i32, [_vp, _u64, C.POINTER(SvOp)])
_sig("lyth_sv_plan_clear", _i32, [_vp])
_sig("lyth_b200_device_error", _i32, [])
_sig("lyth_b200_stream_narrow", _i32, [_i32, _i32, _u64, C.POINTER(_f32), _vp, _vp, _vp, _vp])
_sig("lyth_b200_transpose_narrow", _i32, [_i32, _u32, _u32, _vp, _vp, _vp])
_sig("lyth_b200_reduce_partials_narrow", _i32, [_i32, _i32, _u64, _vp, _vp, _u32, _vp, _vp])
_sig("lyth_b200_wait_selftest", _i32, [_i32, _u32, _vp])
_sig("lyth_b200_fused_layout_selftest", _i32, [_u64, _u32, C.POINTER(_u32), C.POINTER(_u32)])


def check(status: int, what: str = "") -> None:
    if status != OK:
        raise LythError(status, what)


def version() -> int:
    return int(lib.lyth_b200_version())


# ----------------------------------------------------------------------------- pointers
def _ptr(t, dtype=None, name="buffer"):
    """A device pointer from a torch CUDA tensor (checked: CUDA, contiguous, dtype) or an int."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    import torch

    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a torch CUDA tensor or a device pointer, got {type(t)}")
    if not t.is_cuda:
        raise ValueError(f"{name}: must live on a CUDA device (lyth_b200 has no CPU path)")
    if not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name}: expected {dtype}, got {t.dtype}")
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _f32t():
    import torch

    return torch.float32


# ----------------------------------------------------------------------------- streams
def stream_range(n: int, rank: int, world: int, align: int = 1024) -> tuple[int, int]:
    """This rank's contiguous range (offset, count) of an n-element stream split over `world`
    ranks: independent units, no collective (the streams are elementwise). Boundaries fall on
    multiples of `align` elements (16-byte aligned slices keep the vector paths); the ranges
    cover [0, n) exactly once, the last rank taking the remainder."""
    if world < 1 or not 0 <= rank < world or n < 0 or align < 1:
        raise ValueError("bad range request")
    per = (n // world) // align * align
    off = rank * per
    cnt = per if rank < world - 1 else n - off
    return off, cnt


def saxpy(a: float, x, y, stream=None) -> None:
    """examples/saxpy.lyth: y = fma(a, x, y), in place on y."""
    check(lib.lyth_b200_saxpy(y.numel(), a, _ptr(x, _f32t(), "x"), _ptr(y, _f32t(), "y"), _stream(stream)), "saxpy")


def axpby(a: float, b: float, x, y, stream=None) -> None:
    """examples/axpby.lyth: y = fma(a, x, mul(b, y)), in place on y."""
    check(lib.lyth_b200_axpby(y.numel(), a, b, _ptr(x, _f32t(), "x"), _ptr(y, _f32t(), "y"), _stream(stream)), "axpby")


def lerp(t: float, x, y, z, stream=None) -> None:
    """examples/lerp.lyth: z = fma(t, sub(y, x), x)."""
    check(lib.lyth_b200_lerp(z.numel(), t, _ptr(x, _f32t(), "x"), _ptr(y, _f32t(), "y"), _ptr(z, _f32t(), "z"),
                             _stream(stream)), "lerp")


def horner(c0: float, c1: float, c2: float, c3: float, x, y, stream=None) -> None:
    """examples/horner.lyth: y = fma(fma(fma(c3, x, c2), x, c1), x, c0)."""
    check(lib.lyth_b200_horner(y.numel(), c0, c1, c2, c3, _ptr(x, _f32t(), "x"), _ptr(y, _f32t(), "y"),
                               _stream(stream)), "horner")


def copy2d(a, b, stream=None) -> None:
    """examples/copy2d.lyth: b[i, j] = a[i, j] for 2-D a (rows x cols)."""
    rows, cols = a.shape
    check(lib.lyth_b200_copy2d(rows, cols, _ptr(a, _f32t(), "a"), _ptr(b, _f32t(), "b"), _stream(stream)), "copy2d")


def transpose_naive(a, b, stream=None) -> None:
    """examples/transpose.lyth: b[j, i] = a[i, j], untiled (the strided control)."""
    rows, cols = a.shape
    check(lib.lyth_b200_transpose_naive(rows, cols, _ptr(a, _f32t(), "a"), _ptr(b, _f32t(), "b"), _stream(stream)),
          "transpose")


def transpose_tiled(a, b, stream=None) -> None:
    """examples/transpose-tiled.lyth: the same through a bank-skewed shared tile."""
    rows, cols = a.shape
    check(lib.lyth_b200_transpose_tiled(rows, cols, _ptr(a, _f32t(), "a"), _ptr(b, _f32t(), "b"), _stream(stream)),
          "transpose_tiled")


# ----------------------------------------------------------------------------- reductions
def reduce_grid(n: int) -> int:
    """The reference's reduction grid for n elements: ceil(n / 2048) in [1, 2^20]."""
    return int(lib.lyth_b200_reduce_grid(n))


def reduce_partials(op: int, x, y=None, grid: int | None = None, out=None, stream=None):
    """One partial per block in the reference's two-stage order (eval.rs:326-345)."""
    import torch

    n = x.numel()
    grid = grid or reduce_grid(n)
    if out is None:
        out = torch.empty(grid, dtype=torch.float32, device=x.device)
    check(lib.lyth_b200_reduce_partials(op, n, _ptr(x, _f32t(), "x"), _ptr(y, _f32t(), "y"), grid,
                                        _ptr(out, _f32t(), "partial"), _stream(stream)), "reduce_partials")
    return out


def reduce(op: int, x, y=None, out=None, workspace=None, stream=None):
    """The whole reduction to one value (partials, then a cluster/DSMEM combine)."""
    import torch

    n = x.numel()
    ws_bytes = int(lib.lyth_b200_reduce_workspace_bytes(n))
    if workspace is None:
        workspace = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device=x.device)
    if out is None:
        out = torch.empty(1, dtype=torch.float32, device=x.device)
    check(lib.lyth_b200_reduce(op, n, _ptr(x, _f32t(), "x"), _ptr(y, _f32t(), "y"), _ptr(out, _f32t(), "out"),
                               _ptr(workspace, name="workspace"), workspace.numel() * workspace.element_size(),
                               _stream(stream)), "reduce")
    return out


# ----------------------------------------------------------------------------- narrow storage
NARROW_F16, NARROW_BF16 = 1, 2
STREAM_SAXPY, STREAM_AXPBY, STREAM_LERP, STREAM_HORNER, STREAM_COPY = 0, 1, 2, 3, 4


def _narrow_ty(t) -> int:
    import torch

    if t.dtype == torch.float16:
        return NARROW_F16
    if t.dtype == torch.bfloat16:
        return NARROW_BF16
    raise TypeError(f"narrow storage is float16 or bfloat16, got {t.dtype}")


def stream_narrow(op: int, scalars, x, y, out, stream=None) -> None:
    """ADR-0024 narrow-storage streams: x, y, out all float16 (or all bfloat16) CUDA tensors, the f32
    chain of the op on the widened elements, each output rounded once (RNE) at the store."""
    ty = _narrow_ty(out)
    sc = (_f32 * 4)(*([float(v) for v in scalars] + [0.0] * (4 - len(scalars))))
    check(lib.lyth_b200_stream_narrow(op, ty, out.numel(), sc, _ptr(x, x.dtype, "x"),
                                      None if y is None else _ptr(y, x.dtype, "y"), _ptr(out, x.dtype, "out"),
                                      _stream(stream)), "stream_narrow")


def transpose_narrow(a, b, stream=None) -> None:
    rows, cols = a.shape
    check(lib.lyth_b200_transpose_narrow(_narrow_ty(a), rows, cols, _ptr(a, a.dtype, "a"), _ptr(b, a.dtype, "b"),
                                         _stream(stream)), "transpose_narrow")


def reduce_partials_narrow(op: int, x, y=None, grid: int | None = None, stream=None):
    import torch

    n = x.numel()
    g = int(lib.lyth_b200_reduce_grid(n)) if grid is None else grid
    part = torch.empty(g, dtype=torch.float32, device=x.device)
    check(lib.lyth_b200_reduce_partials_narrow(op, _narrow_ty(x), n, _ptr(x, x.dtype, "x"),
                                               None if y is None else _ptr(y, x.dtype, "y"), g,
                                               _ptr(part, _f32t(), "partial"), _stream(stream)), "reduce_partials_narrow")
    return part


# ----------------------------------------------------------------------------- contraction
def matmul_f32(a, b, c, exact: bool = False, stream=None) -> None:
    """examples/matmul.lyth: c = a @ b. exact=True is the reference's order bit for bit."""
    m, k = a.shape
    k2, n = b.shape
    if k2 != k or tuple(c.shape) != (m, n):
        raise ValueError(f"matmul shapes {tuple(a.shape)} x {tuple(b.shape)} -> {tuple(c.shape)}")
    check(lib.lyth_b200_matmul_f32(m, n, k, _ptr(a, _f32t(), "a"), _ptr(b, _f32t(), "b"), _ptr(c, _f32t(), "c"),
                                   int(exact), _stream(stream)), "matmul_f32")


def matmul_bf16(a, b, c, stream=None, pair: bool | None = None) -> None:
    """bf16 a (m x k), b (k x n), f32 c on the tcgen05 tensor cores. pair: None = the library's
    choice (CTA pairs when m is a multiple of 256), True / False = that form."""
    import torch

    m, k = a.shape
    k2, n = b.shape
    if k2 != k or tuple(c.shape) != (m, n):
        raise ValueError(f"matmul shapes {tuple(a.shape)} x {tuple(b.shape)} -> {tuple(c.shape)}")
    args = (m, n, k, _ptr(a, torch.bfloat16, "a"), _ptr(b, torch.bfloat16, "b"), _ptr(c, _f32t(), "c"),
            _stream(stream))
    if pair is None:
        check(lib.lyth_b200_matmul_bf16(*args), "matmul_bf16")
    else:
        check(lib.lyth_b200_matmul_bf16_form(int(pair), *args), "matmul_bf16")


# ----------------------------------------------------------------------------- GEMV
def nf4_codebook():
    arr = (_f32 * 16)()
    lib.lyth_b200_nf4_codebook(arr)
    return list(arr)


def gemv_q4(fmt: int, w, scales, x, y, group: int = 64, stream=None) -> None:
    """y[r] = sum_k dequant(W)[r, k] x[k]; w uint8 [rows, k/2], scales/x/y fp16 (as torch.float16)."""
    import torch

    rows, half_k = w.shape
    check(lib.lyth_b200_gemv_q4(fmt, rows, 2 * half_k, group, _ptr(w, torch.uint8, "w"),
                                _ptr(scales, torch.float16, "scales"), _ptr(x, torch.float16, "x"),
                                _ptr(y, torch.float16, "y"), _stream(stream)), "gemv_q4")


def gemv_dequant(fmt: int, w, scales, out, group: int = 64, stream=None) -> None:
    import torch

    rows, half_k = w.shape
    check(lib.lyth_b200_gemv_dequant(fmt, rows, 2 * half_k, group, _ptr(w, torch.uint8, "w"),
                                     _ptr(scales, torch.float16, "scales"), _ptr(out, _f32t(), "out"),
                                     _stream(stream)), "gemv_dequant")


# ----------------------------------------------------------------------------- gates
def _m8(m):
    return (_f32 * 8)(*[float(v) for v in m])


def hadamard(w: int, s: float, re, im, qr=None, qi=None, stream=None) -> None:
    """examples/hadamard_q.lyth on n = re.numel() amplitudes; in place when qr/qi are omitted."""
    qr = re if qr is None else qr
    qi = im if qi is None else qi
    check(lib.lyth_b200_hadamard(re.numel(), w, s, _ptr(re, _f32t()), _ptr(im, _f32t()), _ptr(qr, _f32t()),
                                 _ptr(qi, _f32t()), _stream(stream)), "hadamard_q")


def gate(w: int, m, re, im, qr=None, qi=None, stream=None) -> None:
    """examples/gate_q.lyth: U = [[a, b], [c, d]] (m = ar ai br bi cr ci dr di) on width w."""
    qr = re if qr is None else qr
    qi = im if qi is None else qi
    check(lib.lyth_b200_gate(re.numel(), w, _m8(m), _ptr(re, _f32t()), _ptr(im, _f32t()), _ptr(qr, _f32t()),
                             _ptr(qi, _f32t()), _stream(stream)), "gate_q")


def cu(wc: int, wt: int, m, re, im, qr=None, qi=None, stream=None) -> None:
    """examples/cu_q.lyth with widths (wc, wt) as widths_ct gives them."""
    qr = re if qr is None else qr
    qi = im if qi is None else qi
    check(lib.lyth_b200_cu(re.numel(), wc, wt, _m8(m), _ptr(re, _f32t()), _ptr(im, _f32t()), _ptr(qr, _f32t()),
                           _ptr(qi, _f32t()), _stream(stream)), "cu_q")


def swap(wc: int, wt: int, re, im, qr=None, qi=None, stream=None) -> None:
    """examples/swap_q.lyth."""
    qr = re if qr is None else qr
    qi = im if qi is None else qi
    check(lib.lyth_b200_swap(re.numel(), wc, wt, _ptr(re, _f32t()), _ptr(im, _f32t()), _ptr(qr, _f32t()),
                             _ptr(qi, _f32t()), _stream(stream)), "swap_q")


from .statevector import Plan, StateVector, unique_id  # noqa: E402,F401
