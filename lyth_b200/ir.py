"""Lowered-kernel descriptors for the back-end entry (``lyth_b200_select`` / ``lyth_b200_launch``).

A ``Kernel`` is the part of lyth-lang's ``KernelIr`` (crates/lyth-lang/src/ir.rs:24-56) this back
end reads: parameters in declaration order, the rank-2 space, tile, coarsen, contraction,
reduction, split views (ir.rs:58-81) and the lowered straight-line body (``Op``, ir.rs:463-503:
Load, Param, Const, Bin, Fma, Neg) with the register each drained buffer takes. The builder
methods append ops and return their registers, so a kernel reads as its lowering::

    k = Kernel("saxpy", [("n", "u32"), ("a", "f32"), ("x", "f32[]"), ("y", "f32[]")])
    k.drain("y", k.fma(k.param("a"), k.load("x"), k.load("y")))
    sel = k.select()            # the kernel class, or LythError with lyth-ptx's refusal text
    sel.launch([n, 2.5, x_ptr, y_ptr], stream)

``select`` maps it to a kernel of this library by what the body computes (operation for
operation, fma formation included) or refuses it; ``launch`` takes the arguments in declaration
order, as lyth-cuda's ``Function::launch_shared`` takes its ``Arg`` slots
(crates/lyth-cuda/src/lib.rs:483-549).
"""
from __future__ import annotations

import ctypes as C

from . import LythError, check, lib

TY = {"u32": 0, "f32": 1, "f32[]": 2, "f16[]": 3, "bf16[]": 4}
LOAD, PARAM, CONST, BIN, FMA, NEG = 0, 1, 2, 3, 4, 5
BINOPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "max": 4, "min": 5}
REDUCE = {"sum": 0, "max": 1, "min": 2}
CLASSES = {1: "saxpy", 2: "axpby", 3: "lerp", 4: "horner", 5: "copy2d", 6: "transpose", 7: "transpose_tiled",
           8: "sum", 9: "dot", 10: "max_of", 11: "min_of", 12: "matmul", 13: "matmul_bf16", 14: "hadamard_q",
           15: "gate_q", 16: "cu_q", 17: "swap_q"}


class _Param(C.Structure):
    _fields_ = [("name", C.c_char_p), ("ty", C.c_int32)]


class _View(C.Structure):
    _fields_ = [("name", C.c_char_p), ("base", C.c_char_p), ("width", C.c_char_p), ("part", C.c_uint32)]


class _Op(C.Structure):
    _fields_ = [("kind", C.c_int32), ("bin", C.c_int32), ("a", C.c_int32), ("b", C.c_int32), ("c", C.c_int32),
                ("value", C.c_double), ("name", C.c_char_p), ("transposed", C.c_uint32)]


class _Drain(C.Structure):
    _fields_ = [("buffer", C.c_char_p), ("reg", C.c_int32), ("transposed", C.c_uint32)]


class _Ir(C.Structure):
    _fields_ = [("name", C.c_char_p), ("machine", C.c_char_p), ("nparams", C.c_uint32),
                ("params", C.POINTER(_Param)), ("rank", C.c_uint32), ("tile", C.c_uint32 * 2),
                ("coarsen", C.c_uint32 * 2), ("contract", C.c_uint32), ("reduce_op", C.c_int32),
                ("reduce_reg", C.c_int32), ("reduce_into", C.c_char_p), ("reduce_via_smem", C.c_uint32),
                ("nviews", C.c_uint32), ("views", C.POINTER(_View)), ("nops", C.c_uint32), ("ops", C.POINTER(_Op)),
                ("ndrains", C.c_uint32), ("drains", C.POINTER(_Drain))]


class _Kernel(C.Structure):
    _fields_ = [("cls", C.c_int32), ("entry", C.c_char * 48), ("nparams", C.c_uint32), ("param_ty", C.c_int32 * 32),
                ("slot", C.c_int32 * 16), ("retargeted", C.c_uint32), ("storage", C.c_int32),
                ("message", C.c_char * 320)]


class _Launch(C.Structure):
    _fields_ = [("grid", C.c_uint32)]


lib.lyth_b200_select.restype = C.c_int
lib.lyth_b200_select.argtypes = [C.POINTER(_Ir), C.POINTER(_Kernel)]
lib.lyth_b200_launch.restype = C.c_int
lib.lyth_b200_launch.argtypes = [C.POINTER(_Kernel), C.POINTER(C.c_void_p), C.POINTER(_Launch), C.c_void_p]
lib.lyth_b200_workspace_bytes.restype = C.c_size_t
lib.lyth_b200_workspace_bytes.argtypes = [C.POINTER(_Kernel), C.POINTER(C.c_void_p)]


class Selected:
    """A kernel class chosen by ``lyth_b200_select``: its name, the declaration-order types, and
    whether the source was written for another machine the sm_100a file accepts."""

    def __init__(self, k: _Kernel):
        self._k = k
        self.cls = int(k.cls)
        self.entry = k.entry.decode()
        self.retargeted = bool(k.retargeted)
        self.storage = int(k.storage)  # 0 f32, 1 f16, 2 bf16 (every data buffer)
        self.note = k.message.decode()
        self.types = [int(k.param_ty[i]) for i in range(k.nparams)]

    def _slots(self, args):
        if len(args) != len(self.types):
            raise ValueError(f"{self.entry}: {len(self.types)} arguments in declaration order, got {len(args)}")
        vals, ptrs = [], (C.c_void_p * len(args))()
        for i, (a, ty) in enumerate(zip(args, self.types)):
            if ty == TY["u32"]:
                v = C.c_uint32(int(a))
            elif ty == TY["f32"]:
                v = C.c_float(float(a))
            else:  # a buffer: a device pointer, or a torch CUDA tensor
                v = C.c_uint64(a if isinstance(a, int) else a.data_ptr())
            vals.append(v)
            ptrs[i] = C.cast(C.byref(v), C.c_void_p)
        return vals, ptrs

    def launch(self, args, stream=0, grid: int | None = None) -> None:
        vals, ptrs = self._slots(args)
        ln = _Launch(grid) if grid else None
        check(lib.lyth_b200_launch(C.byref(self._k), ptrs, C.byref(ln) if ln else None, stream), self.entry)
        del vals

    def workspace_bytes(self, args) -> int:
        vals, ptrs = self._slots(args)
        n = int(lib.lyth_b200_workspace_bytes(C.byref(self._k), ptrs))
        del vals
        return n


class Kernel:
    """A lowered kernel, built op by op (registers are op indices, SSA)."""

    def __init__(self, name: str, params, machine: str = "sm_120", rank: int = 1, tile=(0, 0), coarsen=(0, 0),
                 contract: bool = False):
        self.name, self.machine = name, machine
        self.params = [(n, TY[t]) for n, t in params]
        self.rank, self.tile, self.coarsen, self.contract = rank, tuple(tile), tuple(coarsen), contract
        self.views: list[tuple[str, str, str, int]] = []
        self.ops: list[tuple] = []
        self.drains: list[tuple[str, int, int]] = []
        self.reduction = None  # (op, reg, into, via_smem)

    # -- body
    def _op(self, kind, bin_=0, a=-1, b=-1, c=-1, value=0.0, name=None, transposed=False) -> int:
        self.ops.append((kind, bin_, a, b, c, value, name, int(transposed)))
        return len(self.ops) - 1

    def load(self, buf: str, transposed: bool = False) -> int:
        return self._op(LOAD, name=buf, transposed=transposed)

    def param(self, name: str) -> int:
        return self._op(PARAM, name=name)

    def const(self, v: float) -> int:
        return self._op(CONST, value=v)

    def bin(self, op: str, a: int, b: int) -> int:
        return self._op(BIN, BINOPS[op], a, b)

    def add(self, a, b):
        return self.bin("add", a, b)

    def sub(self, a, b):
        return self.bin("sub", a, b)

    def mul(self, a, b):
        return self.bin("mul", a, b)

    def fma(self, a: int, b: int, c: int) -> int:
        return self._op(FMA, 0, a, b, c)

    def neg(self, a: int) -> int:
        return self._op(NEG, 0, a)

    def split(self, base: str, into: tuple[str, str], width: str) -> None:
        """``split base into v0, v1 : blocks width`` (ADR-0028)."""
        self.views.append((into[0], base, width, 0))
        self.views.append((into[1], base, width, 1))

    def drain(self, buf: str, reg: int, transposed: bool = False) -> None:
        self.drains.append((buf, reg, int(transposed)))

    def reduce(self, op: str, reg: int, into: str, via_smem: bool = True) -> None:
        self.reduction = (REDUCE[op], reg, into, via_smem)

    # -- the descriptor
    def _struct(self):
        keep = []

        def s(x):
            if x is None:
                return None
            b = x.encode()
            keep.append(b)
            return b

        P = (_Param * max(1, len(self.params)))(*[_Param(s(n), t) for n, t in self.params])
        V = (_View * max(1, len(self.views)))(*[_View(s(n), s(b), s(w), p) for n, b, w, p in self.views])
        O = (_Op * max(1, len(self.ops)))(*[_Op(k, bi, a, b, c, v, s(n), t) for k, bi, a, b, c, v, n, t in self.ops])
        D = (_Drain * max(1, len(self.drains)))(*[_Drain(s(b), r, t) for b, r, t in self.drains])
        ir = _Ir()
        ir.name, ir.machine = s(self.name), s(self.machine)
        ir.nparams, ir.params = len(self.params), P
        ir.rank = self.rank
        ir.tile[0], ir.tile[1] = self.tile
        ir.coarsen[0], ir.coarsen[1] = self.coarsen
        ir.contract = int(self.contract)
        if self.reduction:
            ir.reduce_op, ir.reduce_reg, ir.reduce_into, ir.reduce_via_smem = (
                self.reduction[0], self.reduction[1], s(self.reduction[2]), int(self.reduction[3]))
        else:
            ir.reduce_op, ir.reduce_reg = -1, -1
        ir.nviews, ir.views = len(self.views), V
        ir.nops, ir.ops = len(self.ops), O
        ir.ndrains, ir.drains = len(self.drains), D
        return ir, (keep, P, V, O, D)

    def select(self) -> Selected:
        """The kernel class (``lyth_b200_select``), or LythError carrying the refusal."""
        ir, keep = self._struct()
        k = _Kernel()
        st = lib.lyth_b200_select(C.byref(ir), C.byref(k))
        del keep
        if st != 0:
            raise LythError(st, f"select {self.name}: {k.message.decode()}")
        return Selected(k)
