"""ctypes access to the ADR-0016 surface (lyth_<k>_load / _launch / _launch_with), the way a
caller of LYTH's generated C header binds it: CUfunction and CUmodule as opaque pointers,
CUdeviceptr as a 64-bit integer, CUresult as an int."""
import ctypes as C

import lyth_b200 as lb

_vp, _u32, _f32, _u64 = C.c_void_p, C.c_uint32, C.c_float, C.c_uint64

# (kernel, parameter kinds in declaration order): 'u' u32, 'f' f32, 'p' device pointer
SIGS = {
    "saxpy": "ufpp", "axpby": "uffpp", "lerp": "ufppp", "horner": "uffffpp",
    "copy2d": "uupp", "transpose": "uupp", "transpose_tiled": "uupp",
    "sum": "upp", "dot": "uppp", "max_of": "upp", "min_of": "upp",
    "matmul": "uuuppp", "hadamard_q": "uufpppp", "gate_q": "uuffffffffpppp",
    "cu_q": "uuuffffffffpppp", "swap_q": "uuupppp",
}
_T = {"u": _u32, "f": _f32, "p": _u64}


def load(kernel: str):
    fn, mod = _vp(), _vp()
    f = getattr(lb.lib, f"lyth_{kernel}_load")
    f.restype = C.c_int
    f.argtypes = [C.POINTER(_vp), C.POINTER(_vp)]
    rc = f(C.byref(mod), C.byref(fn))
    assert rc == 0, f"lyth_{kernel}_load: CUresult {rc}"
    return fn


def launch(kernel: str, fn, *args, grid: int | None = None) -> int:
    kinds = SIGS[kernel]
    assert len(args) == len(kinds)
    if grid is None:
        f = getattr(lb.lib, f"lyth_{kernel}_launch")
        f.argtypes = [_vp] + [_T[k] for k in kinds]
        f.restype = C.c_int
        return f(fn, *args)
    f = getattr(lb.lib, f"lyth_{kernel}_launch_with")
    f.argtypes = [_vp, _u32] + [_T[k] for k in kinds]
    f.restype = C.c_int
    return f(fn, grid, *args)
