"""Generated bindings and manifests for the ADR-0016 surface (crates/lyth/src/bind_c.rs:39-395,
crates/lyth/src/bind_py.rs, crates/lyth/src/manifest.rs:27-523), from the lowered kernels of
``lyth_b200.examples``.

* ``c_section(name)``: the per-kernel block of include/lyth_b200.h -- the contract macros whose
  figures are derived here (``probe.derive_cost``: DERIVED_INTENSITY, FLOPS_PER_ELEMENT,
  BYTES_PER_ELEMENT) and the five entry points with the generator's exact signatures
  (``lyth_<k>_elements / _grid / _load / _launch / _launch_with``; ``_partial_len`` for a
  reduction, ``_check_splits`` for a split kernel). The committed header must contain exactly
  these lines (tests/test_bindgen.py), the way the reference checks its checked-in bindings
  against the generator (crates/lyth/tests/binding.rs).
* ``manifest(name)``: the ``lyth-manifest/0.1`` record of the kernel as this back end launches it.
* ``py_module()``: a ctypes module over liblyth_b200.so with one launch function per kernel
  (the ADR-0016 `_launch` symbols, declaration order), in the shape of bind_py.rs's output.

``python -m lyth_b200.bindgen manifests DIR`` writes every manifest; ``... py FILE`` the module.
"""
from __future__ import annotations

import json
import os
import sys

from . import examples as ex
from .ir import TY
from .probe import derive_cost

SCHEMA = "lyth-manifest/0.1"

# The ADR-0016 kernels: (example, extents of the index space, buffer shapes, launch facts of this
# back end's `_launch`: block, dynamic shared bytes, max grid, grid rule).
ELEM = ("elementwise", 1)
ADR16 = {
    "saxpy": (["n"], {"x": ["n"], "y": ["n"]}, 256, 0, 1 << 20, ELEM),
    "axpby": (["n"], {"x": ["n"], "y": ["n"]}, 256, 0, 1 << 20, ELEM),
    "lerp": (["n"], {"x": ["n"], "y": ["n"], "z": ["n"]}, 256, 0, 1 << 20, ELEM),
    "horner": (["n"], {"x": ["n"], "y": ["n"]}, 256, 0, 1 << 20, ELEM),
    "copy2d": (["rows", "cols"], {"a": ["rows", "cols"], "b": ["rows", "cols"]}, 256, 0, 1 << 20, ELEM),
    "transpose": (["rows", "cols"], {"a": ["rows", "cols"], "b": ["cols", "rows"]}, 256, 0, 1 << 20, ELEM),
    "transpose_tiled": (["rows", "cols"], {"a": ["rows", "cols"], "b": ["cols", "rows"]}, 256, 16640, 2147483647,
                        ("tiled", 64)),
    "sum": (["n"], {"x": ["n"], "partial": ["blocks"]}, 256, 1024, 1 << 20, ("elementwise", 8)),
    "dot": (["n"], {"x": ["n"], "y": ["n"], "partial": ["blocks"]}, 256, 1024, 1 << 20, ("elementwise", 8)),
    "max_of": (["n"], {"x": ["n"], "partial": ["blocks"]}, 256, 1024, 1 << 20, ("elementwise", 8)),
    "min_of": (["n"], {"x": ["n"], "partial": ["blocks"]}, 256, 1024, 1 << 20, ("elementwise", 8)),
    "hadamard_q": (["n"], {b: ["n"] for b in ("re", "im", "qr", "qi")}, 256, 0, 1 << 20, ELEM),
    "gate_q": (["n"], {b: ["n"] for b in ("re", "im", "qr", "qi")}, 256, 0, 1 << 20, ELEM),
    "cu_q": (["n"], {b: ["n"] for b in ("re", "im", "qr", "qi")}, 256, 0, 1 << 20, ELEM),
    "swap_q": (["n"], {b: ["n"] for b in ("re", "im", "qr", "qi")}, 256, 0, 1 << 20, ELEM),
}
C_TYPE = {TY["u32"]: "unsigned int", TY["f32"]: "float", TY["f32[]"]: "CUdeviceptr", TY["f16[]"]: "CUdeviceptr",
          TY["bf16[]"]: "CUdeviceptr"}
TY_NAME = {TY["u32"]: "u32", TY["f32"]: "f32", TY["f32[]"]: "buf_f32", TY["f16[]"]: "buf_f16", TY["bf16[]"]: "buf_bf16"}


def _kernel(name):
    return ex.IN_SCOPE[name]()


def _width_params(k) -> list[str]:
    out = []
    for _, _, w, _ in k.views:
        if w not in out:
            out.append(w)
    return out


def c_section(name: str) -> dict:
    """The derived contract macros and the declarations of kernel `name`'s ADR-0016 block."""
    k = _kernel(name)
    extents, *_ = ADR16[name]
    c = derive_cost(k)
    up = name.upper()
    macros = {
        f"LYTH_{up}_DERIVED_INTENSITY": repr(float(c["intensity"])),
        f"LYTH_{up}_FLOPS_PER_ELEMENT": repr(float(c["flops"])),
        f"LYTH_{up}_BYTES_PER_ELEMENT": repr(float(c["bytes"])),
    }
    ext = ", ".join(f"unsigned int {e}" for e in extents)
    params = ", ".join(f"{C_TYPE[t]} {n}" for n, t in k.params)
    decls = [f"unsigned int lyth_{name}_elements({ext});",
             f"unsigned int lyth_{name}_grid({ext});"]
    if k.reduction:
        decls.append(f"unsigned int lyth_{name}_partial_len({ext});")
    if k.views:
        ws = ", ".join(f"unsigned int {w}" for w in [extents[0]] + _width_params(k))
        decls.append(f"int lyth_{name}_check_splits({ws});")
    decls += [f"CUresult lyth_{name}_load(CUmodule *module, CUfunction *fn);",
              f"CUresult lyth_{name}_launch(CUfunction fn, {params});",
              f"CUresult lyth_{name}_launch_with(CUfunction fn, unsigned int grid, {params});"]
    return {"macros": macros, "decls": decls}


def manifest(name: str) -> dict:
    """lyth-manifest/0.1 (manifest.rs:27-41) for kernel `name` as this back end launches it."""
    k = _kernel(name)
    extents, shapes, block, shared, max_grid, (rule, per) = ADR16[name]
    into = k.reduction[2] if k.reduction else None
    loaded = {op[6] for op in k.ops if op[0] == 0}
    drained = {d[0] for d in k.drains}
    base = {v[0]: v[1] for v in k.views}

    def root(b):
        while b in base:
            b = base[b]
        return b

    reads = {root(b) for b in loaded}
    writes = {root(b) for b in drained} | ({into} if into else set())
    named = {e for s in shapes.values() for e in s}
    params = [{"name": n, "ty": TY_NAME[t], "shape": shapes.get(n, []),
               "is_extent": t == TY["u32"] and n in named, "written": n in writes, "read": n in reads,
               "sized_by_grid": n == into} for n, t in k.params]
    splits = []
    seen = []
    for vname, b, w, part in k.views:
        if b in seen:
            continue
        seen.append(b)
        pair = [v[0] for v in k.views if v[1] == b]
        depth, x = 0, b
        while x in base:
            depth, x = depth + 1, base[x]
        s = {"base": b, "views": pair, "width": w, "extent": shapes.get(root(b), [""])[0]}
        if depth:
            s["depth"] = depth
        splits.append(s)
    c = derive_cost(k)
    grid = ({"type": "tiled", "tile": [per, per], "extents": extents} if rule == "tiled" else
            {"type": "elementwise", "extents": extents, "min_elements_per_thread": per,
             "split_depth": max((s.get("depth", 0) + 1 for s in splits), default=0)})
    m = {
        "schema": SCHEMA, "kernel": name, "params": params,
        "launch": {"block": block, "shared_bytes": shared, "grid": grid, "max_grid": max_grid,
                   "predicted_bank_conflicts": 0, "block_must_be_power_of_two": bool(k.reduction)},
        "contract": {"machine": "sm_100a", "accepts": ["sm_120"], "declared_intensity": None,
                     "derived_intensity": c["intensity"], "asymptotic": False,
                     "flops_per_element": float(c["flops"]), "bytes_per_element": float(c["bytes"]),
                     "read_bytes_per_element": float(c["read"]), "write_bytes_per_element": float(c["write"]),
                     "counter": "dram__bytes_read.sum / dram__bytes_write.sum (B200: lts__t_bytes counts ~1.5x)"},
        "backend": {"library": "liblyth_b200.so", "load": f"lyth_{name}_load", "launch": f"lyth_{name}_launch",
                    "image": "sm_100a SASS built in (no PTX JIT)"},
        "known_limits": [],
    }
    if splits:
        m["splits"] = splits
    return m


def py_module() -> str:
    """A ctypes module over the library's ADR-0016 launch symbols (bind_py.rs's shape): one
    function per kernel, arguments in declaration order, buffers as device pointers."""
    lines = ['"""Generated by lyth_b200.bindgen: ADR-0016 launches over liblyth_b200.so (do not edit)."""',
             "import ctypes as C", "import os", "",
             "LIB = C.CDLL(os.environ.get('LYTH_B200_LIB', os.path.join(os.path.dirname(os.path.abspath(__file__)), "
             "'liblyth_b200.so')))", ""]
    ct = {TY["u32"]: "C.c_uint", TY["f32"]: "C.c_float", TY["f32[]"]: "C.c_uint64", TY["f16[]"]: "C.c_uint64",
          TY["bf16[]"]: "C.c_uint64"}
    for name in ADR16:
        k = _kernel(name)
        args = ", ".join(n for n, _ in k.params)
        lines += [f"_{name}_fn = C.c_void_p()",
                  f"LIB.lyth_{name}_load(None, C.byref(_{name}_fn))",
                  f"LIB.lyth_{name}_launch.argtypes = [C.c_void_p] + [{', '.join(ct[t] for _, t in k.params)}]",
                  f"LIB.lyth_{name}_launch.restype = C.c_int", "",
                  f"def {name}({args}):",
                  f'    """{name}: CUresult of lyth_{name}_launch (stream 0)."""',
                  f"    return LIB.lyth_{name}_launch(_{name}_fn, {args})", ""]
    return "\n".join(lines)


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) == 2 and argv[0] == "manifests":
        os.makedirs(argv[1], exist_ok=True)
        for name in ADR16:
            with open(os.path.join(argv[1], f"{name}.json"), "w") as f:
                json.dump(manifest(name), f, indent=1)
                f.write("\n")
        return 0
    if len(argv) == 2 and argv[0] == "py":
        with open(argv[1], "w") as f:
            f.write(py_module())
        return 0
    if len(argv) == 1 and argv[0] == "c":
        for name in ADR16:
            sec = c_section(name)
            for k, v in sec["macros"].items():
                print(f"#define {k} {v}")
            print("\n".join(sec["decls"]))
            print()
        return 0
    print("usage: python -m lyth_b200.bindgen manifests DIR | py FILE | c", file=sys.stderr)
    return 2


if __name__ == "__main__":
    sys.exit(main())
