"""lyth-probe's checks for this back end: the B200 machine file, the derived byte model, and the
derived-vs-measured traffic comparison against Nsight Compute.

* ``parse_value`` / ``parse_ncu`` / ``compare``: crates/lyth-probe/src/ncu.rs:38-62 (metric
  names), :230-298 (locale-safe values), :304-449 (per-kernel totals, per level and direction),
  :483-543 (Confirmed / Inflated / Absorbed within a tolerance).
* ``check_machine`` / ``ridge_fp32``: crates/lyth-probe/src/machine.rs:13-330 (a machine file
  against a measurement: schema, id, each level's bandwidth within tol, the measurement's own
  median, the peak, the stored ridge recomputed).
* ``derive_cost``: the per-element bytes and flops of a lowered kernel (lyth_b200.ir.Kernel) for
  the flat classes -- every loaded buffer or view read once, every drained one written once,
  at its element width; fma = 2 flops, add/sub/mul/div = 1, a sum reduction's combine 1, max/min
  0 (crates/lyth-lang/src/ir.rs:2097-2337, the payload terms; the sector and reuse terms of a
  tiled contraction are not restated).

The GPU side (``python -m lyth_b200.probe machine`` and ``... traffic``) measures the machine file
and runs each kernel class once at a size of at least 4x L2 for an ncu capture; ``report`` turns
the capture into the derived-vs-ncu table.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import math
import os
import statistics
import sys

MACHINE_SCHEMA = "lyth-machine/0.1"
MEASUREMENT_SCHEMA = "lyth-machine-measurement/0.1"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MACHINE_FILE = os.path.join(ROOT, "fixtures", "machine", "sm_100a.json")

# ---------------------------------------------------------------------------- ncu CSV
LEVEL_METRICS = [("dram", ["dram__bytes.sum"]), ("l2", ["lts__t_bytes.sum", "lts__t_bytes.sum.per_second"])]
DIR_METRICS = [
    ("dram", "read", ["dram__bytes_op_read.sum", "dram__bytes_read.sum"]),
    ("dram", "write", ["dram__bytes_op_write.sum", "dram__bytes_write.sum"]),
    ("l2", "read", ["lts__t_bytes_op_read.sum"]),
    ("l2", "write", ["lts__t_bytes_op_write.sum"]),
]
COUNT_UNITS = {"sector", "sectors", "request", "requests", "inst", "instructions", "cycle", "cycles", "warp",
               "warps", "thread", "threads", "block", "blocks", "wavefront", "wavefronts", "nsecond", "usecond",
               "msecond", "second", "%", "ns", "us", "ms"}


class NcuError(ValueError):
    pass


def parse_value(raw: str, unit: str):
    """An ncu metric value in base units, or None. Grouping vs decimal separators resolve by
    position (both present: the last is the decimal point), repetition (grouping), then the unit
    (a lone separator in a base byte count groups: a fractional byte does not exist)."""
    u = (unit or "").strip().lower()
    scales = {"": 1.0, "byte": 1.0, "bytes": 1.0, "kbyte": 1e3, "kb": 1e3, "mbyte": 1e6, "mb": 1e6, "gbyte": 1e9,
              "gb": 1e9, "tbyte": 1e12, "tb": 1e12, "kibyte": 1024.0, "mibyte": 1024.0 ** 2, "gibyte": 1024.0 ** 3}
    if u in scales:
        scale = scales[u]
    elif u in COUNT_UNITS:
        scale = 1.0
    else:
        raise NcuError(f"unrecognised unit `{unit}`: refusing to guess a scale")
    base_unit = scale == 1.0
    t = "".join(c for c in raw if not c.isspace())
    if not t or t.lower() == "n/a":
        return None
    dots, commas = t.count("."), t.count(",")
    if dots and commas:
        dec = "." if t.rfind(".") > t.rfind(",") else ","
    elif dots > 1 or commas > 1:
        dec = None
    elif dots == 1:
        dec = None if base_unit else "."
    elif commas == 1:
        dec = None if base_unit else ","
    else:
        dec = None
    if dec is None:
        norm = t.replace(".", "").replace(",", "")
    else:
        norm = "".join("." if c == dec else c for c in t if c == dec or c not in ".,")
    try:
        return float(norm) * scale
    except ValueError:
        return None


def parse_ncu(text: str, kernel: str | None = None, level: str | None = None) -> dict:
    """Per-kernel totals of an `ncu --csv` report: bytes at `level` (dram by default; the sum of
    the read and write halves when only those are present), the halves, the launch count, and
    every metric. `kernel` selects one kernel by substring; None folds them all (and says so)."""
    lines = text.splitlines()
    start = next((i for i, ln in enumerate(lines) if "Metric Name" in ln), None)
    if start is None:
        raise NcuError("no `Metric Name` header: not an ncu --csv report")
    rows = list(csv.reader(io.StringIO("\n".join(lines[start:]))))
    head = [c.strip() for c in rows[0]]

    def col(name, required=True):
        if name in head:
            return head.index(name)
        if required:
            raise NcuError(f"no `{name}` column")
        return None

    c_name, c_val = col("Metric Name"), col("Metric Value")
    c_unit, c_kernel = col("Metric Unit", False), col("Kernel Name", False)
    per_kernel: dict[str, dict[str, list]] = {}
    for f in rows[1:]:
        if len(f) <= max(c_name, c_val):
            continue
        unit = f[c_unit] if c_unit is not None and c_unit < len(f) else ""
        v = parse_value(f[c_val], unit)
        if v is None or not math.isfinite(v):
            continue
        kname = f[c_kernel].strip() if c_kernel is not None else "<all>"
        e = per_kernel.setdefault(kname, {}).setdefault(f[c_name].strip(), [0.0, 0])
        e[0] += v
        e[1] += 1
    if kernel is not None:
        hit = [k for k in per_kernel if kernel in k]
        if not hit:
            raise NcuError(f"no kernel matching `{kernel}`; present: {', '.join(per_kernel)}")
        kname, metrics = hit[0], per_kernel[hit[0]]
    else:
        kname = " + ".join(per_kernel) if len(per_kernel) > 1 else next(iter(per_kernel), "<none>")
        metrics = {}
        for m in per_kernel.values():
            for name, (b, n) in m.items():
                e = metrics.setdefault(name, [0.0, 0])
                e[0] += b
                e[1] += n
    found = []
    for lvl, names in LEVEL_METRICS:
        for n in names:
            if n in metrics:
                found.append((lvl, metrics[n][0], n, metrics[n][1]))
                break

    def half(lvl, d):
        for lv, dd, names in DIR_METRICS:
            if lv == lvl and dd == d:
                for n in names:
                    if n in metrics:
                        return metrics[n]
        return None

    if not any(f[0] == "dram" for f in found):
        r, w = half("dram", "read"), half("dram", "write")
        if r and w:
            found.append(("dram", r[0] + w[0], "dram__bytes_op_read.sum + dram__bytes_op_write.sum", r[1]))
    if not found:
        raise NcuError("the report has no dram byte metric")
    want = level or "dram"
    pick = next((f for f in found if f[0] == want), None)
    if pick is None:
        raise NcuError(f"no `{want}` level in the report; have {', '.join(f[0] for f in found)}")
    lvl, nbytes, metric, launches = pick
    r, w = half(lvl, "read"), half(lvl, "write")
    return {"kernel": kname, "level": lvl, "bytes": nbytes, "launches": launches, "metric": metric,
            "read": r[0] if r else None, "write": w[0] if w else None,
            "metrics": {k: v[0] for k, v in metrics.items()}}


def compare(bytes_per_element: float, elements: float, measured: dict, direction: str = "all",
            tol: float = 0.02) -> dict:
    """Derived bytes/element x elements against the measured bytes of one direction: within tol
    `confirmed`, above `inflated`, below `absorbed` (each with its likely causes)."""
    if elements <= 0:
        raise NcuError("elements must be > 0")
    if bytes_per_element <= 0:
        raise NcuError(f"the accounting has no {direction} bytes to compare")
    if not 0.0 <= tol < 1.0:
        raise NcuError(f"tol must be in [0,1), got {tol}")
    if direction == "all":
        got = measured["bytes"]
    else:
        got = measured.get(direction)
        if got is None:
            raise NcuError(f"the report has no {direction} half: capture dram__bytes_op_{direction}.sum "
                           f"(or dram__bytes_{direction}.sum)")
    expected = bytes_per_element * elements
    ratio = got / expected
    out = {"expected": expected, "measured": got, "ratio": ratio, "tol": tol}
    if abs(ratio - 1.0) <= tol:
        out["verdict"] = "confirmed"
    elif ratio > 1.0:
        out["verdict"] = "inflated"
        out["causes"] = ["cache-line granularity: a scattered pattern moves whole sectors",
                         "uncoalesced access within a warp", "partial-line writes turning into read-modify-write",
                         "register spills to local memory", "traffic the accounting does not list"]
    else:
        out["verdict"] = "absorbed"
        out["causes"] = (["write-back absorption: stores still in L2 when the kernel ends reach DRAM later"]
                         if direction != "read" else []) + [
            "the accounting names the wrong level", "the working set fits in cache at this size"]
    return out


# ---------------------------------------------------------------------------- machine file
def ridge_fp32(machine: dict):
    peak = machine.get("peak_tflops")
    dram = next((lv for lv in machine.get("levels", []) if lv.get("name") == "dram"), None)
    if peak is None or dram is None or dram.get("bandwidth_gbs", 0) <= 0:
        return None
    return peak * 1e3 / dram["bandwidth_gbs"]


def check_machine(machine: dict, meas: dict, tol: float = 0.05) -> dict:
    """machine-check: {"verdict": "pass", "checked": [...]} or {"verdict": "fail", "mismatches":
    [...]}; a schema or id mismatch raises."""
    if machine.get("schema") != MACHINE_SCHEMA:
        raise ValueError(f"machine schema must be `{MACHINE_SCHEMA}`, got `{machine.get('schema')}`")
    if meas.get("schema") != MEASUREMENT_SCHEMA:
        raise ValueError(f"measurement schema must be `{MEASUREMENT_SCHEMA}`, got `{meas.get('schema')}`")
    if machine.get("id") != meas.get("machine_id"):
        raise ValueError(f"machine id `{machine.get('id')}` != measurement machine_id `{meas.get('machine_id')}`")
    if not 0.0 <= tol < 1.0:
        raise ValueError(f"tol must be in [0,1), got {tol}")
    checked, bad = [], []
    for m in meas.get("levels", []):
        runs = m.get("runs") or []
        if runs:
            med = statistics.median(runs)
            if abs(m["bandwidth_gbs"] - med) / med > 0.005:
                bad.append(f"{m['name']}: measurement claims {m['bandwidth_gbs']:.2f} GB/s but the median of its "
                           f"{len(runs)} runs is {med:.2f} GB/s: the measurement is not self-consistent")
                continue
        lv = next((x for x in machine.get("levels", []) if x.get("name") == m["name"]), None)
        if lv is None:
            bad.append(f"measurement has level `{m['name']}` not in machine file")
            continue
        claimed, got = lv["bandwidth_gbs"], m["bandwidth_gbs"]
        rel = math.inf if claimed == 0 else abs(got - claimed) / claimed
        if rel <= tol:
            checked.append(f"{m['name']}: claimed {claimed:.2f} GB/s, measured {got:.2f} GB/s (rel {rel:.3f})")
        else:
            bad.append(f"{m['name']}: machine file claims {claimed:.2f} GB/s, measured {got:.2f} GB/s "
                       f"(rel {rel:.3f} > tol {tol})")
    if machine.get("peak_tflops") is not None and meas.get("peak_tflops") is not None:
        c, g = machine["peak_tflops"], meas["peak_tflops"]
        rel = abs(g - c) / max(c, 1e-300)
        (checked if rel <= tol else bad).append(
            f"peak: claimed {c:.2f} TFLOP/s, measured {g:.2f} TFLOP/s (rel {rel:.3f})")
    stated = (machine.get("ridge_flop_per_byte") or {}).get("fp32")
    derived = ridge_fp32(machine)
    if stated is not None and derived is not None:
        rel = abs(stated - derived) / max(derived, 1e-300)
        if rel <= 0.005:
            checked.append(f"ridge fp32: stated {stated:.2f}, derived {derived:.2f} flop/byte from this file")
        else:
            bad.append(f"ridge_flop_per_byte.fp32 states {stated:.2f} but the file's peak over its dram bandwidth "
                       f"derives {derived:.2f}: a stored ridge drifts when one of its inputs is edited")
    return {"verdict": "pass", "checked": checked} if not bad else {"verdict": "fail", "mismatches": bad}


def accepts(machine: dict, source_machine: str) -> bool:
    """Whether a kernel whose `machine` line names `source_machine` runs against this file: its
    own id, or an id listed in its `accepts` (the retarget is recorded, never silent)."""
    return source_machine == machine.get("id") or source_machine in machine.get("accepts", [])


# ---------------------------------------------------------------------------- derived cost
WIDTH = {2: 4, 3: 2, 4: 2}  # LYTH_TY_BUF_F32 / F16 / BF16


def derive_cost(k) -> dict:
    """Bytes read, bytes written and flops per element of the index space of a flat kernel
    (lyth_b200.ir.Kernel): every loaded buffer or view read once, every drained one written once
    (views at their base's width), fma 2 flops, add/sub/mul/div 1, neg/max/min 0; a reduction adds
    its combine (sum 1, max/min 0). A contraction is refused (its cost is an expression)."""
    from .ir import BIN, FMA, LOAD, NEG

    if k.contract:
        raise ValueError(f"{k.name}: a contraction's cost is symbolic in the contracted extent")
    ty = dict(k.params)
    base = {v[0]: v[1] for v in k.views}

    def width(name):
        while name in base:
            name = base[name]
        return WIDTH[ty[name]]

    loaded = sorted({op[6] for op in k.ops if op[0] == LOAD})
    drained = sorted({d[0] for d in k.drains})
    read = sum(width(b) for b in loaded)
    write = sum(width(b) for b in drained)
    flops = 0
    for op in k.ops:
        if op[0] == FMA:
            flops += 2
        elif op[0] == BIN and op[1] in (0, 1, 2, 3):
            flops += 1
        elif op[0] == NEG:
            pass
    if k.reduction:
        flops += 1 if k.reduction[0] == 0 else 0
    return {"read": read, "write": write, "bytes": read + write, "flops": flops,
            "intensity": flops / (read + write) if read + write else 0.0}


# ---------------------------------------------------------------------------- GPU side
def _median_gbs(fn, nbytes: float, reps: int = 7, flush=None) -> tuple[float, list[float]]:
    import torch

    for _ in range(3):
        fn()
    runs = []
    for _ in range(reps):
        if flush is not None:
            flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        runs.append(nbytes / (s.elapsed_time(e) * 1e-3) / 1e9)
    return statistics.median(runs), [round(r, 1) for r in runs]


def measure_machine(out_machine: str, out_meas: str) -> dict:
    """Measure this GPU and write the lyth-machine/0.1 file and its measurement (build_machine):
    HBM read (sum partials), copy (copy2d) and triad (lerp) with this library's kernels over 2 GiB
    per buffer, FFMA and bf16 tensor peaks (cuBLAS SGEMM with TF32 off, and bf16 GEMM, at 8192),
    and the device's properties. Clocks are sampled, never set."""
    import subprocess

    import torch

    import lyth_b200 as lb

    dev = torch.device("cuda")
    props = torch.cuda.get_device_properties(0)
    n = 1 << 29  # 2 GiB per f32 buffer: 16x L2
    x = torch.rand(n, device=dev)
    y = torch.rand(n, device=dev)
    z = torch.empty(n, device=dev)
    part = torch.empty(int(lb.lib.lyth_b200_reduce_grid(n)), device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    _, read_runs = _median_gbs(lambda: lb.lib.lyth_b200_reduce_partials(
        0, n, x.data_ptr(), None, part.numel(), part.data_ptr(), stream), 4.0 * n)
    side = 1 << 14
    _, copy_runs = _median_gbs(lambda: lb.copy2d(x[:side * side].view(side, side), z[:side * side].view(side, side)),
                               8.0 * side * side)
    _, triad_runs = _median_gbs(lambda: lb.lerp(0.3, x, y, z), 12.0 * n)
    del x, y, z
    torch.backends.cuda.matmul.allow_tf32 = False
    a = torch.randn(8192, 8192, device=dev)
    b = torch.randn(8192, 8192, device=dev)
    _, f32_runs = _median_gbs(lambda: torch.matmul(a, b), 2.0 * 8192 ** 3)
    ab, bb = a.bfloat16(), b.bfloat16()
    _, bf16_runs = _median_gbs(lambda: torch.matmul(ab, bb), 2.0 * 8192 ** 3)
    del a, b, ab, bb
    try:
        clk = subprocess.run(["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,clocks.mem", "--format=csv,noheader,nounits",
                              "-i", "0"], capture_output=True, text=True, timeout=20).stdout.strip()
    except Exception:
        clk = "unavailable"
    device = {"name": props.name, "sm_count": props.multi_processor_count, "total_memory": props.total_memory,
              "l2_bytes": getattr(props, "L2_cache_size", None),
              "shared_optin": getattr(props, "shared_memory_per_block_optin", None), "clocks_sm_max_mem": clk}
    runs = {"read": read_runs, "copy": copy_runs, "triad": triad_runs,
            "sgemm_tflops": [round(r / 1e3, 2) for r in f32_runs], "bf16_tflops": [round(r / 1e3, 1) for r in bf16_runs]}
    machine, meas = build_machine(device, runs)
    for path, doc in ((out_machine, machine), (out_meas, meas)):
        if path:
            with open(path, "w") as f:
                json.dump(doc, f, indent=1)
                f.write("\n")
    return machine


def build_machine(device: dict, runs: dict) -> tuple[dict, dict]:
    """The machine file and its measurement from the probe's runs (GB/s per pattern, TFLOP/s):
    dram bandwidth_gbs = the median of the fastest pattern (read, copy or triad; a kernel that
    moves bytes another way cannot exceed it), peak_tflops = the SGEMM median, the ridge derived
    from the two. The L2, shared-memory and register levels carry no bandwidth: no probe here
    measures them with one long kernel, and a number made of short launches would describe the
    launch overhead (the reference leaves them at 0 for the same reason)."""
    med = {k: statistics.median(v) for k, v in runs.items()}
    best = max(("read", "copy", "triad"), key=lambda k: med[k])
    dram, peak, bf16 = round(med[best], 1), round(med["sgemm_tflops"], 2), round(med["bf16_tflops"], 1)
    machine = {
        "schema": MACHINE_SCHEMA, "id": "sm_100a", "isa": "sm_100a (precompiled, no PTX JIT)",
        "accepts": ["sm_120"],
        "accepts_note": "A `.lyth` source whose machine line says sm_120 runs against this file: every kernel class "
                        "of the back end computes the same bits on either machine, and the retarget is recorded "
                        "in lyth_b200_select's result (lyth_kernel.retargeted). Any other id is refused.",
        "device": device.get("name"),
        "peak_tflops": peak, "peak_tflops_bf16_tensor": bf16,
        "sm_count": device.get("sm_count"),
        "max_threads_per_block": 1024,
        "max_shared_bytes_per_block": 49152,
        "max_shared_bytes_per_block_optin": device.get("shared_optin") or 232448,
        "smem_banks": 32, "smem_bank_bytes": 4,
        "l2_bytes": device.get("l2_bytes"),
        "levels": [
            {"name": "dram", "capacity": f"{(device.get('total_memory') or 0) / 2**30:.0f} GiB HBM3e",
             "bandwidth_gbs": dram, "bandwidth_pattern": best,
             "bandwidth_gbs_by_pattern": {k: round(med[k], 1) for k in ("read", "copy", "triad")}, "latency_cyc": None},
            {"name": "l2", "capacity": f"{(device.get('l2_bytes') or 0) / 2**20:.0f} MiB (two dies)",
             "bandwidth_gbs": 0.0, "latency_cyc": None},
            {"name": "smem", "capacity": "228 KiB/SM, 227 KiB/block opt-in", "bandwidth_gbs": 0.0, "latency_cyc": None},
            {"name": "reg", "capacity": "64K x 32-bit per SM", "bandwidth_gbs": 0.0, "latency_cyc": None},
        ],
        "ops": [{"name": "fma.f32", "status": "present", "at": "reg"},
                {"name": "fma.f32x2", "status": "present", "at": "reg"},
                {"name": "tcgen05", "status": "present", "at": "sm"},
                {"name": "tma", "status": "present", "at": "sm"},
                {"name": "wgmma", "status": "absent", "at": "sm"}],
        "ridge_flop_per_byte": {"fp32": round(peak * 1e3 / dram, 3), "bf16_tensor": round(bf16 * 1e3 / dram, 2),
                                "note": "achieved over achieved: SGEMM (or bf16 GEMM) TFLOP/s over the dram bandwidth"},
        "notes": ["Every number is measured on a B200 by `python -m lyth_b200.probe machine`: read = this library's "
                  "sum-partials kernel over 2^29 f32 (4 B/element), copy = copy2d 16384^2 (8 B/element), triad = "
                  "lerp over 2^29 (12 B/element); peak_tflops = cuBLAS SGEMM n = 8192 with TF32 off; bf16 = cuBLAS "
                  "bf16 GEMM n = 8192. Medians of 7 timed runs after 3 warm-ups, CUDA events; every buffer is 16x L2.",
                  "smem banking (32 banks x 4 bytes) and the block limits are the device's properties.",
                  "lts__t_bytes on this two-die L2 counts about 1.5x the payload of a streaming kernel (copy2d: "
                  "12.15 B/element for 8 moved), so derived bytes are checked against DRAM read bytes, and the L2 "
                  "level only through that calibration."],
        "measurement": {"method": "python -m lyth_b200.probe machine", "runs": len(runs["read"]),
                        "clocks_sm_max_mem": device.get("clocks_sm_max_mem"),
                        "clock_state": "unlocked (default boost, never set by the probe)"},
    }
    meas = {"schema": MEASUREMENT_SCHEMA, "machine_id": "sm_100a", "source": "python -m lyth_b200.probe machine",
            "clock_state": "unlocked", "peak_tflops": peak,
            "levels": [{"name": "dram", "bandwidth_gbs": round(statistics.median(runs[best]), 1), "runs": runs[best]}],
            "runs": runs, "device": device}
    return machine, meas


def traffic_cases():
    """(name, kernel-name regex for ncu, elements, derived cost, run()) per class, every working
    set at least 4x L2 so the writes reach DRAM within the launch's lifetime as well as they can."""
    import torch

    import lyth_b200 as lb
    from lyth_b200 import circuit as cc
    from lyth_b200 import examples as ex

    dev = torch.device("cuda")
    out = []
    n = 1 << 27

    def streams():
        x, y, z = (torch.rand(n, device=dev) for _ in range(3))
        return x, y, z

    def add(name, regex, elements, kern, setup):
        out.append((name, regex, elements, derive_cost(kern), setup))

    add("saxpy", "saxpy_kernel", n, ex.saxpy(), lambda: (lambda t: (lambda: lb.saxpy(2.5, t[0], t[1])))(streams()))
    add("axpby", "axpby_kernel", n, ex.axpby(), lambda: (lambda t: (lambda: lb.axpby(1.5, 0.5, t[0], t[1])))(streams()))
    add("lerp", "lerp_kernel", n, ex.lerp(), lambda: (lambda t: (lambda: lb.lerp(0.3, t[0], t[1], t[2])))(streams()))
    add("horner", "horner_kernel", n, ex.horner(),
        lambda: (lambda t: (lambda: lb.horner(0.1, 0.2, 0.3, 0.4, t[0], t[1])))(streams()))
    side = 1 << 14

    def mats():
        return torch.rand(side, side, device=dev), torch.empty(side, side, device=dev)

    add("copy2d", "copy2d_kernel", side * side, ex.copy2d(), lambda: (lambda t: (lambda: lb.copy2d(t[0], t[1])))(mats()))
    add("transpose_tiled", "transpose_tiled", side * side, ex.transpose(True),
        lambda: (lambda t: (lambda: lb.transpose_tiled(t[0], t[1])))(mats()))
    m = 1 << 28
    add("sum", "sum_partials|reduce_partials", m, ex.reduction("sum"),
        lambda: (lambda x: (lambda: lb.reduce_partials(lb.SUM, x)))(torch.rand(m, device=dev)))
    add("dot", "reduce_partials|dot", n, ex.reduction("dot"),
        lambda: (lambda t: (lambda: lb.reduce_partials(lb.SUM, t[0], t[1])))(streams()))
    q = 27
    nq = 1 << q
    H8 = cc.f32s(cc.H)

    def state():
        return torch.rand(nq, device=dev), torch.rand(nq, device=dev)

    # the gate kernels' index space is the pair (quad): derived bytes per pair / per quad
    add("gate_q", "gate_q", nq // 2, ex.gate_q(), lambda: (lambda t: (lambda: lb.gate(1 << 10, H8, t[0], t[1])))(state()))
    wc, wt = cc.widths_ct(12, 13)
    add("swap_q", "swap_q|swap_kernel", nq // 4, ex.swap_q(),
        lambda: (lambda t: (lambda: lb.swap(wc, wt, t[0], t[1], t[0].clone(), t[1].clone())))(state()))
    return out


def run_traffic(only: str | None, reps: int) -> None:
    import torch

    for name, regex, elements, cost, setup in traffic_cases():
        if only and name != only:
            continue
        fn = setup()
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
        print(json.dumps({"case": name, "kernel_regex": regex, "elements": elements, "derived": cost}))
        del fn
        torch.cuda.empty_cache()


def report(csv_dir: str, out_md: str | None, tol: float = 0.02) -> list[dict]:
    """For every traffic case with a capture `<csv_dir>/<name>.csv` (one launch), the derived bytes
    per element against ncu's DRAM bytes, per direction, and the L2 total."""
    rows = []
    import glob

    meta = {}
    for p in glob.glob(os.path.join(csv_dir, "*.json")):
        with open(p) as f:
            for ln in f:
                if ln.startswith("{"):
                    d = json.loads(ln)
                    meta[d["case"]] = d
    for name, d in sorted(meta.items()):
        p = os.path.join(csv_dir, f"{name}.csv")
        if not os.path.exists(p):
            continue
        with open(p) as f:
            text = f.read()
        t = parse_ncu(text)
        n = t["launches"] or 1
        el = d["elements"] * n
        row = {"case": name, "elements": d["elements"], "el": el, "derived_read": d["derived"]["read"],
               "derived_write": d["derived"]["write"]}
        for direction, bpe in (("read", d["derived"]["read"]), ("write", d["derived"]["write"]),
                               ("all", d["derived"]["bytes"])):
            if bpe > 0:
                try:
                    row[direction] = compare(bpe, el, t, direction, tol)
                except NcuError as e:
                    row[direction] = {"verdict": "n/a", "why": str(e)}
        l2 = t["metrics"].get("lts__t_bytes.sum")
        if l2:
            row["l2_bytes_per_element"] = l2 / el
        rows.append(row)
    if out_md:
        with open(out_md, "w") as f:
            f.write(md_table(rows, tol))
    return rows


def md_table(rows, tol) -> str:
    lines = ["| class | elements x launches | derived R / W B/elem | DRAM read B/elem (ratio) | "
             f"DRAM write B/elem (ratio) | R+W verdict (tol {tol:.0%}) | L2 B/elem |",
             "|---|---:|---:|---:|---:|---|---:|"]
    for r in rows:
        def cell(d):
            if not d or "ratio" not in d:
                return (d or {}).get("verdict", "-")
            return f"{d['measured'] / r['el']:.3f} ({d['ratio']:.4f})"
        al = r.get("all") or {}
        lines.append(f"| {r['case']} | {r['el']:,.0f} | {r['derived_read']} / {r['derived_write']} | "
                     f"{cell(r.get('read'))} | {cell(r.get('write'))} | {al.get('verdict', '-')} | "
                     f"{r.get('l2_bytes_per_element', float('nan')):.3f} |")
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m lyth_b200.probe")
    sub = ap.add_subparsers(dest="cmd", required=True)
    m = sub.add_parser("machine", help="measure this GPU; write the machine file and its measurement")
    m.add_argument("--out", default=MACHINE_FILE)
    m.add_argument("--meas", default=None)
    t = sub.add_parser("traffic", help="run each kernel class (or one) for an ncu capture")
    t.add_argument("--case", default=None)
    t.add_argument("--reps", type=int, default=1)
    t.add_argument("--list", action="store_true")
    r = sub.add_parser("report", help="derived bytes/element against the ncu captures in a directory")
    r.add_argument("dir")
    r.add_argument("--out", default=None)
    r.add_argument("--tol", type=float, default=0.02)
    c = sub.add_parser("check", help="machine-check: a machine file against a measurement")
    c.add_argument("machine")
    c.add_argument("measurement")
    c.add_argument("--tol", type=float, default=0.05)
    a = ap.parse_args(argv)
    if a.cmd == "machine":
        print(json.dumps(measure_machine(a.out, a.meas), indent=1))
    elif a.cmd == "traffic":
        if a.list:
            for name, regex, *_ in traffic_cases():
                print(name, regex)
        else:
            run_traffic(a.case, a.reps)
    elif a.cmd == "report":
        for row in report(a.dir, a.out, a.tol):
            print(json.dumps(row))
    else:
        with open(a.machine) as f1, open(a.measurement) as f2:
            v = check_machine(json.load(f1), json.load(f2), a.tol)
        print(json.dumps(v, indent=1))
        return 0 if v["verdict"] == "pass" else 1
    return 0


if __name__ == "__main__":
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    sys.exit(main())
