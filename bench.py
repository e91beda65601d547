#!/usr/bin/env python
"""bench.py -- the headline measurement of lyth_b200 on B200.

Metric: 33-qubit state-vector gates/s at 1-8 GPUs, and HBM GB/s (% of the
measured B200 peak) per kernel class.

One JSON line on rank 0:
  * value      whole-job gates/s of the layered circuit (H on every qubit, CU(phase) on adjacent
               pairs, SWAP on a random pairing; 81 gates per layer at 33 qubits) from a seeded
               random normalised state resident in HBM; one step = one layer; strong scaling
               (33 qubits at every N, sharded on the high qubits). Device time (CUDA events on
               the engine's stream), max over ranks.
  * roofline   the dominant kernel (the fused pass, tile_pass_kernel: one pass per group of
               consecutive gates on <= 13 qubits): algorithmic bytes (16 B per amplitude: read
               and write re and im once) / its average device duration inside the timed region;
               traffic = DRAM bytes per launch from an ncu capture of the same kernel, scaled.
  * e2e        the same metric through the public API with host buffers: each step uploads the
               shard from pinned host memory, applies the layer, and reads the shard back.
  * cpu_baseline  the host evaluator port (oracle/) on a bounded sample, rank 0, N = 1.
  * per_kernel HBM GB/s of every other kernel class at its BASELINE config (rank 0, N = 1).
  * sharded_streams  at N > 1: saxpy over 2^33 elements split into one contiguous range per rank
               (independent units, no collective), aggregate GB/s over the max of the ranks'
               device times.

``--impl reference`` times the reference's algorithm on the host cores instead (the oracle
port: the reference is Rust and cannot be built in this image) and prints the same line.

Run: python bench.py [--gpus N] [--steps K] [--warmup W]; N > 1 under torch.distributed.run.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}
METRIC = "33-qubit statevector gates/s (HBM GB/s per kernel alongside)"
# DRAM bytes (read + write) per amplitude of one fused pass (tile_pass_kernel): the mean over the
# 12 launches of two layers of the benchmark circuit at 2^28 amplitudes (a 4 GiB state, 32x L2),
# ncu dram__bytes_read.sum + dram__bytes_write.sum (8.064 + 7.775); the algorithmic figure is 16.
# Traffic grows with the amplitudes a launch processes, so a launch's traffic is this x its
# amplitudes.
FUSED_PASS_DRAM_BYTES_PER_AMP = 15.839
L2_BYTES = 126 * 1024 * 1024


def circuit_module():
    """lyth_b200/circuit.py (the host side of lyth-circuit: gates, Rng, circuits) loaded by path,
    without importing the lyth_b200 package: the reference arm must map no library of this
    repository except the oracle's."""
    import importlib.util

    name = "lyth_circuit_host"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "lyth_b200", "circuit.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def machine_file_peak():
    """The dram bandwidth of fixtures/machine/sm_100a.json (lyth-machine/0.1, measured by
    `python -m lyth_b200.probe machine`), or None."""
    try:
        with open(os.path.join(ROOT, "fixtures", "machine", "sm_100a.json")) as f:
            m = json.load(f)
        return next(lv["bandwidth_gbs"] for lv in m["levels"] if lv["name"] == "dram")
    except Exception:
        return None


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--qubits", type=int, default=33)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--skip-kernels", action="store_true", help="omit the per-kernel table")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-streams", action="store_true", help="omit the sharded-stream line at N > 1")
    ap.add_argument("--cpu-qubits", type=int, default=30, help="host state size of the cpu_baseline sample")
    ap.add_argument("--ref-qubits", type=int, default=30, help="host state size of the reference arm's steps")
    ap.add_argument("--ref-gates", type=int, default=1, help="gates per reference-arm step")
    ap.add_argument("--parity-qubits", type=int, default=22)
    ap.add_argument("--skip-parity", action="store_true")
    ap.add_argument("--fuse", type=int, default=None, help="max qubits per fused pass (1..13; default: the engine's)")
    ap.add_argument("--swap-batch", type=int, default=None,
                    help="most rank-bit qubits per swap-in (1..6; default: the engine's)")
    ap.add_argument("--transport", choices=["copy_engine", "peer_load", "mixed", "peer_store", "nccl"], default=None,
                    help="swap-in transport at N > 1 (default: the engine's, mixed when every rank maps every peer)")
    ap.add_argument("--pull-queues", type=int, default=None,
                    help="copy-engine queues per swap-in pull at N > 1 (1..8; default: the engine's, one per partner slice)")
    ap.add_argument("--diagonal", type=int, choices=[0, 1], default=None,
                    help="diagonal rank-bit gates without an exchange (1) or like any other gate (0); "
                         "default: the engine's")
    ap.add_argument("--case", default=None, help="run one kernel case (small config) and exit")
    ap.add_argument("--case-reps", type=int, default=3)
    ap.add_argument("--list-cases", action="store_true")
    return ap.parse_args()


# --------------------------------------------------------------------------- clocks
class Clocks:
    """nvidia-smi sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.lines: list[str] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", self.gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_id_for(dev_index: int) -> str:
    import torch

    try:
        u = str(torch.cuda.get_device_properties(dev_index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            return vis.split(",")[dev_index]
        return str(dev_index)


# --------------------------------------------------------------------------- distributed
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self):
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(self.local)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if not self.pg:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def min(self, v: float) -> float:
        if not self.pg:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MIN)
        return float(t.item())

    def bcast_bytes(self, b: bytes | None) -> bytes:
        if not self.pg:
            return b
        obj = [b]
        self.pg.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


# --------------------------------------------------------------------------- CPU baseline
def host_state(qubits: int, seed: int = 3):
    """A seeded random state for the host samples: re, im ~ U[-1, 1) from two SplitMix64 streams
    (the oracle's generator), scaled in place to unit norm (f64 sum over chunks). Two arrays of
    2^qubits f32 and nothing else, so a 30-qubit sample holds 8 GiB."""
    import numpy as np

    from oracle import oracle as orc

    n = 1 << qubits
    re, im = orc.uniform(seed, n), orc.uniform(seed + 1, n)
    norm2, step = 0.0, 1 << 24
    for a in (re, im):
        for i in range(0, n, step):
            c = a[i:i + step].astype(np.float64)
            norm2 += float(np.dot(c, c))
    f = np.float32(1.0 / np.sqrt(norm2))
    re *= f
    im *= f
    return re, im


def apply_host_gate(cc, orc, g, re, im):
    """One gate of the circuit with the host evaluator port, unfused, in place (lyth-circuit's
    execute on the host: gate_q / cu_q / swap_q over the whole state)."""
    if isinstance(g, cc.U):
        orc.gate_q(1 << g.q, cc.f32s(g.m), re, im, inplace=True)
    elif isinstance(g, cc.CU):
        wc, wt = orc.widths_ct(g.c, g.t)
        orc.cu_q(wc, wt, cc.f32s(g.m), re, im, inplace=True)
    else:
        wc, wt = orc.widths_ct(g.a, g.b)
        orc.swap_q(wc, wt, re, im, inplace=True)


class HostSample:
    """The host evaluator port applying the benchmark circuit's gates on a 2^qubits state, all host
    cores. Each `run(ngates)` applies the next gates of the circuit in order and returns the seconds
    it took; work per gate is one pass over the state, so gates/s at 33 qubits is gates/s at this
    size x 2^(qubits - 33)."""

    def __init__(self, qubits: int, qubits_config: int = 33):
        cc = circuit_module()
        from oracle import oracle as orc

        self.cc, self.orc, self.q, self.qc = cc, orc, qubits, qubits_config
        # the layered circuit at the sample's size: the 33-qubit layer's gate mix (H on every qubit,
        # CU(phase) on adjacent pairs, SWAP on a random pairing) in circuit order
        self.gates = cc.layered(qubits, 2, cc.Rng(cc.BENCH_SEED))
        self.re, self.im = host_state(qubits)
        self.pos = 0

    def run(self, ngates: int) -> float:
        t0 = time.perf_counter()
        for _ in range(ngates):
            g = self.gates[self.pos % len(self.gates)]
            apply_host_gate(self.cc, self.orc, g, self.re, self.im)
            self.pos += 1
        return time.perf_counter() - t0

    def scale(self) -> float:
        return float(2.0 ** (self.q - self.qc))

    def cores(self) -> int:
        return self.orc.threads()

    def describe(self, ngates: int) -> str:
        return (f"{ngates} gate(s) per step of the layered circuit (H, CU(phase), SWAP in circuit order) applied "
                f"by the host evaluator port (oracle/lythref.c, unfused, in place) to a {self.q}-qubit state "
                f"(2^{self.q} amplitudes) on {self.cores()} host threads; gates/s scaled to {self.qc} qubits by "
                f"2^{self.q - self.qc} (each gate is one pass over the state, so its work is linear in the state)")


def cpu_sample(qubits: int, budget_s: float = 15.0) -> dict:
    """The host evaluator port on a bounded sample (about budget_s of host time) of the benchmark
    circuit's gates on a 2^qubits state, all host cores; gates/s scaled to 33 qubits."""
    hs = HostSample(qubits)
    done, dt = 0, 0.0
    while dt < budget_s:
        dt += hs.run(1)
        done += 1
    gps = done / dt
    return {"gates": done, "seconds": dt, "gates_per_s_at_sample": gps,
            "gates_per_s_at_33": gps * hs.scale(), "cores": hs.cores(),
            "sample": f"{done} gates in {dt:.1f} s: " + hs.describe(1)}


def reference_arm(a, dist: Dist) -> None:
    """--impl reference: the reference's algorithm on the host cores -- its host evaluator, as the
    oracle port (the Rust reference cannot be built in this image) -- on this arm's config. Rank 0
    only; the other ranks exit without work. One step = a bounded sample of the 33-qubit layered
    circuit: `--ref-gates` gates applied to a `--ref-qubits` state (default 30 qubits, the BASELINE
    single-GPU size, 8 GiB of host memory), gates/s scaled to 33 qubits. No library of this
    repository is loaded except the oracle's (the circuit generator is read by path)."""
    if dist.rank != 0:
        return
    hs = HostSample(a.ref_qubits)
    for _ in range(a.warmup):
        hs.run(1)
    secs = [hs.run(a.ref_gates) for _ in range(a.steps)]
    t = sum(secs)
    v = a.ref_gates * a.steps / t * hs.scale()
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "gates/s", "n_gpus": a.gpus,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1000.0 * t / a.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: SplitMix64-seeded random state scaled to unit norm; layered circuit seed 20260930",
        "config": config_of(33, 81, a.gpus),
        "step": f"{a.ref_gates} gate(s) of the 33-qubit layer on a {a.ref_qubits}-qubit host state "
                f"(ms_per_step is that sample's host time)",
        "cpu_baseline": {"value": v, "unit": "gates/s", "cores": hs.cores(), "kind": "port",
                         "sample": hs.describe(a.ref_gates)},
        "e2e": {"value": v, "unit": "gates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "QuantumDrizzy/LYTH is Rust (no cargo/rustc in this image); its host evaluator is timed "
                "through this repository's C restatement of it (oracle/lythref.c)",
    }
    print(json.dumps(line), flush=True)


def config_of(q: int, per: int, world: int) -> dict:
    import math

    return {"workload": f"statevector layered circuit, {q} qubits, {per} gates per layer "
                        "(H on every qubit, CU(phase) on adjacent pairs, SWAP on a random pairing), one step = one layer",
            "qubits": q, "gates_per_step": per, "global_qubits": int(math.log2(world)) if world > 1 else 0,
            "parallelism": f"sharded on the high {int(math.log2(world))} qubits" if world > 1 else "1 GPU, in place",
            "l2": f"inputs larger than L2: the state is {8 * (1 << q) / 2**30:.0f} GiB"}


# --------------------------------------------------------------------------- per-kernel table
def kernel_cases(dev, small: bool = False):
    """Named cases, each (setup -> (callable, algorithmic bytes or flops, kind)). The BASELINE
    configs; `small` shrinks the large ones for an ncu capture (inputs still larger than L2)."""
    import torch

    import lyth_b200 as lb

    g = torch.Generator(device=dev)
    g.manual_seed(1)
    cases = {}

    def stream_case(name, p, body, nbytes_per):
        def setup():
            n = 1 << p
            x = torch.rand(n, device=dev, generator=g)
            y = torch.rand(n, device=dev, generator=g)
            z = torch.empty_like(x)
            return (lambda: body(x, y, z)), nbytes_per * n, "bytes"
        cases[name] = setup

    for p in (20, 22, 24, 26, 28, 30):
        if not small or p == 26:
            stream_case(f"saxpy_2^{p}", p, lambda x, y, z: lb.saxpy(2.5, x, y), 12.0)
    P = 26 if small else 28
    stream_case(f"axpby_2^{P}", P, lambda x, y, z: lb.axpby(1.5, 0.5, x, y), 12.0)
    stream_case(f"lerp_2^{P}", P, lambda x, y, z: lb.lerp(0.3, x, y, z), 12.0)
    stream_case(f"horner_2^{P}", P, lambda x, y, z: lb.horner(0.1, 0.2, 0.3, 0.4, x, z), 8.0)
    stream_case(f"sum_2^{P}", P, lambda x, y, z: lb.reduce_partials(lb.SUM, x), 4.0)
    stream_case(f"max_2^{P}", P, lambda x, y, z: lb.reduce_partials(lb.MAX, x), 4.0)
    stream_case(f"dot_2^{P}", P, lambda x, y, z: lb.reduce_partials(lb.SUM, x, y), 8.0)

    def transpose_case(name, fn):
        def setup():
            a = torch.rand(4096, 4096, device=dev, generator=g)
            b = torch.empty(4096, 4096, device=dev)
            return (lambda: fn(a, b)), 8.0 * 4096 * 4096, "bytes"
        cases[name] = setup

    transpose_case("transpose_tiled_4096", lb.transpose_tiled)
    transpose_case("copy2d_4096", lb.copy2d)
    transpose_case("transpose_naive_4096", lb.transpose_naive)

    def big_transpose_case(name, fn, side):
        def setup():
            a = torch.rand(side, side, device=dev, generator=g)
            b = torch.empty(side, side, device=dev)
            return (lambda: fn(a, b)), 8.0 * side * side, "bytes"
        cases[name] = setup

    # at 16x L2 (2 GiB moved): the HBM figures of the transpose and its coalesced control
    S = 8192 if small else 16384
    big_transpose_case(f"transpose_tiled_{S}", lb.transpose_tiled, S)
    big_transpose_case(f"copy2d_{S}", lb.copy2d, S)

    def narrow_case(name, p, body, nbytes_per, dt):
        def setup():
            n = 1 << p
            x = torch.rand(n, device=dev, generator=g).to(dt)
            y = torch.rand(n, device=dev, generator=g).to(dt)
            return (lambda: body(x, y)), nbytes_per * n, "bytes"
        cases[name] = setup

    # ADR-0024 narrow storage: the same kernels at half the bytes
    narrow_case(f"saxpy_bf16_2^{P}", P, lambda x, y: lb.stream_narrow(lb.STREAM_SAXPY, [2.5], x, y, y), 6.0,
                torch.bfloat16)
    narrow_case(f"saxpy_f16_2^{P}", P, lambda x, y: lb.stream_narrow(lb.STREAM_SAXPY, [2.5], x, y, y), 6.0,
                torch.float16)
    narrow_case(f"sum_bf16_2^{P}", P, lambda x, y: lb.reduce_partials_narrow(lb.SUM, x), 2.0, torch.bfloat16)

    def narrow_transpose_case(name, side):
        def setup():
            a = torch.rand(side, side, device=dev, generator=g).to(torch.bfloat16)
            b = torch.empty(side, side, device=dev, dtype=torch.bfloat16)
            return (lambda: lb.transpose_narrow(a, b)), 4.0 * side * side, "bytes"
        cases[name] = setup

    narrow_transpose_case(f"transpose_bf16_{S}", S)

    def gemv_case(name, fmt):
        def setup():
            rows, k, grp = 14336, 4096, 64
            w = torch.randint(0, 256, (rows, k // 2), dtype=torch.uint8, device=dev, generator=g)
            sc = (torch.rand(rows * (k // grp), device=dev, generator=g) * 0.02).half()
            xv = torch.randn(k, device=dev, generator=g).half()
            yv = torch.empty(rows, dtype=torch.float16, device=dev)
            nbytes = rows * k / 2 + rows * (k // grp) * 2 + k * 2 + rows * 2
            return (lambda: lb.gemv_q4(fmt, w, sc, xv, yv, grp)), nbytes, "bytes"
        cases[name] = setup

    gemv_case("gemv_int4_4096x14336", lb.GEMV_INT4)
    gemv_case("gemv_nf4_4096x14336", lb.GEMV_NF4)

    def mm_case(name, fn, m, dtype=torch.float32):
        # operands made (and rounded to the storage type) in setup: only the contraction is timed
        def setup():
            A = (torch.randn(m, m, device=dev, generator=g) / 64.0).to(dtype)
            B = (torch.randn(m, m, device=dev, generator=g) / 64.0).to(dtype)
            C = torch.empty(m, m, device=dev)
            return (lambda: fn(A, B, C)), 2.0 * m ** 3, "flops"
        cases[name] = setup

    M = 2048 if small else 4096
    mm_case(f"matmul_f32_ffma_{M}", lambda A, B, C: lb.matmul_f32(A, B, C, exact=False), M)
    mm_case(f"matmul_f32_exact_{M}", lambda A, B, C: lb.matmul_f32(A, B, C, exact=True), M)
    mm_case(f"matmul_bf16_{M}", lambda A, B, C: lb.matmul_bf16(A, B, C), M, torch.bfloat16)
    mm_case(f"matmul_bf16_1sm_{M}", lambda A, B, C: lb.matmul_bf16(A, B, C, pair=False), M, torch.bfloat16)

    def gate_case(name, q, fn):
        def setup():
            n = 1 << q
            re = torch.rand(n, device=dev, generator=g)
            im = torch.rand(n, device=dev, generator=g)
            return (lambda: fn(n, re, im)), 16.0 * n if "cu" not in name else 8.0 * n, "bytes"
        cases[name] = setup

    from lyth_b200 import circuit as cc

    Q = 28 if small else 30
    H8 = cc.f32s(cc.H)
    gate_case(f"gate_q_q10_2^{Q}", Q, lambda n, re, im: lb.gate(1 << 10, H8, re, im))
    gate_case(f"gate_q_q0_2^{Q}", Q, lambda n, re, im: lb.gate(1, H8, re, im))
    wc, wt = cc.widths_ct(12, 13)
    gate_case(f"cu_q_inplace_12_13_2^{Q}", Q, lambda n, re, im: lb.cu(wc, wt, cc.f32s(cc.phase(0.3)), re, im))
    return cases


def per_kernel(pk: dict, only: str | None = None, small: bool = False, reps: int = 10) -> dict:
    """HBM GB/s (or TFLOP/s) of each kernel class at its BASELINE config: CUDA events on the
    current stream, L2 flushed before every timed launch by READING a 256 MiB buffer (a read
    leaves clean lines, so no write-back lands inside the timed window), median of the reps."""
    import torch

    import lyth_b200 as lb

    dev = torch.device("cuda")
    hbm = pk["hbm_gbs"]
    flush = torch.ones(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    sink = torch.empty(1, device=dev)
    ffma_peak = 148 * 128 * 2 * pk.get("sm_max_mhz", 1965.0) * 1e6 / 1e12
    out = {}
    for name, setup in kernel_cases(dev, small).items():
        if only and name != only:
            continue
        try:
            fn, amount, kind = setup()
        except Exception as e:  # a case whose entry point refuses (e.g. an unsupported shape)
            out[name] = {"unavailable": str(e)[:160]}
            continue
        try:
            for _ in range(3):
                fn()
            ts = []
            for _ in range(reps):
                torch.sum(flush, dim=0, keepdim=True, out=sink)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                fn()
                e.record()
                e.synchronize()
                ts.append(s.elapsed_time(e))
        except Exception as e:
            out[name] = {"unavailable": str(e)[:160]}
            continue
        ms = statistics.median(ts)
        if kind == "bytes":
            gbs = amount / (ms * 1e-3) / 1e9
            out[name] = {"GB_s": round(gbs, 1), "frac_hbm": round(gbs / hbm, 4), "ms": round(ms, 5),
                         "bytes": int(amount)}
        else:
            tf = amount / (ms * 1e-3) / 1e12
            r = {"TFLOP_s": round(tf, 2), "ms": round(ms, 4)}
            if "bf16" in name:
                r["frac_bf16_measured"] = round(tf / pk["bf16_tflops"], 4)
                if "1sm" not in name:
                    r["cta_pairs"] = int(lb.lib.lyth_b200_matmul_bf16_pairs())
            else:
                r["frac_fp32_nominal"] = round(tf / ffma_peak, 4)
                r["fp32_nominal_tflops"] = round(ffma_peak, 1)
            out[name] = r
        del fn
        torch.cuda.empty_cache()
    return out


def run_case(name: str, reps: int) -> None:
    """--case NAME: one kernel case on its small config, `reps` launches (for an ncu capture).
    `sv_layer_2^Q` runs `reps` layers of the benchmark circuit on a Q-qubit state (the engine's
    fused passes, as in the headline)."""
    import torch

    torch.cuda.set_device(0)
    if name.startswith("sv_layer_2^"):
        import lyth_b200 as lb
        from lyth_b200 import circuit as cc

        q = int(name.split("^")[1])
        gates = cc.layered(q, reps, cc.Rng(cc.BENCH_SEED))
        with lb.StateVector(q, device=0) as sv:
            sv.init_random(cc.BENCH_SEED)
            sv.apply(gates)
            sv.sync()
            st = sv.stats()
        print(json.dumps({"case": name, "layers": reps, "passes": st["passes"], "bytes_per_pass": 16 << q}))
        return
    cases = kernel_cases(torch.device("cuda"), small=True)
    fn, amount, kind = cases[name]()
    for _ in range(reps):
        fn()
    torch.cuda.synchronize()
    print(json.dumps({"case": name, "reps": reps, kind: amount}))


# --------------------------------------------------------------------------- sharded streams
def sharded_streams(dist: Dist, peak: float, log2n: int = 33, reps: int = 5) -> dict:
    """saxpy over 2^log2n elements, one contiguous range per rank (lyth_b200.stream_range): the
    large streams shard as independent units with no collective on the data path. Device time of
    `reps` launches per rank, max over ranks. Afterwards every rank checks its range: 4096 sampled
    elements of y (and the range's first and last) against fma(2.5, x, y0) applied once per launch
    on the host (the evaluator's saxpy), from saved copies of x and y0, and the ranges must tile [0, n) exactly. Every rank
    takes the same collective steps whatever happens locally, so a local failure is reported
    instead of hanging the others."""
    import numpy as np
    import torch

    import lyth_b200 as lb

    n = 1 << log2n
    off, cnt = lb.stream_range(n, dist.rank, dist.world)
    ok, ms, x, y, launches = 1.0, 0.0, None, None, 0
    idx = None
    try:
        x = torch.empty(cnt, dtype=torch.float32, device="cuda").uniform_(-1.0, 1.0)
        y = torch.empty(cnt, dtype=torch.float32, device="cuda").uniform_(-1.0, 1.0)
        g = np.random.default_rng(dist.rank)
        idx = torch.from_numpy(np.unique(np.concatenate([[0, cnt - 1], g.integers(0, cnt, 4096)]))).cuda()
        xs, y0s = x[idx].cpu().numpy(), y[idx].cpu().numpy()
        for _ in range(3):
            lb.saxpy(2.5, x, y)
            launches += 1
        torch.cuda.synchronize()
    except Exception:
        ok = 0.0
    dist.barrier()
    if ok:
        try:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                lb.saxpy(2.5, x, y)
                launches += 1
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            from oracle import oracle as orc

            want = y0s.copy()
            for _ in range(launches):
                want = orc.saxpy(2.5, xs, want)
            got = y[idx].cpu().numpy()
            if not np.array_equal(got.view(np.uint32), want.view(np.uint32)):
                ok = 0.0
        except Exception:
            ok = 0.0
    dist.barrier()
    ms = dist.max(ms)
    failed = dist.sum(1.0 - ok)
    covered = dist.sum(float(cnt))
    # contiguity: rank r's range must start where rank r-1's ended
    ends = [None] * dist.world
    if dist.pg:
        dist.pg.all_gather_object(ends, (off, cnt))
    else:
        ends = [(off, cnt)]
    tiles = all(ends[i][0] + ends[i][1] == ends[i + 1][0] for i in range(len(ends) - 1)) and ends[0][0] == 0
    del x, y
    torch.cuda.empty_cache()
    if failed:
        return {"error": f"{int(failed)} rank(s) could not run or verify their range"}
    if int(covered) != n or not tiles:
        return {"error": f"the ranges do not tile [0, {n}): {ends}"}
    gbs = 12.0 * n / (ms * 1e-3) / 1e9
    return {"kernel": "saxpy", "elements": n, "elements_per_rank": cnt, "ms": round(ms, 4),
            "GB_s_aggregate": round(gbs, 1), "frac_hbm_per_gpu": round(gbs / dist.world / peak, 4),
            "collective": "none", "l2": "inputs larger than L2",
            "verified": "ranges tile [0, n); 4098 sampled elements per rank bit-exact vs fma on the host"}


# --------------------------------------------------------------------------- parity before timing
def configure(sv, a, dist: Dist) -> None:
    """The engine settings of the command line (collective ones on every rank alike)."""
    import lyth_b200 as lb

    if a.fuse:
        sv.set_fusion(a.fuse)
    if a.swap_batch:
        sv.set_swap_batch(a.swap_batch)
    if a.diagonal is not None:
        sv.set_diagonal(bool(a.diagonal))
    if a.transport and dist.world > 1:
        sv.set_transport(a.transport)
    if a.pull_queues and dist.world > 1:
        lb.check(lb.lib.lyth_sv_set_pull_queues(sv._h, a.pull_queues), "set_pull_queues")


def sharded_parity(a, dist: Dist) -> dict:
    """Bit-exactness on the same N ranks, before anything is timed: a `--parity-qubits` (default 22)
    state sharded over the N ranks exactly as the timed run shards its state, with the timed run's
    engine settings, two layers of the layered circuit through the engine (tile passes, swap-ins of
    rank-bit qubits, diagonal rank-bit gates as scalars, SWAPs as relabels, read-out undoing the
    qubit map), and every rank's shard compared bit for bit with the
    host evaluator applying the same gates unfused in order to the same input
    (crates/lyth-circuit/tests/fusion.rs:53-92). Every rank takes the same collective steps
    whatever happens locally; `ok` is the minimum over ranks."""
    import numpy as np

    import lyth_b200 as lb
    from lyth_b200 import circuit as cc
    from oracle import oracle as orc

    q = a.parity_qubits
    ok, detail, gates, st = 1.0, "", [], {}
    nid = lb.unique_id() if (dist.world > 1 and dist.rank == 0) else None
    nid = dist.bcast_bytes(nid)
    try:
        gates = cc.layered(q, 2, cc.Rng(cc.BENCH_SEED + 1))
        re0, im0 = orc.random_state(cc.BENCH_SEED + 1, q)
        orc.set_threads(max(1, (os.cpu_count() or 1) // dist.world))
        wr, wi = orc.run_gates(cc.as_tuples(gates), re0.copy(), im0.copy(), inplace=True)
        with lb.StateVector(q, device=dist.local, rank=dist.rank, nranks=dist.world, nccl_id=nid) as sv:
            configure(sv, a, dist)
            n = sv.local_len
            lo = dist.rank * n
            sv.set_local(np.ascontiguousarray(re0[lo:lo + n]), np.ascontiguousarray(im0[lo:lo + n]))
            sv.apply(gates)
            sv.sync()
            gr, gi = np.empty(n, np.float32), np.empty(n, np.float32)
            sv.get_local(gr, gi)
            st = sv.stats()
        bad = int(np.count_nonzero(gr.view(np.uint32) != wr[lo:lo + n].view(np.uint32)))
        bad += int(np.count_nonzero(gi.view(np.uint32) != wi[lo:lo + n].view(np.uint32)))
        if bad:
            ok, detail = 0.0, f"rank {dist.rank}: {bad} words differ"
    except Exception as e:  # reported, not raised: the other ranks still take the same steps
        ok, detail, st = 0.0, f"rank {dist.rank}: {type(e).__name__}: {str(e)[:120]}", {}
    ok = dist.min(ok)
    out = {"ok": bool(ok), "qubits": q, "ranks": dist.world, "layers": 2, "gates": len(gates),
           "compare": "every rank's shard, bit for bit, against the host evaluator (unfused, in order)",
           "engine_passes": st.get("passes"), "engine_exchanges": st.get("exchanges")}
    if detail:
        out["detail"] = detail
    return out


# --------------------------------------------------------------------------- our arm
def ours(a, dist: Dist) -> None:
    import numpy as np
    import torch

    import lyth_b200 as lb
    from lyth_b200 import circuit as cc
    from lyth_b200.statevector import gates_array

    pk, pk_kind = peaks()
    q = a.qubits
    parity = None if a.skip_parity else sharded_parity(a, dist)
    if parity is not None and not parity["ok"]:
        if dist.rank == 0:
            print(json.dumps({"metric": METRIC, "value": None, "unit": "gates/s", "n_gpus": dist.world,
                              "error": "parity check failed: no value is reported", "parity": parity}), flush=True)
        return
    nid = lb.unique_id() if (dist.world > 1 and dist.rank == 0) else None
    nid = dist.bcast_bytes(nid)
    sv = lb.StateVector(q, device=dist.local, rank=dist.rank, nranks=dist.world, nccl_id=nid)
    configure(sv, a, dist)
    total_layers = a.warmup + a.steps
    gates = cc.layered(q, total_layers, cc.Rng(cc.BENCH_SEED))
    per = len(gates) // total_layers
    layers = [gates_array(gates[i * per:(i + 1) * per]) for i in range(total_layers)]
    # The warm-up layers and the timed layers each go to the engine as one gate list, as a user
    # applies a circuit: the engine then sees the layers ahead when it picks which local qubit to
    # trade for a rank-bit one. Per-step time is the timed region over the K layers.
    warm_arr = gates_array(gates[:a.warmup * per])
    timed_arr = gates_array(gates[a.warmup * per:])
    sv.init_random(cc.BENCH_SEED)
    lb.check(lb.lib.lyth_sv_apply(sv._h, warm_arr, a.warmup * per), "apply")
    sv.sync()
    stream = torch.cuda.ExternalStream(sv.stream)
    clocks = Clocks(gpu_id_for(dist.local))
    launches0 = sv.stats()["launches"]
    sent0 = sv.stats()["bytes_sent"]
    sv.reset_timing()
    sv.set_timing(True)
    dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    lb.check(lb.lib.lyth_sv_apply(sv._h, timed_arr, a.steps * per), "apply")
    t_end.record(stream)
    sv.sync()
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop()
    ms_local = t_start.elapsed_time(t_end)
    ms = dist.max(ms_local)
    sv.set_timing(False)
    tim = sv.timing()
    launches = dist.sum(float(sv.stats()["launches"] - launches0))
    st = sv.stats()
    sv_transport = sv.transport
    gates_timed = a.steps * per
    value = gates_timed / (ms * 1e-3)

    # roofline of the dominant kernel: the in-place fused pass (every amplitude read and written
    # once: 16 B per local amplitude per launch); the single-gate passes are reported beside it.
    def cls_row(n_ms, bytes_per_launch):
        n, tot = n_ms
        if not n:
            return None
        avg = tot / n
        return {"launches": n, "avg_ms": round(avg, 4), "GB_s": round(bytes_per_launch / (avg * 1e-3) / 1e9, 1)}

    pass_bytes = 16.0 * sv.local_len
    dominant = "fused" if tim["fused"][0] else "u"
    d_n, d_ms = tim[dominant]
    d_avg = d_ms / d_n if d_n else float("nan")
    achieved = pass_bytes / (d_avg * 1e-3) / 1e9 if d_n else None
    peak = pk["hbm_gbs"]
    roofline = {"bound": "hbm", "achieved": round(achieved, 1) if achieved else None, "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4) if achieved else None, "traffic": None,
                "peak_source": pk_kind,
                "kernel": "tile_pass_kernel (fused pass: <= 13 qubits, in place, TMA-staged 2^13-amplitude tiles)"
                if dominant == "fused" else "gate_q_kernel (in-place 1-qubit pass)",
                "algorithmic_bytes_per_launch": int(pass_bytes), "avg_launch_ms": round(d_avg, 4),
                "launches_timed": d_n,
                "share_of_timed_region": round(d_ms / ms, 4) if ms else None,
                "single_u_pass": cls_row(tim["u"], pass_bytes),
                "single_cu_pass": cls_row(tim["cu"], 8.0 * sv.local_len),
                "exchange": {"gates": tim["exchange"][0],
                             "avg_ms": round(tim["exchange"][1] / tim["exchange"][0], 4) if tim["exchange"][0] else None},
                "swap_in": {"count": tim["swap"][0],
                            "avg_ms": round(tim["swap"][1] / tim["swap"][0], 4) if tim["swap"][0] else None,
                            # what this rank sent in its swap-ins (half the shard for a pairwise
                            # one, (2^k - 1) / 2^k for a batched one among 2^k ranks) over their
                            # device time; as much arrives
                            "GB_s_each_way": round((st["bytes_sent"] - sent0) / (tim["swap"][1] * 1e-3) / 1e9, 1)
                            if tim["swap"][0] and not tim["exchange"][0] else None,
                            "share_of_timed_region": round(tim["swap"][1] / ms, 4) if ms else None}}
    mf = machine_file_peak()
    if mf and achieved:
        roofline["machine_file"] = {"peak": mf, "frac": round(achieved / mf, 4),
                                    "source": "fixtures/machine/sm_100a.json dram bandwidth_gbs (triad pattern)"}
    if dominant == "fused" and FUSED_PASS_DRAM_BYTES_PER_AMP:
        roofline["traffic"] = int(FUSED_PASS_DRAM_BYTES_PER_AMP * sv.local_len)

    # e2e: upload the shard from pinned host memory, apply one layer, read the shard back.
    e2e = None
    if not a.skip_e2e:
        hre = torch.empty(sv.local_len, dtype=torch.float32, pin_memory=True)
        him = torch.empty(sv.local_len, dtype=torch.float32, pin_memory=True)
        sv.get_local(hre.data_ptr(), him.data_ptr())
        order = [a.warmup + (i % a.steps) for i in range(1 + a.e2e_steps)]
        times = []
        for j, li in enumerate(order):
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            sv.set_local(hre.data_ptr(), him.data_ptr())
            lb.check(lb.lib.lyth_sv_apply(sv._h, layers[li], per), "apply")
            sv.get_local(hre.data_ptr(), him.data_ptr())
            e1.record(stream)
            e1.synchronize()
            dist.barrier()
            if j > 0:
                times.append(dist.max(e0.elapsed_time(e1)))
            else:
                dist.max(0.0)
        e_ms = sum(times) / len(times)
        nbytes = 8 * sv.local_len * dist.world
        e2e = {"value": per / (e_ms * 1e-3), "unit": "gates/s", "h2d_bytes_per_step": nbytes,
               "d2h_bytes_per_step": nbytes, "ms_per_step": round(e_ms, 2), "steps": len(times),
               "what": "lyth_sv_set_local (pinned host -> HBM), lyth_sv_apply (one layer), lyth_sv_get_local "
                       "(qubit map undone, HBM -> pinned host)"}
        del hre, him
    sv.close()
    torch.cuda.empty_cache()

    streams = sharded_streams(dist, pk["hbm_gbs"]) if dist.world > 1 and not a.skip_streams else None

    cpu = None
    kernels = None
    if dist.rank == 0 and dist.world == 1:
        if not a.skip_kernels:
            kernels = per_kernel(pk)
        if not a.skip_cpu:
            cpu = cpu_sample(a.cpu_qubits)
    if dist.rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "gates/s", "n_gpus": dist.world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: SplitMix64-seeded normalised random complex64 state (split re/im f32); "
                    "layered circuit from circuits::Rng seed 20260930",
            "config": config_of(q, per, dist.world),
            "roofline": roofline,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"]},
            "engine": {"passes": st["passes"], "exchanges": st["exchanges"], "bytes_sent": st["bytes_sent"],
                       "settings": {"fusion": a.fuse or 13, "swap_batch": a.swap_batch or 6,
                                    "diagonal_rank_gates": "no exchange" if a.diagonal in (None, 1) else "exchange",
                                    "transport": sv_transport if dist.world > 1
                                    else None, "pull_queues": (a.pull_queues or "one per partner slice") if dist.world > 1
                                    else None}},
            "parity": parity,
        }
        if cpu:
            line["cpu_baseline"] = {"value": cpu["gates_per_s_at_33"], "unit": "gates/s", "cores": cpu["cores"],
                                    "kind": "port", "sample": cpu["sample"]}
        if kernels:
            line["per_kernel"] = kernels
        if streams:
            line["sharded_streams"] = streams
        print(json.dumps(line), flush=True)


def main():
    a = args_()
    if a.list_cases:
        import torch

        print("\n".join(kernel_cases(torch.device("cpu"), small=True)))
        return
    if a.case:
        run_case(a.case, a.case_reps)
        return
    dist = Dist()
    if a.impl == "reference":
        reference_arm(a, dist)
        return
    dist.init()
    try:
        ours(a, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
