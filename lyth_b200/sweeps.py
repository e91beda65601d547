"""The reference's pre-registered sweeps, re-run on B200 (tools/grid_sweep.py, tools/split_sweep.py,
tools/cu_sweep.py, tools/fusion_sweep.py; protocols docs/prereg/ADR-0012, ADR-0028, ADR-0029,
ADR-0030), with this back end's kernels in place of the emitted PTX.

Method, as the reference fixes it: passes are interleaved (every point once per pass, the point's
figure is the median over passes), so a clock or thermal drift is noise shared by all points
rather than a fake result at one; `within` is the spread of one point's repetitions inside a
pass, `across` the spread of its pass medians. A difference smaller than `across` is not a
result. CUDA events on the current stream; L2 is flushed (a 256 MiB read) before every timed
launch unless the state is far larger than L2 anyway.

    python -m lyth_b200.sweeps [grid|split|cu|fusion|all] [--out FILE]

Each prediction is restated from its protocol and answered `holds` / `fails` on the numbers.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import statistics
import sys


def _timer(fn, reps, flush=None, stream=None):
    import torch

    ts = []
    for _ in range(reps):
        if flush is not None:
            flush()
            torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        e.synchronize()
        ts.append(s.elapsed_time(e))
    return ts


def _interleaved(points: dict, passes: int, reps: int, flush=None, stream=None) -> dict:
    for fn in points.values():  # warm-up
        for _ in range(2):
            fn()
    per = {k: [] for k in points}
    within = {k: [] for k in points}
    for _ in range(passes):
        for k, fn in points.items():
            ts = _timer(fn, reps, flush, stream)
            med = statistics.median(ts)
            per[k].append(med)
            within[k].append((max(ts) - min(ts)) / med if med else 0.0)
    out = {}
    for k in points:
        med = statistics.median(per[k])
        out[k] = {"ms": med, "within": round(max(within[k]), 4),
                  "across": round((max(per[k]) - min(per[k])) / med, 4) if med else 0.0}
    return out


def _flusher():
    import torch

    buf = torch.ones(64 << 20, device="cuda")
    sink = torch.empty(1, device="cuda")
    return lambda: torch.sum(buf, dim=0, keepdim=True, out=sink)


def grid_sweep(passes=5, reps=5) -> dict:
    """ADR-0012: does grid-stride buy anything against one element per thread? saxpy over 2^26
    through the ADR-0016 launch with an explicit grid, from one block per SM up to ceil(n/256)
    (every thread runs the loop once: the old shape). Prediction: the one-element-per-thread
    point is no faster than the best grid-stride point (within `across`)."""
    import torch

    import lyth_b200 as lb

    n = 1 << 26
    x = torch.rand(n, device="cuda")
    y = torch.rand(n, device="cuda")
    mod, fn = C.c_void_p(), C.c_void_p()
    lb.lib.lyth_saxpy_load.argtypes = [C.c_void_p, C.c_void_p]
    assert lb.lib.lyth_saxpy_load(C.byref(mod), C.byref(fn)) == 0
    lb.lib.lyth_saxpy_launch_with.argtypes = [C.c_void_p, C.c_uint, C.c_uint, C.c_float, C.c_uint64, C.c_uint64]
    grids = [148, 296, 592, 1184, 2368, 4736, 9472, 37888, (n + 255) // 256]
    pts = {g: (lambda g=g: lb.lib.lyth_saxpy_launch_with(fn, g, n, 2.5, x.data_ptr(), y.data_ptr())) for g in grids}
    r = _interleaved(pts, passes, reps, _flusher())
    res = {str(g): {**v, "GB_s": round(12.0 * n / (v["ms"] * 1e-3) / 1e9, 1)} for g, v in r.items()}
    one = r[grids[-1]]["ms"]
    best = min(v["ms"] for g, v in r.items() if g != grids[-1])
    noise = max(v["across"] for v in r.values())
    verdict = "holds" if one >= best * (1 - noise) else "fails"
    return {"sweep": "grid (ADR-0012)", "n": n, "points": res,
            "prediction": "one element per thread is no faster than the best grid-stride grid", "verdict": verdict,
            "one_element_per_thread_ms": one, "best_grid_stride_ms": best}


def split_sweep(passes=5, reps=5) -> dict:
    """ADR-0028: a 1-qubit gate (gate_q) over 2^27 amplitudes (1 GiB: 8x L2; the reference's 2^23
    fit its 16 GB card's DRAM but sit in B200's 126 MiB L2) at every split width w = 2^q.
    Predictions: P1 the payload is width-independent (16 B per amplitude, by construction); the
    time is width-independent within 5 % (B200: every width takes the vectorised path except
    q = 0, 1, which pair inside a 16-byte vector)."""
    import torch

    import lyth_b200 as lb
    from lyth_b200 import circuit as cc

    q_all = 27
    n = 1 << q_all
    re = torch.rand(n, device="cuda")
    im = torch.rand(n, device="cuda")
    m = cc.f32s(cc.zyz(0.3, 1.1, -0.7))
    pts = {q: (lambda q=q: lb.gate(1 << q, m, re, im)) for q in range(q_all)}
    r = _interleaved(pts, passes, reps, _flusher())
    res = {str(q): {**v, "GB_s": round(16.0 * n / (v["ms"] * 1e-3) / 1e9, 1)} for q, v in r.items()}
    times = [v["ms"] for v in r.values()]
    spread = (max(times) - min(times)) / statistics.median(times)
    return {"sweep": "split (ADR-0028)", "amplitudes": n, "points": res,
            "prediction": "time independent of the width within 5 %", "spread": round(spread, 4),
            "verdict": "holds" if spread <= 0.05 else "fails"}


def cu_sweep(passes=3, reps=5) -> dict:
    """ADR-0029: cu_q over 2^27 amplitudes at every ordered pair of qubits {0,1,2,3,4,8,16,26},
    against a 1-qubit gate_q at the target as the control. Prediction: cu_q (in place, it moves
    only the control = 1 half: 8 B per amplitude) takes at most 1.10x the control's time x 0.5."""
    import torch

    import lyth_b200 as lb
    from lyth_b200 import circuit as cc

    n = 1 << 27
    re = torch.rand(n, device="cuda")
    im = torch.rand(n, device="cuda")
    m = cc.f32s(cc.zyz(0.3, 1.1, -0.7))
    qs = [0, 1, 2, 3, 4, 8, 16, 26]
    pts = {}
    for c in qs:
        for t in qs:
            if c != t:
                wc, wt = cc.widths_ct(c, t)
                pts[(c, t)] = (lambda wc=wc, wt=wt: lb.cu(wc, wt, m, re, im))
    ctrl = {t: (lambda t=t: lb.gate(1 << t, m, re, im)) for t in qs}
    r = _interleaved(pts, passes, reps, _flusher())
    rc = _interleaved(ctrl, passes, reps, _flusher())
    res = {f"{c},{t}": {**v, "ratio_to_half_control": round(v["ms"] / (0.5 * rc[t]["ms"]), 4)} for (c, t), v in r.items()}
    worst = max(v["ratio_to_half_control"] for v in res.values())
    return {"sweep": "cu (ADR-0029)", "amplitudes": n, "points": res,
            "control_ms": {str(t): v["ms"] for t, v in rc.items()},
            "prediction": "an in-place cu_q costs at most 1.10x half a 1-qubit pass", "worst_ratio": worst,
            "verdict": "holds" if worst <= 1.10 else "fails"}


def fusion_sweep(passes=3, reps=3) -> dict:
    """ADR-0030 Q2/Q3 on B200, at 2^27 amplitudes (the reference's 2^23 is L2-resident here): Q2 --
    a group of g gates on a fixed qubit set costs about one pass whatever g (g = 1, 2, 5, 10, 20, 40
    on sets A = {7,6,5,4,3} and B = {4,3,2,1,0}); Q3 -- a 27-qubit random circuit (depth 10) runs
    faster fused, at every fusion width 2..13."""
    import torch

    import lyth_b200 as lb
    from lyth_b200 import circuit as cc

    q = 27
    re = torch.rand(1 << q, device="cuda")
    im = torch.rand(1 << q, device="cuda")
    sets = {"A": [7, 6, 5, 4, 3], "B": [4, 3, 2, 1, 0]}
    rng = cc.Rng(20260930)
    m = cc.zyz(0.6, 0.1, 0.2)
    q2 = {}
    for name, bits in sets.items():
        for g in (1, 2, 5, 10, 20, 40):
            gates = [cc.U(bits[i % len(bits)], m) for i in range(g)]
            sv = lb.StateVector(q, device=0)
            sv.set_local(re, im)
            pts = {g: (lambda sv=sv, gates=gates: sv.apply(gates))}
            r = _interleaved(pts, passes, reps, stream=torch.cuda.ExternalStream(sv.stream))
            q2[f"{name}:{g}"] = {**r[g], "passes": sv.stats()["passes"] // (2 + passes * reps)}
            sv.close()
    circ = cc.random(q, 10, rng)
    q3 = {}
    for k in (1, 2, 3, 4, 5, 6, 8, 10, 13):
        sv = lb.StateVector(q, device=0)
        sv.set_fusion(k)
        sv.set_local(re, im)
        r = _interleaved({k: (lambda sv=sv: sv.apply(circ))}, passes, reps, stream=torch.cuda.ExternalStream(sv.stream))
        p0 = sv.stats()["passes"]
        q3[str(k)] = {**r[k], "passes_per_run": p0 // (2 + passes * reps)}
        sv.close()
    base = q2["A:1"]["ms"]
    worst_q2 = max(v["ms"] / base for v in q2.values())
    unf = q3["1"]["ms"]
    return {"sweep": "fusion (ADR-0030)", "qubits": q, "Q2": q2, "Q3": q3,
            "Q2_prediction": "a fused group costs about one pass: at most 1.5x one gate's pass up to 40 gates",
            "Q2_worst_ratio": round(worst_q2, 3), "Q2_verdict": "holds" if worst_q2 <= 1.5 else "fails",
            "Q3_prediction": "fused faster than unfused at every width >= 2",
            "Q3_speedups": {k: round(unf / v["ms"], 3) for k, v in q3.items()},
            "Q3_verdict": "holds" if all(unf / v["ms"] > 1.0 for k, v in q3.items() if k != "1") else "fails"}


SWEEPS = {"grid": grid_sweep, "split": split_sweep, "cu": cu_sweep, "fusion": fusion_sweep}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m lyth_b200.sweeps")
    ap.add_argument("which", choices=list(SWEEPS) + ["all"])
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    import torch

    torch.cuda.set_device(0)
    out = {}
    for name in (SWEEPS if a.which == "all" else [a.which]):
        out[name] = SWEEPS[name]()
        print(json.dumps({name: {k: v for k, v in out[name].items() if k not in ("points", "Q2", "Q3")}}), flush=True)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(out, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
