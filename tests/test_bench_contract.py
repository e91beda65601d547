"""bench.py's reference arm on the host (no GPU): one JSON line with the contract's keys."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                          "--ref-qubits", "16"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "gates/s"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert "workload" in line["config"]


def test_bench_uses_the_handle_api_as_declared():
    # bench.py's GPU path cannot run here; at least every `sv.<name>` it uses must exist on the
    # StateVector handle, called when it is a method and read when it is a property.
    import ast
    import inspect

    from lyth_b200.statevector import StateVector

    tree = ast.parse(open(os.path.join(ROOT, "bench.py")).read())
    called = {n.func.attr for n in ast.walk(tree)
              if isinstance(n, ast.Call) and isinstance(n.func, ast.Attribute)
              and isinstance(n.func.value, ast.Name) and n.func.value.id == "sv"}
    used = {n.attr for n in ast.walk(tree)
            if isinstance(n, ast.Attribute) and isinstance(n.value, ast.Name) and n.value.id == "sv"}
    assert used, "bench.py drives a handle named sv"
    src = inspect.getsource(StateVector)
    for name in used:
        if not hasattr(StateVector, name):  # an attribute the constructor sets
            assert f"self.{name} =" in src or f"self.{name}, " in src, name
            assert name not in called, f"sv.{name} is data, called as a method"
            continue
        member = inspect.getattr_static(StateVector, name)
        if name in called:
            assert not isinstance(member, property), f"sv.{name} is a property, called as a method"
        elif isinstance(member, property):
            continue
