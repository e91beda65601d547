"""The ADR-0016 surface is generated, not typed in: every kernel's contract macros (derived bytes,
flops and intensity per element) and its five entry points in include/lyth_b200.h are exactly
what lyth_b200.bindgen emits from the kernel's lowered body (the reference checks its checked-in
bindings against its generator the same way, crates/lyth/tests/binding.rs); the library exports
every generated symbol; the committed lyth-manifest/0.1 records equal the generator's."""
import json
import os

import pytest

from lyth_b200 import bindgen

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = open(os.path.join(ROOT, "include", "lyth_b200.h")).read()
LINES = {ln.strip() for ln in HEADER.splitlines()}


@pytest.mark.parametrize("name", sorted(bindgen.ADR16))
def test_header_block_is_the_generated_one(name):
    sec = bindgen.c_section(name)
    for k, v in sec["macros"].items():
        assert f"#define {k} {v}" in LINES, (name, k, v)
    for d in sec["decls"]:
        assert d in LINES, (name, d)


@pytest.mark.parametrize("name", sorted(bindgen.ADR16))
def test_generated_symbols_are_exported(name):
    import lyth_b200 as lb

    for d in bindgen.c_section(name)["decls"]:
        sym = d.split("(")[0].split()[-1].lstrip("*")
        assert hasattr(lb.lib, sym), sym


@pytest.mark.parametrize("name", sorted(bindgen.ADR16))
def test_committed_manifest_is_the_generated_one(name):
    with open(os.path.join(ROOT, "fixtures", "manifest", f"{name}.json")) as f:
        assert json.load(f) == json.loads(json.dumps(bindgen.manifest(name)))


def test_manifest_facts():
    m = bindgen.manifest("sum")
    part = next(p for p in m["params"] if p["name"] == "partial")
    assert part["sized_by_grid"] and part["written"] and part["shape"] == ["blocks"]
    assert m["launch"]["block_must_be_power_of_two"] and m["launch"]["grid"]["min_elements_per_thread"] == 8
    m = bindgen.manifest("cu_q")
    assert {s["base"] for s in m["splits"]} >= {"re", "hr0"} and any(s.get("depth") == 1 for s in m["splits"])
    re = next(p for p in m["params"] if p["name"] == "re")
    qr = next(p for p in m["params"] if p["name"] == "qr")
    assert re["read"] and not re["written"] and qr["written"]
    assert bindgen.manifest("saxpy")["contract"]["bytes_per_element"] == 12.0


def test_py_module_compiles():
    compile(bindgen.py_module(), "generated.py", "exec")
