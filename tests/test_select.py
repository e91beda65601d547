"""The back-end entry on the host (no GPU): every in-scope example's lowered body maps to its
kernel class; kernels this back end does not compute, or that lyth-ptx refuses
(crates/lyth-ptx/src/lib.rs:48-180: NoBound, NoDrain, UnknownTarget, reg -> dram reductions,
coarsened non-contractions), are refused with the reason, never run another way."""
import pytest

import lyth_b200 as lb
from lyth_b200 import ir
from lyth_b200 import examples as ex


@pytest.mark.parametrize("name", sorted(ex.IN_SCOPE))
def test_every_in_scope_example_selects_its_class(name):
    sel = ex.IN_SCOPE[name]().select()
    assert sel.entry == name
    assert sel.retargeted  # the examples say `machine sm_120`: accepted and recorded
    assert "retarget" in sel.note


def test_own_machine_is_not_a_retarget():
    k = ex.saxpy()
    k.machine = "sm_100a"
    sel = k.select()
    assert sel.entry == "saxpy" and not sel.retargeted


def refused(k, status=lb.E_UNSUPPORTED):
    with pytest.raises(lb.LythError) as e:
        k.select()
    assert e.value.status == status
    return str(e.value)


def test_a_different_rounding_is_a_different_kernel():
    # y = a * x + y with the product rounded first (mul then add): not saxpy's fma, refused
    k = ir.Kernel("saxpy_unfused", [("n", "u32"), ("a", "f32"), ("x", "f32[]"), ("y", "f32[]")])
    k.drain("y", k.add(k.mul(k.param("a"), k.load("x")), k.load("y")))
    assert "no kernel for" in refused(k)


def test_out_of_scope_bodies_are_refused():
    # examples/complex-mul.lyth's kind of body: no kernel class computes it
    k = ir.Kernel("cmul", [("n", "u32"), ("ar", "f32[]"), ("ai", "f32[]"), ("br", "f32[]"), ("bi", "f32[]"),
                           ("cr", "f32[]")])
    k.drain("cr", k.sub(k.mul(k.load("ar"), k.load("br")), k.mul(k.load("ai"), k.load("bi"))))
    assert "no kernel for" in refused(k)
    # mixed narrow storage (an f16 input, a bf16 output) is no class of this library
    k = ir.Kernel("saxpy_mixed", [("n", "u32"), ("a", "f32"), ("x", "f16[]"), ("y", "bf16[]")])
    k.drain("y", k.fma(k.param("a"), k.load("x"), k.load("y")))
    refused(k)
    # a narrow state-vector gate is not either (the gate kernels are f32)
    k = ex.gate_q()
    k.params = [(n, 3 if t == 2 else t) for n, t in k.params]
    refused(k)


@pytest.mark.parametrize("name", ["saxpy", "axpby", "lerp", "horner", "copy2d", "transpose_tiled", "sum", "dot",
                                  "max_of", "min_of"])
@pytest.mark.parametrize("ty", ["f16[]", "bf16[]"])
def test_narrow_storage_selects_the_class(name, ty):
    # ADR-0024: every data buffer f16 (or every one bf16), f32 arithmetic; partials stay f32
    k = ex.IN_SCOPE[name]()
    into = k.reduction[2] if k.reduction else None
    k.params = [(n, ir.TY[ty] if t == ir.TY["f32[]"] and n != into else t) for n, t in k.params]
    sel = k.select()
    assert sel.entry == name + ("_f16" if ty == "f16[]" else "_bf16")
    assert sel.storage == (1 if ty == "f16[]" else 2)


def test_lyth_ptx_refusals():
    k = ex.saxpy()
    k.machine = "sm_90"
    assert "machine `sm_90`" in refused(k)                      # UnknownTarget
    k = ir.Kernel("nobound", [("a", "f32"), ("x", "f32[]"), ("y", "f32[]")])
    k.drain("y", k.fma(k.param("a"), k.load("x"), k.load("y")))
    assert "bounds the index space" in refused(k)               # NoBound
    k = ir.Kernel("nodrain", [("n", "u32"), ("x", "f32[]")])
    k.load("x")
    assert "drains nothing" in refused(k)                       # NoDrain
    k = ex.reduction("sum")
    k.reduction = (0, k.reduction[1], "partial", False)
    assert "reg -> dram" in refused(k)                          # reduction not staged
    k = ex.transpose(True)
    k.coarsen = (2, 2)
    assert "coarsens a tile that does not contract" in refused(k)


def test_malformed_descriptors_are_invalid():
    k = ir.Kernel("bad", [("n", "u32"), ("x", "f32[]"), ("y", "f32[]")])
    k.drain("y", k.load("nowhere"))
    refused(k, lb.E_INVALID)
    k = ir.Kernel("bad2", [("n", "u32"), ("x", "f32[]"), ("y", "f32[]")])
    k.drain("y", 7)
    refused(k, lb.E_INVALID)


def test_workspace_query_is_zero_for_every_class():
    for name, make in ex.IN_SCOPE.items():
        sel = make().select()
        args = [0] * len(sel.types)
        assert sel.workspace_bytes(args) == 0, name
