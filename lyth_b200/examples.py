"""The in-scope examples of the reference, as lowered-kernel descriptors (lyth_b200.ir.Kernel):
each body is what lyth-lang's lowering makes of the example's `at reg:` lines, fma formed
exactly where ir.rs:2388-2429 forms one (a * b + c -> fma(a, b, c); lhs + t * d -> fma(t, d,
lhs); a product of a negated parameter -> neg then mul), the file cited per kernel."""
from .ir import Kernel

U, F, B, H = "u32", "f32", "f32[]", "bf16[]"


def saxpy():  # examples/saxpy.lyth: y = a * x + y
    k = Kernel("saxpy", [("n", U), ("a", F), ("x", B), ("y", B)])
    k.drain("y", k.fma(k.param("a"), k.load("x"), k.load("y")))
    return k


def axpby():  # examples/axpby.lyth: y = a * x + b * y
    k = Kernel("axpby", [("n", U), ("a", F), ("b", F), ("x", B), ("y", B)])
    a, x, b, y = k.param("a"), k.load("x"), k.param("b"), k.load("y")
    k.drain("y", k.fma(a, x, k.mul(b, y)))
    return k


def lerp():  # examples/lerp.lyth: z = x + t * (y - x)
    k = Kernel("lerp", [("n", U), ("t", F), ("x", B), ("y", B), ("z", B)])
    x, t, y = k.load("x"), k.param("t"), k.load("y")
    k.drain("z", k.fma(t, k.sub(y, x), x))
    return k


def horner():  # examples/horner.lyth: y = ((c3 * x + c2) * x + c1) * x + c0
    k = Kernel("horner", [("n", U), ("c0", F), ("c1", F), ("c2", F), ("c3", F), ("x", B), ("y", B)])
    x = k.load("x")
    v = k.fma(k.param("c3"), x, k.param("c2"))
    v = k.fma(v, x, k.param("c1"))
    k.drain("y", k.fma(v, x, k.param("c0")))
    return k


def copy2d():  # examples/copy2d.lyth: b[i, j] = a[i, j]
    k = Kernel("copy2d", [("rows", U), ("cols", U), ("a", B), ("b", B)], rank=2)
    k.drain("b", k.load("a"))
    return k


def transpose(tiled=False):  # examples/transpose.lyth, transpose-tiled.lyth: b[j, i] = a[i, j]
    k = Kernel("transpose_tiled" if tiled else "transpose", [("rows", U), ("cols", U), ("a", B), ("b", B)], rank=2,
               tile=(32, 32) if tiled else (0, 0))
    k.drain("b", k.load("a"), transposed=True)
    return k


def reduction(which):  # examples/{sum,dot,max,min}.lyth
    if which == "dot":
        k = Kernel("dot", [("n", U), ("x", B), ("y", B), ("partial", B)])
        k.reduce("sum", k.mul(k.load("x"), k.load("y")), "partial")
        return k
    k = Kernel({"sum": "sum", "max": "max_of", "min": "min_of"}[which], [("n", U), ("x", B), ("partial", B)])
    k.reduce(which, k.load("x"), "partial")
    return k


def matmul(bf16=False):  # examples/matmul.lyth: c[i, j] = a[i, p] * b[p, j], contract sum p : k
    t = H if bf16 else B
    k = Kernel("matmul", [("m", U), ("n", U), ("k", U), ("a", t), ("b", t), ("c", B)], rank=2, tile=(32, 32),
               contract=True)
    k.drain("c", k.mul(k.load("a"), k.load("b")))
    return k


def _splits(k, names, widths):
    for base, parts, w in zip(names, widths[0], widths[1]):
        k.split(base, parts, w)


def hadamard_q():  # examples/hadamard_q.lyth
    k = Kernel("hadamard_q", [("n", U), ("w", U), ("s", F), ("re", B), ("im", B), ("qr", B), ("qi", B)])
    for base, a, b in (("re", "p0r", "p1r"), ("im", "p0i", "p1i"), ("qr", "q0r", "q1r"), ("qi", "q0i", "q1i")):
        k.split(base, (a, b), "w")
    s = k.param("s")
    for out, op, a, b in (("q0r", "add", "p0r", "p1r"), ("q0i", "add", "p0i", "p1i"),
                          ("q1r", "sub", "p0r", "p1r"), ("q1i", "sub", "p0i", "p1i")):
        k.drain(out, k.mul(s, k.bin(op, k.load(a), k.load(b))))
    return k


def _chain(k, c0, v0, c1, v1, c2, v2, c3, v3, neg1, neg3):
    """fma(c0, v0, fma(+-c1, v1, fma(c2, v2, mul(+-c3, v3)))) (examples/gate_q.lyth:38-42)."""
    p = lambda n: k.param(n)
    inner = k.mul(k.neg(p(c3)) if neg3 else p(c3), k.load(v3))
    mid = k.fma(p(c2), k.load(v2), inner)
    out = k.fma(k.neg(p(c1)) if neg1 else p(c1), k.load(v1), mid)
    return k.fma(p(c0), k.load(v0), out)


M8 = [("ar", F), ("ai", F), ("br", F), ("bi", F), ("cr", F), ("ci", F), ("dr", F), ("di", F)]


def gate_q():  # examples/gate_q.lyth
    k = Kernel("gate_q", [("n", U), ("w", U)] + M8 + [("re", B), ("im", B), ("qr", B), ("qi", B)])
    for base, a, b in (("re", "p0r", "p1r"), ("im", "p0i", "p1i"), ("qr", "q0r", "q1r"), ("qi", "q0i", "q1i")):
        k.split(base, (a, b), "w")
    k.drain("q0r", _chain(k, "ar", "p0r", "ai", "p0i", "br", "p1r", "bi", "p1i", True, True))
    k.drain("q0i", _chain(k, "ar", "p0i", "ai", "p0r", "br", "p1i", "bi", "p1r", False, False))
    k.drain("q1r", _chain(k, "cr", "p0r", "ci", "p0i", "dr", "p1r", "di", "p1i", True, True))
    k.drain("q1i", _chain(k, "cr", "p0i", "ci", "p0r", "dr", "p1i", "di", "p1r", False, False))
    return k


def _quad_splits(k):
    for base, h, (a, b), (c, d) in (("re", ("hr0", "hr1"), ("pr00", "pr01"), ("pr10", "pr11")),
                                    ("im", ("hi0", "hi1"), ("pi00", "pi01"), ("pi10", "pi11")),
                                    ("qr", ("gr0", "gr1"), ("qr_00", "qr_01"), ("qr_10", "qr_11")),
                                    ("qi", ("gi0", "gi1"), ("qi_00", "qi_01"), ("qi_10", "qi_11"))):
        k.split(base, h, "wc")
        k.split(h[0], (a, b), "wt")
        k.split(h[1], (c, d), "wt")


def cu_q():  # examples/cu_q.lyth
    k = Kernel("cu_q", [("n", U), ("wc", U), ("wt", U)] + M8 + [("re", B), ("im", B), ("qr", B), ("qi", B)])
    _quad_splits(k)
    k.drain("qr_10", _chain(k, "ar", "pr10", "ai", "pi10", "br", "pr11", "bi", "pi11", True, True))
    k.drain("qi_10", _chain(k, "ar", "pi10", "ai", "pr10", "br", "pi11", "bi", "pr11", False, False))
    k.drain("qr_11", _chain(k, "cr", "pr10", "ci", "pi10", "dr", "pr11", "di", "pi11", True, True))
    k.drain("qi_11", _chain(k, "cr", "pi10", "ci", "pr10", "dr", "pi11", "di", "pr11", False, False))
    for out, src in (("qr_00", "pr00"), ("qi_00", "pi00"), ("qr_01", "pr01"), ("qi_01", "pi01")):
        k.drain(out, k.load(src))
    return k


def swap_q():  # examples/swap_q.lyth
    k = Kernel("swap_q", [("n", U), ("wc", U), ("wt", U), ("re", B), ("im", B), ("qr", B), ("qi", B)])
    _quad_splits(k)
    for out, src in (("qr_00", "pr00"), ("qi_00", "pi00"), ("qr_01", "pr10"), ("qi_01", "pi10"),
                     ("qr_10", "pr01"), ("qi_10", "pi01"), ("qr_11", "pr11"), ("qi_11", "pi11")):
        k.drain(out, k.load(src))
    return k


IN_SCOPE = {
    "saxpy": saxpy, "axpby": axpby, "lerp": lerp, "horner": horner, "copy2d": copy2d,
    "transpose": lambda: transpose(False), "transpose_tiled": lambda: transpose(True),
    "sum": lambda: reduction("sum"), "dot": lambda: reduction("dot"), "max_of": lambda: reduction("max"),
    "min_of": lambda: reduction("min"), "matmul": lambda: matmul(False), "matmul_bf16": lambda: matmul(True),
    "hadamard_q": hadamard_q, "gate_q": gate_q, "cu_q": cu_q, "swap_q": swap_q,
}
