"""Circuits: the host side of lyth-circuit (crates/lyth-circuit/src/lib.rs), restated.

A circuit is a list of gates on 2^q amplitudes, split re/im, little-endian (bit q of an index
is qubit q). Matrices are f64 and enter a kernel rounded to f32 once (``f32s``, lib.rs:49-56).
``fuse`` is the reference's greedy in-order grouping (lib.rs:72-100); ``Rng`` its SplitMix64
(lib.rs:418-433); ``ghz``, ``qft`` and ``random`` its circuits (lib.rs:436-468). ``layered`` is
the benchmark circuit of this back end: H on every qubit, a controlled phase on each adjacent
pair, then SWAPs on consecutive pairs of a Fisher-Yates permutation.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

S = 1.0 / math.sqrt(2.0)  # FRAC_1_SQRT_2
H = ((S, 0.0), (S, 0.0), (S, 0.0), (-S, 0.0))
X = ((0.0, 0.0), (1.0, 0.0), (1.0, 0.0), (0.0, 0.0))
Z = ((1.0, 0.0), (0.0, 0.0), (0.0, 0.0), (-1.0, 0.0))


def phase(phi: float):
    return ((1.0, 0.0), (0.0, 0.0), (0.0, 0.0), (math.cos(phi), math.sin(phi)))


def zyz(theta: float, phi: float, lam: float):
    c, s = math.cos(theta / 2.0), math.sin(theta / 2.0)

    def e(x):
        return (math.cos(x), math.sin(x))

    def sc(k, z):
        return (k * z[0], k * z[1])

    return ((c, 0.0), sc(-s, e(lam)), sc(s, e(phi)), sc(c, e(phi + lam)))


def f32s(m) -> list[float]:
    """``ar ai br bi cr ci dr di`` as f32 (round-to-nearest-even from f64, as `as f32`)."""
    out = []
    for r, i in m:
        out.append(float(np.float32(r)))
        out.append(float(np.float32(i)))
    return out


@dataclass(frozen=True)
class U:
    q: int
    m: tuple

    def qubits(self):
        return [self.q]


@dataclass(frozen=True)
class CU:
    c: int
    t: int
    m: tuple

    def qubits(self):
        return [self.c, self.t]


@dataclass(frozen=True)
class Swap:
    a: int
    b: int

    def qubits(self):
        return [self.a, self.b]


@dataclass
class Group:
    qubits: list[int]
    gates: list = field(default_factory=list)

    def widths(self) -> list[int]:
        return [1 << q for q in self.qubits]


def fuse(gates, k: int) -> list[Group]:
    """Greedy in circuit order: a gate joins the open group while the union of qubits stays
    within k (at least 1); a group's qubits are sorted descending (lib.rs:72-100)."""
    out: list[Group] = []
    cur: Group | None = None
    for g in gates:
        if cur is not None:
            union = list(cur.qubits)
            for q in g.qubits():
                if q not in union:
                    union.append(q)
            if len(union) <= max(k, 1):
                cur.qubits = union
                cur.gates.append(g)
                continue
            out.append(cur)
        cur = Group(list(g.qubits()), [g])
    if cur is not None:
        out.append(cur)
    for grp in out:
        grp.qubits.sort(reverse=True)
    return out


def widths_ct(c: int, t: int) -> tuple[int, int]:
    """The inner width counts elements of the view that lost bit c (lib.rs:387-389)."""
    return 1 << c, (1 << t) if t < c else (1 << (t - 1))


class Rng:
    """SplitMix64 (lib.rs:418-433)."""

    MASK = (1 << 64) - 1

    def __init__(self, seed: int):
        self.state = seed & self.MASK

    def next_u64(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & self.MASK
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & self.MASK
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & self.MASK
        return z ^ (z >> 31)

    def angle(self) -> float:
        return (self.next_u64() >> 11) / float(1 << 53) * (2.0 * math.pi)

    def below(self, n: int) -> int:
        return self.next_u64() % n


def ghz(n: int):
    return [U(0, H)] + [CU(0, t, X) for t in range(1, n)]


def qft(n: int, rng: Rng):
    g = [U(q, zyz(rng.angle(), rng.angle(), rng.angle())) for q in range(n)]
    for j in reversed(range(n)):
        g.append(U(j, H))
        for k in reversed(range(j)):
            g.append(CU(k, j, phase(math.pi / float(1 << (j - k)))))
    g.extend(Swap(i, n - 1 - i) for i in range(n // 2))
    return g


def _fisher_yates(n: int, rng: Rng) -> list[int]:
    qs = list(range(n))
    for i in reversed(range(1, n)):
        j = rng.below(i + 1)
        qs[i], qs[j] = qs[j], qs[i]
    return qs


def random(n: int, depth: int, rng: Rng):
    g = []
    for _ in range(depth):
        g.extend(U(q, zyz(rng.angle(), rng.angle(), rng.angle())) for q in range(n))
        qs = _fisher_yates(n, rng)
        for p in range(0, n - 1, 2):
            c, t = (qs[p], qs[p + 1]) if rng.below(2) == 0 else (qs[p + 1], qs[p])
            g.append(CU(c, t, X if rng.below(2) == 0 else Z))
    return g


def layered(n: int, layers: int, rng: Rng):
    """The benchmark circuit: per layer, H on qubits 0..n-1 in order; CU(phase(theta)) on
    (i, i+1) for i = 0..n-2 with theta = rng.angle(); SWAP on consecutive pairs of a
    Fisher-Yates permutation. n + (n-1) + n//2 gates per layer."""
    g = []
    for _ in range(layers):
        g.extend(U(q, H) for q in range(n))
        g.extend(CU(i, i + 1, phase(rng.angle())) for i in range(n - 1))
        qs = _fisher_yates(n, rng)
        g.extend(Swap(qs[p], qs[p + 1]) for p in range(0, n - 1, 2))
    return g


BENCH_SEED = 20260930


def as_tuples(gates):
    """The gates as (kind, q0, q1, m8) tuples -- kind 0 = U on q0, 1 = CU(c = q0, t = q1),
    2 = SWAP(q0, q1) -- the form the host evaluator's ``run_gates`` takes."""
    out = []
    for g in gates:
        if isinstance(g, U):
            out.append((0, g.q, 0, f32s(g.m)))
        elif isinstance(g, CU):
            out.append((1, g.c, g.t, f32s(g.m)))
        else:
            out.append((2, g.a, g.b, [0.0] * 8))
    return out
