"""The sharded state vector (lyth_sv_* in include/lyth_b200.h), from Python.

Mirrors lyth-circuit's ``execute`` (crates/lyth-circuit/src/lib.rs:327-371) one rank at a time:
a handle owns this rank's shard of 2^qubits complex64 amplitudes (split re/im), applies a gate
list in order on its own stream, and reads the shard back in logical qubit order.
"""
from __future__ import annotations

import ctypes as C

from . import GATE_CU, GATE_SWAP, GATE_U, Gate, SvOp, check, lib
from .circuit import CU, Swap, U, f32s


def unique_id() -> bytes:
    """An NCCL unique id for a multi-rank state vector (call on one rank, share with all)."""
    buf = C.create_string_buffer(128)
    check(lib.lyth_sv_unique_id(buf), "lyth_sv_unique_id")
    return buf.raw


def gates_array(gates) -> "C.Array[Gate]":
    """lyth-circuit Gate values -> a ``lyth_gate`` array (matrices rounded to f32 once, f32s)."""
    arr = (Gate * max(len(gates), 1))()
    for i, g in enumerate(gates):
        if isinstance(g, U):
            arr[i].kind, arr[i].q0, arr[i].q1 = GATE_U, g.q, 0
            arr[i].m[:] = f32s(g.m)
        elif isinstance(g, CU):
            arr[i].kind, arr[i].q0, arr[i].q1 = GATE_CU, g.c, g.t
            arr[i].m[:] = f32s(g.m)
        elif isinstance(g, Swap):
            arr[i].kind, arr[i].q0, arr[i].q1 = GATE_SWAP, g.a, g.b
        else:
            raise TypeError(f"not a gate: {g!r}")
    return arr


# lyth_sv_set_transport's kinds, by index
TRANSPORTS = ("nccl", "copy_engine", "peer_load", "mixed", "peer_store")


class StateVector:
    """One rank's shard. ``nranks`` must be a power of two; ``nccl_id`` is required when > 1."""

    def __init__(self, qubits: int, device: int = 0, rank: int = 0, nranks: int = 1, nccl_id: bytes | None = None):
        h = C.c_void_p()
        check(lib.lyth_sv_create(C.byref(h), qubits, device, rank, nranks, nccl_id), "lyth_sv_create")
        self._h = h
        self.qubits, self.device, self.rank, self.nranks = qubits, device, rank, nranks
        self.local_len = int(lib.lyth_sv_local_len(h))

    def close(self) -> None:
        if self._h:
            check(lib.lyth_sv_destroy(self._h), "lyth_sv_destroy")
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        """The cudaStream_t every operation of this handle is ordered on."""
        return int(lib.lyth_sv_stream(self._h) or 0)

    def init_basis(self, index: int = 0) -> None:
        check(lib.lyth_sv_init_basis(self._h, index), "init_basis")

    def init_random(self, seed: int) -> None:
        check(lib.lyth_sv_init_random(self._h, seed), "init_random")

    def set_local(self, re, im) -> None:
        """re/im: this rank's shard, as torch tensors (CPU or CUDA) or raw pointers."""
        check(lib.lyth_sv_set_local(self._h, _addr(re), _addr(im)), "set_local")

    def get_local(self, re, im) -> None:
        check(lib.lyth_sv_get_local(self._h, _addr(re), _addr(im)), "get_local")

    def apply(self, gates) -> None:
        arr = gates if isinstance(gates, C.Array) else gates_array(gates)
        count = len(gates)
        check(lib.lyth_sv_apply(self._h, arr, count), "apply")

    def sync(self) -> None:
        check(lib.lyth_sv_sync(self._h), "sync")

    def stats(self) -> dict:
        p, e, b = C.c_uint64(), C.c_uint64(), C.c_uint64()
        check(lib.lyth_sv_stats(self._h, C.byref(p), C.byref(e), C.byref(b)), "stats")
        return {"passes": p.value, "exchanges": e.value, "bytes_sent": b.value,
                "launches": int(lib.lyth_sv_launches(self._h))}

    def set_timing(self, on: bool) -> None:
        check(lib.lyth_sv_set_timing(self._h, int(on)), "set_timing")

    def set_fusion(self, max_qubits: int) -> None:
        """Fuse consecutive local gates touching at most max_qubits (1..13) bits; 1 = unfused.
        A group must also fit one pass: at most 8 bits above bit 4 (the tile pass, shards of 2^14
        amplitudes and more), at most 6 bits (the register pass, smaller shards)."""
        check(lib.lyth_sv_set_fusion(self._h, max_qubits), "set_fusion")

    def set_deadline(self, ms: float) -> None:
        """Host deadline of the handle's NCCL waits (ms): past it, or on an NCCL async error, the
        communicator is aborted and sync returns an error instead of hanging."""
        check(lib.lyth_sv_set_deadline(self._h, float(ms)), "set_deadline")

    def set_remap(self, on: bool) -> None:
        """Rank-bit gates: swap the qubit into a local bit first (True, default) or exchange the
        whole shard and compute this rank's row (False)."""
        check(lib.lyth_sv_set_remap(self._h, int(on)), "set_remap")

    def set_diagonal(self, on: bool) -> None:
        """Diagonal gates on rank-bit targets: no exchange, each shard applies its row's scalar
        (True, default; equal in value, the sign of an exactly-zero amplitude may differ) or like
        any other gate (False; bit-identical in every case). Collective."""
        check(lib.lyth_sv_set_diagonal(self._h, int(on)), "set_diagonal")

    def set_swap_batch(self, max_qubits: int) -> None:
        """Most rank-bit qubits one swap-in brings in together (default 6; 1 = one at a time).
        Collective: every rank sets the same value at the same point."""
        check(lib.lyth_sv_set_swap_batch(self._h, max_qubits), "set_swap_batch")

    TRANSPORTS = TRANSPORTS

    def set_transport(self, kind) -> None:
        """Swap-in transport: "copy_engine" (copy engines over CUDA IPC), "peer_load" (the same
        mappings, the SMs load the partners' packed chunks straight into the shard), "mixed" (copy
        engines for pairwise swap-ins, peer loads for batched ones; the default when every rank
        mapped every peer), "peer_store" (the SMs store this rank's packed chunks straight into
        the partners' shards) or "nccl". True / False mean "copy_engine" / "nccl".
        Collective: every rank sets the same value at the same point."""
        if isinstance(kind, bool):
            kind = "copy_engine" if kind else "nccl"
        if kind not in TRANSPORTS:
            raise ValueError(f"transport {kind!r}: one of {TRANSPORTS}")
        check(lib.lyth_sv_set_transport(self._h, TRANSPORTS.index(kind)), "set_transport")

    def set_chunk(self, elements: int) -> None:
        """Exchange pipeline chunk, amplitudes per component (power of two >= 1024). Collective."""
        check(lib.lyth_sv_set_chunk(self._h, elements), "set_chunk")

    @property
    def transport(self) -> str:
        return TRANSPORTS[lib.lyth_sv_transport(self._h)]

    def timing(self) -> dict:
        """{class: (count, total ms)}: 'u' (1-qubit passes), 'cu' (2-qubit), 'exchange',
        'fused' (fused multi-gate passes), 'swap' (rank-bit qubits swapped into local bits)."""
        out = {}
        for cls, name in enumerate(("u", "cu", "exchange", "fused", "swap")):
            n, ms = C.c_uint64(), C.c_double()
            check(lib.lyth_sv_timing(self._h, cls, C.byref(n), C.byref(ms)), "timing")
            out[name] = (n.value, ms.value)
        return out

    def reset_timing(self) -> None:
        check(lib.lyth_sv_reset_timing(self._h), "reset_timing")


_OP_NAMES = ("u", "cu", "fused", "exchange", "swap_local", "swap_lr", "swap_rr", "swap_multi", "permute")


class Plan:
    """A plan handle (lyth_sv_plan_create): the engine's planner for ``rank`` of ``nranks``, with
    no device memory. ``apply`` and ``finish`` (the read-out's permutation steps) append the
    steps the engine would run; ``ops`` returns them as dicts:

    * ``u``: U on local bit ``a``, matrix ``m``; ``cu``: control ``a``, target ``b``;
    * ``fused``: ``gates`` = [(target bit, control bit or -1, m), ...] in order;
    * ``exchange``: the gate ``m`` on rank bit ``a`` (control local bit ``c`` or -1), with the
      partner rank ^ (1 << a); this rank keeps its row;
    * ``swap_local`` (bits a, b), ``swap_lr`` (local bit a, rank bit b), ``swap_rr`` (rank bits);
    * ``swap_multi``: local bits ``bits[j]`` with rank bits ``rbits[j]`` in one exchange among the
      2^k ranks that differ only in those rank bits;
    * ``permute``: one local pass moving bit ``bits[j]`` to bit ``rbits[j]`` (the read-out).
    """

    def __init__(self, qubits: int, rank: int = 0, nranks: int = 1):
        h = C.c_void_p()
        check(lib.lyth_sv_plan_create(C.byref(h), qubits, rank, nranks), "lyth_sv_plan_create")
        self._h = h
        self.qubits, self.rank, self.nranks = qubits, rank, nranks
        self.local_len = int(lib.lyth_sv_local_len(h))

    def close(self) -> None:
        if self._h:
            check(lib.lyth_sv_destroy(self._h), "lyth_sv_destroy")
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_fusion(self, max_qubits: int) -> None:
        check(lib.lyth_sv_set_fusion(self._h, max_qubits), "set_fusion")

    def set_remap(self, on: bool) -> None:
        check(lib.lyth_sv_set_remap(self._h, int(on)), "set_remap")

    def set_diagonal(self, on: bool) -> None:
        check(lib.lyth_sv_set_diagonal(self._h, int(on)), "set_diagonal")

    def set_swap_batch(self, max_qubits: int) -> None:
        check(lib.lyth_sv_set_swap_batch(self._h, max_qubits), "set_swap_batch")

    def apply(self, gates) -> None:
        arr = gates if isinstance(gates, C.Array) else gates_array(gates)
        check(lib.lyth_sv_apply(self._h, arr, len(gates)), "apply")

    def finish(self) -> None:
        """Record the steps that undo the qubit map (what lyth_sv_get_local runs first)."""
        check(lib.lyth_sv_get_local(self._h, None, None), "get_local")

    def clear(self) -> None:
        check(lib.lyth_sv_plan_clear(self._h), "plan_clear")

    def stats(self) -> dict:
        p, e, b = C.c_uint64(), C.c_uint64(), C.c_uint64()
        check(lib.lyth_sv_stats(self._h, C.byref(p), C.byref(e), C.byref(b)), "stats")
        return {"passes": p.value, "exchanges": e.value, "bytes_sent": b.value}

    def ops(self) -> list[dict]:
        out = []
        op = SvOp()
        for i in range(int(lib.lyth_sv_plan_count(self._h))):
            check(lib.lyth_sv_plan_op(self._h, i, C.byref(op)), "plan_op")
            d = {"kind": _OP_NAMES[op.kind], "a": op.a, "b": op.b, "c": op.c, "m": tuple(op.m)}
            if op.kind in (7, 8):
                d["bits"], d["rbits"] = list(op.bits[: op.k]), list(op.rbits[: op.k])
            if op.kind == 2:
                bits = list(op.bits[: op.k])
                d["gates"] = [(bits[op.gt[j]], bits[op.gc[j]] if op.gc[j] >= 0 else -1, tuple(op.gm[j]))
                              for j in range(op.ngates)]
            out.append(d)
        return out


def _addr(t) -> int:
    if isinstance(t, int):
        return t
    try:
        import numpy as np

        if isinstance(t, np.ndarray):
            if t.dtype != np.float32 or not t.flags["C_CONTIGUOUS"]:
                raise TypeError("expected a contiguous float32 array")
            return t.ctypes.data
    except ImportError:
        pass
    if not t.is_contiguous():
        raise ValueError("buffer must be contiguous")
    return t.data_ptr()
