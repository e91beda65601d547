"""Host-side tests without a GPU: the C-ABI library loads and exports every symbol the header
declares, the launch arithmetic of the ADR-0016 surface (manifest.rs figures), refusals that
happen before any device work, and the circuit host logic (fuse, generators)."""
import ctypes as C
import os
import re

import pytest

import lyth_b200 as lb
from lyth_b200 import circuit as cc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "lyth_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = set(re.findall(r"\b(lyth_\w+)\s*\(", text))
    inline = set(re.findall(r"static inline [\w\s\*]+?\b(lyth_\w+)\s*\(", text))
    return sorted(names - inline)


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) > 100
    missing = [n for n in names if not hasattr(lb.lib, n)]
    assert not missing, f"declared in include/lyth_b200.h but not exported: {missing}"


def test_every_adr16_kernel_has_the_full_family():
    kernels = ["saxpy", "axpby", "lerp", "horner", "copy2d", "transpose", "transpose_tiled", "sum", "dot",
               "max_of", "min_of", "matmul", "hadamard_q", "gate_q", "cu_q", "swap_q"]
    for k in kernels:
        for suffix in ["elements", "grid", "load", "launch", "launch_with"]:
            assert hasattr(lb.lib, f"lyth_{k}_{suffix}"), f"lyth_{k}_{suffix}"


def test_manifest_launch_figures():
    # manifest.rs:617-857: one element per thread -> 262144 blocks at 2^26; a reduction walks 8
    # per thread -> 32768; a tile gets one block.
    assert lb.lib.lyth_saxpy_grid(1 << 26) == 262144
    assert lb.lib.lyth_sum_grid(1 << 26) == 32768
    assert lb.lib.lyth_sum_partial_len(1 << 26) == 32768
    assert lb.lib.lyth_saxpy_grid(0) == 0
    assert lb.lib.lyth_saxpy_grid(1 << 31) == 1 << 20  # capped at MAX_GRID
    assert lb.lib.lyth_transpose_tiled_grid(4096, 4096) == 64 * 64
    assert lb.lib.lyth_transpose_tiled_grid(4097, 33) == 65 * 1
    assert lb.lib.lyth_copy2d_elements(1 << 16, 1 << 16) == 0  # overflows a 32-bit index
    assert lb.lib.lyth_gate_q_grid(1 << 22) == (1 << 21) // 256
    assert lb.lib.lyth_cu_q_grid(1 << 22) == (1 << 20) // 256
    assert lb.reduce_grid(1 << 26) == 32768 and lb.reduce_grid(1) == 1


def test_split_checks_refuse_before_any_device_work():
    assert lb.lib.lyth_gate_q_check_splits(12, 0) == lb.E_SPLIT
    assert lb.lib.lyth_gate_q_check_splits(12, 4) == lb.E_SPLIT
    assert lb.lib.lyth_gate_q_check_splits(96, 3) == lb.OK
    assert lb.lib.lyth_cu_q_check_splits(64, 4, 2) == lb.OK
    assert lb.lib.lyth_cu_q_check_splits(64, 16, 32) == lb.E_SPLIT
    m = (C.c_float * 8)()
    assert lb.lib.lyth_b200_gate(12, 4, m, 1, 1, 1, 1, None) == lb.E_SPLIT
    assert lb.lib.lyth_b200_cu(64, 16, 32, m, 1, 1, 1, 1, None) == lb.E_SPLIT
    with pytest.raises(lb.LythError) as e:
        lb.check(lb.E_SPLIT, "gate_q")
    assert "2*width" in str(e.value)


def test_error_strings_cover_every_code():
    for code in range(-7, 1):
        assert lb.lib.lyth_b200_error_string(code)
    assert b"unknown" in lb.lib.lyth_b200_error_string(-99)


def test_gemv_shape_refusals_are_host_side():
    assert lb.lib.lyth_b200_gemv_q4(0, 8, 100, 64, 16, 16, 16, 16, None) == lb.E_UNSUPPORTED
    assert lb.lib.lyth_b200_gemv_q4(0, 8, 4096, 48, 16, 16, 16, 16, None) == lb.E_UNSUPPORTED
    assert lb.lib.lyth_b200_gemv_q4(7, 8, 4096, 64, 16, 16, 16, 16, None) == lb.E_UNSUPPORTED


def test_nf4_codebook_matches_the_oracle():
    from oracle import oracle as orc

    assert lb.nf4_codebook() == orc.nf4_codebook().tolist()


# ------------------------------------------------------------------ lyth-circuit host logic
def suite():
    rng = cc.Rng(20_260_930)
    return [
        ("GHZ(12)", 12, cc.ghz(12)),
        ("QFT(10)", 10, cc.qft(10, rng)),
        ("random(10, depth 20)", 10, cc.random(10, 20, rng)),
        ("random(20, depth 10)", 20, cc.random(20, 10, cc.Rng(20_260_931))),
    ]


def test_fuser_keeps_every_gate_in_order_and_respects_k():
    for name, _, gates in suite():
        for k in range(1, 6):
            groups = cc.fuse(gates, k)
            flat = [g for grp in groups for g in grp.gates]
            assert flat == gates, name
            for grp in groups:
                need = max(len(g.qubits()) for g in grp.gates)
                assert len(grp.qubits) <= max(k, need)
                assert all(a > b for a, b in zip(grp.qubits, grp.qubits[1:]))


def test_layered_circuit_gate_counts():
    for q, per in [(30, 74), (33, 81)]:
        g = cc.layered(q, 20, cc.Rng(cc.BENCH_SEED))
        assert len(g) == 20 * per
        assert sum(isinstance(x, cc.Swap) for x in g) == 20 * (q // 2)


def test_f32s_rounds_once():
    m = cc.f32s(cc.H)
    assert m[0] == float(__import__("numpy").float32(1 / 2 ** 0.5))
    assert m[6] == -m[0] and m[1] == 0.0


def test_gate_array_packs_kind_and_qubits():
    from lyth_b200.statevector import gates_array

    arr = gates_array([cc.U(3, cc.H), cc.CU(1, 2, cc.X), cc.Swap(0, 5)])
    assert (arr[0].kind, arr[0].q0) == (lb.GATE_U, 3)
    assert (arr[1].kind, arr[1].q0, arr[1].q1) == (lb.GATE_CU, 1, 2)
    assert (arr[2].kind, arr[2].q0, arr[2].q1) == (lb.GATE_SWAP, 0, 5)
    assert list(arr[1].m) == cc.f32s(cc.X)


def test_sv_create_refuses_bad_arguments_without_a_device():
    h = C.c_void_p()
    assert lb.lib.lyth_sv_create(C.byref(h), 10, 0, 0, 3, None) == lb.E_INVALID  # not a power of 2
    assert lb.lib.lyth_sv_create(C.byref(h), 10, 0, 2, 2, None) == lb.E_INVALID  # rank out of range
    assert lb.lib.lyth_sv_create(C.byref(h), 10, 0, 0, 2, None) == lb.E_INVALID  # no id
    assert lb.lib.lyth_sv_create(C.byref(h), 2, 0, 0, 4, b"x" * 128) == lb.E_INVALID  # too few qubits


def test_fused_layout_selftest():
    # The tile pass's planner, on the host: random groups (up to 13 bits, 8 above bit 4) and
    # permutations over 14..33 local qubits: every map consistent, every quarter-warp access free
    # of bank conflicts under the swizzle, every gate on its segment's register levels.
    import ctypes as C

    import lyth_b200 as lb

    planned, boxes = C.c_uint32(), C.c_uint32()
    st = lb.lib.lyth_b200_fused_layout_selftest(20_260_930, 4000, C.byref(planned), C.byref(boxes))
    assert st == 0, f"layout check {st} failed"
    assert planned.value == 4000 and boxes.value > 4000


def test_plan_handle_settings_are_validated_on_the_host():
    # Plan handles take the engine's settings with the engine's checks and no device.
    import lyth_b200 as lb
    from lyth_b200.statevector import Plan

    with Plan(20, 0, 2) as p:
        for bad in (0, 14):
            with pytest.raises(lb.LythError):
                p.set_fusion(bad)
        for bad in (0, 7):
            with pytest.raises(lb.LythError):
                p.set_swap_batch(bad)
        assert lb.lib.lyth_sv_set_chunk(p._h, 1000) == lb.E_UNSUPPORTED   # not a power of two
        assert lb.lib.lyth_sv_set_chunk(p._h, 512) == lb.E_UNSUPPORTED    # below 1024
        assert lb.lib.lyth_sv_set_chunk(p._h, 1 << 20) == lb.E_UNSUPPORTED  # beyond the shard
        assert lb.lib.lyth_sv_set_chunk(p._h, 1 << 12) == lb.OK
        # no peers are mapped on a plan handle: the copy-engine transport is refused
        assert lb.lib.lyth_sv_set_transport(p._h, 1) == lb.E_UNSUPPORTED
        assert lb.lib.lyth_sv_set_transport(p._h, 2) == lb.E_UNSUPPORTED
        assert lb.lib.lyth_sv_set_transport(p._h, 3) == lb.E_UNSUPPORTED
        assert lb.lib.lyth_sv_set_transport(p._h, 4) == lb.E_UNSUPPORTED
        assert lb.lib.lyth_sv_set_transport(p._h, 5) == lb.E_INVALID
        assert lb.lib.lyth_sv_set_transport(p._h, -1) == lb.E_INVALID
        assert lb.lib.lyth_sv_set_transport(p._h, 0) == lb.OK
        assert lb.lib.lyth_sv_transport(p._h) == 0
    with pytest.raises(lb.LythError):
        Plan(20, 2, 2)   # rank out of range
    with pytest.raises(lb.LythError):
        Plan(20, 0, 3)   # not a power of two
    with pytest.raises(lb.LythError):
        Plan(2, 0, 4)    # fewer than two local qubits


def test_plan_counters_do_not_depend_on_the_chunk():
    # Bytes sent and exchanges are properties of the schedule, not of its pipelining.
    from lyth_b200 import circuit as cc
    from lyth_b200.statevector import Plan

    gates = cc.layered(20, 2, cc.Rng(cc.BENCH_SEED))
    stats = []
    for chunk in (None, 1 << 12):
        with Plan(20, 1, 4) as p:
            if chunk:
                import lyth_b200 as lb
                assert lb.lib.lyth_sv_set_chunk(p._h, chunk) == lb.OK
            p.apply(gates)
            p.finish()
            stats.append(p.stats())
    assert stats[0] == stats[1] and stats[0]["exchanges"] > 0


@pytest.mark.parametrize("k", [2, 3, 4, 5, 6])
def test_engine_fusion_groups_match_lyth_circuit_fuse(k):
    # lyth-circuit's fuse (lib.rs:72-100, restated in circuit.fuse) against the engine's own groups,
    # read from a plan handle: on circuits without SWAPs (the engine relabels those instead of
    # fusing them) and with no group above the engine's 48-gate cap, the groups are the same gates
    # on the same qubits, in the same order.
    from lyth_b200 import circuit as cc
    from lyth_b200.statevector import Plan

    rng = cc.Rng(20_260_930)
    circuits = [(12, cc.ghz(12)), (10, cc.qft(10, rng)), (10, cc.random(10, 20, rng)), (14, cc.random(14, 12, rng))]
    for q, gates in circuits:
        gates = [g for g in gates if not isinstance(g, cc.Swap)]
        want = cc.fuse(gates, k)
        if any(len(grp.gates) > 48 for grp in want):
            continue
        with Plan(q, 0, 1) as p:
            p.set_fusion(k)
            p.apply(gates)
            ops = p.ops()
        got = []
        for o in ops:
            if o["kind"] == "fused":
                got.append(sorted({b for t, c, _ in o["gates"] for b in (t, c) if b >= 0}, reverse=True))
            else:
                assert o["kind"] in ("u", "cu"), o["kind"]
                got.append(sorted({o["a"]} | ({o["b"]} if o["kind"] == "cu" else set()), reverse=True))
        assert got == [grp.qubits for grp in want], (q, k)


def test_nccl_wait_deadline_logic_on_the_host():
    # The multi-GPU sync's failure path (ncclCommGetAsyncError polling, ncclCommAbort on an error
    # or at a host deadline) with fake hooks: no device, no NCCL.
    import ctypes as C

    import lyth_b200 as lb

    aborts, polls = C.c_int32(), C.c_uint64()
    assert lb.lib.lyth_sv_deadline_selftest(0, 1000.0, C.byref(aborts), C.byref(polls)) == lb.OK
    assert aborts.value == 0 and polls.value == 3
    assert lb.lib.lyth_sv_deadline_selftest(1, 1000.0, C.byref(aborts), C.byref(polls)) == lb.E_NCCL
    assert aborts.value == 1 and polls.value == 2
    import time

    t0 = time.perf_counter()
    assert lb.lib.lyth_sv_deadline_selftest(2, 50.0, C.byref(aborts), C.byref(polls)) == lb.E_TIMEOUT
    assert aborts.value == 1 and 0.04 < time.perf_counter() - t0 < 5.0
    assert lb.lib.lyth_sv_deadline_selftest(3, 1000.0, C.byref(aborts), C.byref(polls)) == 719  # cudaErrorLaunchFailure
    assert aborts.value == 0


def test_deadline_setting_is_checked():
    import lyth_b200 as lb
    from lyth_b200.statevector import Plan

    with Plan(20, 0, 2) as p:
        assert lb.lib.lyth_sv_set_deadline(p._h, 0.5) == lb.E_UNSUPPORTED
        assert lb.lib.lyth_sv_set_deadline(p._h, 2000.0) == lb.OK


def test_pull_queue_setting_range():
    # 0 = one queue per partner slice (the default), 1..8 = that many pieces and queues
    import lyth_b200 as lb
    from lyth_b200.statevector import Plan

    with Plan(12, 0, 4) as p:
        for q in (0, 1, 5, 8):
            assert lb.lib.lyth_sv_set_pull_queues(p._h, q) == 0
        for q in (-1, 9):
            assert lb.lib.lyth_sv_set_pull_queues(p._h, q) == lb.E_UNSUPPORTED


def test_transport_names_map_onto_the_c_abi_kinds():
    # StateVector.set_transport / .transport are the names of lyth_sv_set_transport's kinds
    # 0..4; a handle without IPC mappings (a plan handle here) takes only NCCL, and an unknown
    # name is refused before any call
    import lyth_b200 as lb
    from lyth_b200.statevector import Plan, StateVector

    assert StateVector.TRANSPORTS == ("nccl", "copy_engine", "peer_load", "mixed", "peer_store")
    with Plan(16, 0, 2) as p:
        StateVector.set_transport(p, "nccl")
        StateVector.set_transport(p, False)
        assert StateVector.transport.fget(p) == "nccl"
        for kind in ("copy_engine", "peer_load", "mixed", "peer_store", True):
            with pytest.raises(lb.LythError):
                StateVector.set_transport(p, kind)
        with pytest.raises(ValueError):
            StateVector.set_transport(p, "shared_memory")
        assert StateVector.transport.fget(p) == "nccl"
