"""The state vector at the benchmark's single-GPU size: the first AND the last layer of the
20-layer benchmark circuit on a 30-qubit state (2^30 amplitudes, 8 GiB on the device), each
bit for bit against the host evaluator applying that layer's gates unfused, in order, to the
same input (lyth-circuit's execute, crates/lyth-circuit/src/lib.rs:327-371; the fusion claim of
crates/lyth-circuit/tests/fusion.rs:53-92 at full size).

The engine runs the whole circuit as the benchmark does (fused tile passes, SWAPs as
relabels); the state is read out (qubit map undone) before layer 1, after layer 1, before layer
20 and after layer 20. The evaluator applies layer 1 to the first read-out and layer 20 to the
third, in place on all host cores. Host memory: 16 GiB at the peak; host time: about two
evaluator layers (74 gates each over 2^30 amplitudes)."""
import gc

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

Q = 30
LAYERS = 20


def _read(sv):
    re, im = np.empty(1 << Q, np.float32), np.empty(1 << Q, np.float32)
    sv.get_local(re, im)
    return re, im


def _check_layer(tuples, before, after, what):
    from oracle import oracle as orc

    wr, wi = orc.run_gates(tuples, before[0], before[1], inplace=True)
    gr, gi = after
    bad_re = int(np.count_nonzero(gr.view(np.uint32) != wr.view(np.uint32)))
    bad_im = int(np.count_nonzero(gi.view(np.uint32) != wi.view(np.uint32)))
    assert bad_re == 0 and bad_im == 0, f"{what}: {bad_re} re and {bad_im} im words differ"


def test_first_and_last_layer_at_30_qubits_bit_exact(cuda):
    import lyth_b200 as lb
    from lyth_b200 import circuit as cc
    from tests.test_gpu_statevector import as_tuples

    gates = cc.layered(Q, LAYERS, cc.Rng(cc.BENCH_SEED))
    per = len(gates) // LAYERS
    assert per == 74
    first, middle, last = gates[:per], gates[per:(LAYERS - 1) * per], gates[(LAYERS - 1) * per:]
    with lb.StateVector(Q, device=0) as sv:
        sv.init_random(cc.BENCH_SEED)
        s0 = _read(sv)                      # the seeded input, as the device made it
        sv.apply(first)
        sv.sync()
        s1 = _read(sv)
        passes_first = sv.stats()["passes"]
        _check_layer(as_tuples(first), s0, s1, "layer 1")
        del s0, s1
        gc.collect()
        sv.apply(middle)
        sv.sync()
        s19 = _read(sv)
        sv.apply(last)
        sv.sync()
        s20 = _read(sv)
        _check_layer(as_tuples(last), s19, s20, f"layer {LAYERS}")
    assert passes_first < per // 4  # fused: far fewer passes than gates
