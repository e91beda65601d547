"""The state vector at the benchmark's single-GPU size: one layer of the benchmark circuit on a
30-qubit state (8 GiB), bit for bit against the host evaluator on the same seeded input -- the
full-size check of the circuit table (first layer, per gate, on all host cores). It takes a few
minutes of host time and 24 GiB of host memory, so it runs only with LYTH_FULL_SIZE=1."""
import os

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


@pytest.mark.skipif(os.environ.get("LYTH_FULL_SIZE") != "1", reason="set LYTH_FULL_SIZE=1 (host minutes, 24 GiB)")
def test_first_layer_at_30_qubits_bit_exact(cuda):
    import lyth_b200 as lb
    from lyth_b200 import circuit as cc
    from oracle import oracle as orc
    from tests.test_gpu_statevector import as_tuples

    q = 30
    gates = cc.layered(q, 1, cc.Rng(cc.BENCH_SEED))
    with lb.StateVector(q, device=0) as sv:
        sv.init_random(cc.BENCH_SEED)
        re0, im0 = np.empty(1 << q, np.float32), np.empty(1 << q, np.float32)
        sv.get_local(re0, im0)          # the seeded input, as the device made it
        sv.apply(gates)
        sv.sync()
        gr, gi = np.empty_like(re0), np.empty_like(im0)
        sv.get_local(gr, gi)
        st = sv.stats()
    wr, wi = orc.run_gates(as_tuples(gates), re0, im0)
    assert np.array_equal(gr.view(np.uint32), wr.view(np.uint32))
    assert np.array_equal(gi.view(np.uint32), wi.view(np.uint32))
    assert st["passes"] < len(gates) // 4  # fused: far fewer passes than gates
