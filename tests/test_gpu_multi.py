"""The sharded state vector on 2 (or more) GPUs: each rank's shard, after whole circuits whose
gates hit the rank bits (exchange), a rank-bit control (rank-local) and SWAPs across the
boundary (relabels undone by real exchanges at read-out), is bit-identical to the host
evaluator's unsharded result. One process per GPU, spawned by the test; NVLS off."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ngpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _worker(rank, nranks, q, case, nid, out_dir, remap=True, batch=6, ce=True, chunk=None, queues=None):
    import sys

    sys.path.insert(0, ROOT)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import lyth_b200 as lb
    from tests.test_gpu_statevector import as_tuples, suite

    torch.cuda.set_device(rank)
    from oracle import oracle as orc

    name, q, gates = case_gates(case, q)
    re0, im0 = orc.random_state(300 + case, q)
    L = (1 << q) // nranks
    lo, hi = rank * L, (rank + 1) * L
    with lb.StateVector(q, device=rank, rank=rank, nranks=nranks, nccl_id=nid) as sv:
        sv.set_remap(remap)
        sv.set_swap_batch(batch)
        sv.set_transport(ce)
        if chunk:
            sv.set_chunk(chunk)
        if queues:
            lb.check(lb.lib.lyth_sv_set_pull_queues(sv._h, queues), "set_pull_queues")
        transport = sv.transport
        sv.set_local(np.ascontiguousarray(re0[lo:hi]), np.ascontiguousarray(im0[lo:hi]))
        sv.apply(gates)
        sv.sync()
        gr, gi = np.empty(L, np.float32), np.empty(L, np.float32)
        sv.get_local(gr, gi)
        st = sv.stats()
    with lb.Plan(q, rank, nranks) as plan:  # the same planner, recording only
        plan.set_remap(remap)
        plan.set_swap_batch(batch)
        plan.apply(gates)
        plan.finish()
        pst = plan.stats()
    same_plan = all(pst[k] == st[k] for k in ("passes", "exchanges", "bytes_sent"))
    wr, wi = orc.run_gates(as_tuples(gates), re0, im0)
    ok = np.array_equal(gr.view(np.uint32), wr[lo:hi].view(np.uint32)) and \
        np.array_equal(gi.view(np.uint32), wi[lo:hi].view(np.uint32))
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(f"{int(ok)} {st['exchanges']} {st['bytes_sent']} {int(same_plan)} {transport}\n")
    del suite


def case_gates(case, q):
    from lyth_b200 import circuit as cc

    if case == 0:
        return "layered", q, cc.layered(q, 3, cc.Rng(cc.BENCH_SEED))
    if case == 1:
        return "random", q, cc.random(q, 6, cc.Rng(20_260_931))
    # gates aimed at the top (rank) bits: U on them, CU with rank-bit control / target, swaps
    t = q - 1
    g = [cc.U(t, cc.H), cc.CU(t, 0, cc.X), cc.CU(1, t, cc.zyz(0.3, 0.2, 0.1)), cc.Swap(0, t),
         cc.U(t, cc.zyz(1.0, 2.0, 3.0)), cc.CU(t, t - 1, cc.phase(0.7)), cc.Swap(t - 1, 2), cc.U(0, cc.H)]
    return "rank-bit gates", q, g


def _run_ranks(nranks, q, case, remap, batch, tmp_path, ce=True, chunk=None, queues=None):
    import lyth_b200 as lb

    nid = lb.unique_id()
    ctx = torch.multiprocessing.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, nranks, q, case, nid, str(tmp_path), remap, batch, ce, chunk,
                                               queues))
             for r in range(nranks)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for r, p in enumerate(procs):
        assert p.exitcode == 0, f"rank {r} exit {p.exitcode}"
        ok, ex, sent, same_plan, transport = open(tmp_path / f"r{r}.txt").read().split()
        assert transport == (ce if isinstance(ce, str) else "copy_engine" if ce else "nccl")
        assert ok == "1", f"rank {r}: shard differs from the evaluator"
        assert same_plan == "1", f"rank {r}: the plan handle's counters differ from the engine's"
        assert int(ex) > 0, "the circuit must exercise the exchange"


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("remap", [True, False])
@pytest.mark.parametrize("case", [0, 1, 2])
def test_two_ranks_bit_exact(case, remap, tmp_path):
    _run_ranks(2, 18, case, remap, 6, tmp_path)


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("ce", [True, False])
@pytest.mark.parametrize("case", [0, 2])
def test_two_ranks_many_chunks(case, ce, tmp_path):
    # 1024-amplitude chunks: every swap-in and exchange runs as a long pipeline, so both send and
    # receive slots are reused many times within one exchange (flags, events, slot waits)
    _run_ranks(2, 18, case, True, 6, tmp_path, ce=ce, chunk=1024)


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("queues", [1, 5, 8])
def test_two_ranks_pull_queues(queues, tmp_path):
    # a swap-in pull cut into pieces over 1, 5 or 8 copy-engine queues (and short chunks, so the
    # pieces of consecutive chunks interleave on every queue)
    _run_ranks(2, 18, 0, True, 6, tmp_path, chunk=4096, queues=queues)


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("kind", ["peer_load", "peer_store"])
@pytest.mark.parametrize("chunk", [None, 1024])
@pytest.mark.parametrize("case", [0, 1, 2])
def test_two_ranks_peer_transport(case, chunk, kind, tmp_path):
    # the SMs pull the partner's packed chunks and store them into the shard (no receive buffer),
    # or store this rank's packed chunks into the partner's shard; with 1024-amplitude chunks the
    # send slots are reused many times within one exchange
    _run_ranks(2, 18, case, True, 6, tmp_path, ce=kind, chunk=chunk)


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("case", [0, 2])
def test_two_ranks_nccl_transport(case, tmp_path):
    _run_ranks(2, 18, case, True, 6, tmp_path, ce=False)


@pytest.mark.skipif(_ngpus() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("batch", [6, 1])
@pytest.mark.parametrize("case", [0, 2])
def test_four_ranks_bit_exact(case, batch, tmp_path):
    # two rank bits: batch 6 takes the batched (all-to-all among 4 ranks) swap-ins
    _run_ranks(4, 19, case, True, batch, tmp_path)


@pytest.mark.skipif(_ngpus() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("batch", [1, 6])
def test_four_ranks_many_chunks(batch, tmp_path):
    _run_ranks(4, 19, 0, True, batch, tmp_path, chunk=1024)


@pytest.mark.skipif(_ngpus() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("kind", ["peer_load", "mixed", "peer_store"])
@pytest.mark.parametrize("batch", [6, 1])
def test_four_ranks_peer_transport(batch, kind, tmp_path):
    # batched swap-ins pull from 3 partners at once with SM loads, in short chunks; "mixed" takes
    # the copy engines for the pairwise ones in between
    _run_ranks(4, 19, 0, True, batch, tmp_path, ce=kind, chunk=1024)


@pytest.mark.skipif(_ngpus() < 4, reason="needs 4 GPUs")
def test_four_ranks_nccl_transport(tmp_path):
    _run_ranks(4, 19, 0, True, 6, tmp_path, ce=False)


@pytest.mark.skipif(_ngpus() < 8, reason="needs 8 GPUs")
@pytest.mark.parametrize("case", [0, 2])
def test_eight_ranks_bit_exact(case, tmp_path):
    # three rank bits: batched swap-ins among up to 8 ranks over the copy engines
    _run_ranks(8, 20, case, True, 6, tmp_path)


@pytest.mark.skipif(_ngpus() < 8, reason="needs 8 GPUs")
@pytest.mark.parametrize("kind", ["peer_load", "mixed", "peer_store"])
def test_eight_ranks_peer_transport(kind, tmp_path):
    _run_ranks(8, 20, 0, True, 6, tmp_path, ce=kind, chunk=1024)
