"""The multi-rank state vector's planner on CPU ranks (gloo): every rank records, through a plan
handle (lyth_sv_plan_create), the exact steps its engine would run -- fused passes, swap-ins of
rank-bit qubits, pairwise exchanges, the read-out's permutation steps -- and replays them on its
own shard with the host evaluator's gates, trading shards with its partner over gloo where a
step crosses ranks. Every rank's final shard must equal the unsharded evaluator's, bit for bit,
and every pair of ranks must take the steps between them in the same order.

This covers the sharding logic (the qubit map, victim choice, rank-bit controls, rank-rank
swaps) without a GPU; the GPU tests check the kernels that run each step."""
import os
import socket

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COMM = ("exchange", "swap_lr", "swap_rr", "swap_multi")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def circuits(q):
    from lyth_b200 import circuit as cc

    t = q - 1
    aimed = [cc.U(t, cc.H), cc.CU(t, 0, cc.X), cc.CU(1, t, cc.zyz(0.3, 0.2, 0.1)), cc.Swap(0, t),
             cc.U(t, cc.zyz(1.0, 2.0, 3.0)), cc.CU(t, t - 1, cc.phase(0.7)), cc.Swap(t - 1, 2),
             cc.CU(t - 1, t, cc.zyz(-0.4, 0.9, 1.3)), cc.Swap(t, t - 1), cc.U(0, cc.H)]
    return [
        ("layered", cc.layered(q, 3, cc.Rng(cc.BENCH_SEED))),
        ("random", cc.random(q, 12, cc.Rng(20_260_931))),
        ("qft", cc.qft(q, cc.Rng(20_260_932))),
        ("ghz", cc.ghz(q)),
        ("rank-bit gates", aimed),
    ]


def _trade(mine, partner):
    """Send this rank's (re, im) to `partner` and return the partner's."""
    import torch.distributed as dist

    out = torch.from_numpy(np.concatenate(mine))
    back = torch.empty_like(out)
    reqs = [dist.isend(out, partner), dist.irecv(back, partner)]
    for r in reqs:
        r.wait()
    n = mine[0].size
    b = back.numpy()
    return np.ascontiguousarray(b[:n]), np.ascontiguousarray(b[n:])


def _paired(rank, bit, re, im, partner_state, fn):
    """Run `fn` on the 2L-amplitude sub-state (this shard, the partner's) ordered by rank bit
    `bit`, and keep this rank's half."""
    pr, pi = partner_state
    low = not ((rank >> bit) & 1)
    cr = np.concatenate([re, pr] if low else [pr, re])
    ci = np.concatenate([im, pi] if low else [pi, im])
    cr, ci = fn(cr, ci)
    n = re.size
    sl = slice(0, n) if low else slice(n, 2 * n)
    return np.ascontiguousarray(cr[sl]), np.ascontiguousarray(ci[sl])


def partners_of(op, rank):
    """The ranks a communication step trades with (none: no data moves)."""
    if op["kind"] == "swap_multi":
        mask = sum(1 << b for b in op["rbits"])
        return [r for r in range(rank & ~mask, (rank | mask) + 1) if (r & ~mask) == (rank & ~mask) and r != rank]
    p = partner_of(op, rank)
    return [] if p == rank else [p]


def partner_of(op, rank):
    """The rank a pairwise communication step trades with (this rank itself: no data moves)."""
    if op["kind"] == "exchange":
        return rank ^ (1 << op["a"])
    if op["kind"] == "swap_lr":
        return rank ^ (1 << op["b"])
    if ((rank >> op["a"]) & 1) != ((rank >> op["b"]) & 1):
        return rank ^ (1 << op["a"]) ^ (1 << op["b"])
    return rank


def pairs_agree(seqs):
    """Each pair of ranks takes the steps between them in the same order. (Ranks whose
    rank-bit control is 0 skip a controlled exchange together with their partner, so whole
    sequences may differ between pairs.)"""
    for r, seq in enumerate(seqs):
        for p in range(len(seqs)):
            if p != r and [e[:3] for e in seq if e[3] == p] != [e[:3] for e in seqs[p] if e[3] == r]:
                return False
    return True


def _swap_multi(vbits, rbits, rank, local_bits, re, im, run):
    """Local bits vbits[j] <-> rank bits rbits[j]: gather the 2^k shards of the ranks that differ in
    those rank bits (ordered by their values), swap bit vbits[j] with bit local_bits + j of the
    combined state, and keep this rank's part."""
    import torch.distributed as dist

    k = len(vbits)
    mask = sum(1 << b for b in rbits)
    def rank_of(q):
        r = rank & ~mask
        for j, b in enumerate(rbits):
            r |= ((q >> j) & 1) << b
        return r
    qself = sum(((rank >> b) & 1) << j for j, b in enumerate(rbits))
    mine = torch.from_numpy(np.concatenate([re, im]))
    parts = {qself: (re, im)}
    reqs, bufs = [], {}
    for q in range(1 << k):
        if q == qself:
            continue
        bufs[q] = torch.empty_like(mine)
        reqs.append(dist.isend(mine, rank_of(q)))
        reqs.append(dist.irecv(bufs[q], rank_of(q)))
    for r in reqs:
        r.wait()
    n = re.size
    for q, t in bufs.items():
        b = t.numpy()
        parts[q] = (np.ascontiguousarray(b[:n]), np.ascontiguousarray(b[n:]))
    cr = np.concatenate([parts[q][0] for q in range(1 << k)])
    ci = np.concatenate([parts[q][1] for q in range(1 << k)])
    cr, ci = run([(2, v, local_bits + j, [0.0] * 8) for j, v in enumerate(vbits)], cr, ci)
    sl = slice(qself * n, (qself + 1) * n)
    return np.ascontiguousarray(cr[sl]), np.ascontiguousarray(ci[sl])


def _permute(src, dst, re, im):
    """The value at index i moves to the index whose bit dst[j] is bit src[j] of i."""
    idx = np.arange(re.size, dtype=np.int64)
    to = idx.copy()
    for b in src:
        to &= ~(1 << b)
    for s_, d_ in zip(src, dst):
        to |= ((idx >> s_) & 1) << d_
    out_r, out_i = np.empty_like(re), np.empty_like(im)
    out_r[to] = re
    out_i[to] = im
    return out_r, out_i


def replay(ops, rank, local_bits, re, im):
    from oracle import oracle as orc

    run = orc.run_gates
    for op in ops:
        k, a, b, c, m = op["kind"], op["a"], op["b"], op["c"], op["m"]
        if k == "u":
            re, im = run([(0, a, 0, m)], re, im)
        elif k == "cu":
            re, im = run([(1, a, b, m)], re, im)
        elif k == "fused":
            re, im = run([(0, t, 0, gm) if cb < 0 else (1, cb, t, gm) for t, cb, gm in op["gates"]], re, im)
        elif k == "swap_local":
            re, im = run([(2, a, b, [0.0] * 8)], re, im)
        elif k == "exchange":
            other = _trade((re, im), rank ^ (1 << a))
            g = (0, local_bits, 0, m) if c < 0 else (1, c, local_bits, m)
            re, im = _paired(rank, a, re, im, other, lambda x, y: run([g], x, y))
        elif k == "swap_lr":
            other = _trade((re, im), rank ^ (1 << b))
            re, im = _paired(rank, b, re, im, other, lambda x, y: run([(2, a, local_bits, [0.0] * 8)], x, y))
        elif k == "swap_rr":
            if ((rank >> a) & 1) != ((rank >> b) & 1):
                re, im = _trade((re, im), rank ^ (1 << a) ^ (1 << b))
        elif k == "swap_multi":
            re, im = _swap_multi(op["bits"], op["rbits"], rank, local_bits, re, im, run)
        elif k == "permute":
            re, im = _permute(op["bits"], op["rbits"], re, im)
        else:
            raise AssertionError(k)
    return re, im


def _worker(rank, nranks, q, port, out_dir):
    import sys

    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from lyth_b200.statevector import Plan
    from oracle import oracle as orc
    from tests.test_gpu_statevector import as_tuples

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=nranks)
    lines = []
    try:
        L = (1 << q) // nranks
        local_bits = L.bit_length() - 1
        lo, hi = rank * L, (rank + 1) * L
        cases = [(name, gates, False) for name, gates in circuits(q)]
        cases.append(("layered, zeros", circuits(q)[0][1], True))
        for ci, (name, gates, zeros) in enumerate(cases):
            re0, im0 = orc.random_state(400 + ci, q)
            if zeros:  # a third of the components exactly +0 or -0
                rng = np.random.default_rng(ci)
                for a in (re0, im0):
                    hit = rng.random(a.size) < 1 / 3
                    a[hit] = np.where(rng.random(hit.sum()) < 0.5, np.float32(0.0), np.float32(-0.0))
            want_r, want_i = orc.run_gates(as_tuples(gates), re0, im0)
            for fuse, remap, batch, diag in ((6, True, 6, True), (6, True, 1, True), (3, True, 6, True),
                                             (1, True, 6, True), (6, False, 6, True), (1, False, 6, True),
                                             (6, True, 1, False), (6, False, 6, False)):
                with Plan(q, rank, nranks) as p:
                    p.set_fusion(fuse)
                    p.set_remap(remap)
                    p.set_swap_batch(batch)
                    p.set_diagonal(diag)
                    p.apply(gates)
                    p.finish()
                    ops, st = p.ops(), p.stats()
                comm = [(o["kind"], o["a"], o["b"], p) for o in ops if o["kind"] in COMM
                        for p in partners_of(o, rank)]
                seqs = [None] * nranks
                dist.all_gather_object(seqs, comm)
                same = pairs_agree(seqs)
                re, im = replay(ops, rank, local_bits, np.ascontiguousarray(re0[lo:hi]),
                                np.ascontiguousarray(im0[lo:hi]))
                wr, wi = want_r[lo:hi], want_i[lo:hi]
                bits = np.array_equal(re.view(np.uint32), wr.view(np.uint32)) and \
                    np.array_equal(im.view(np.uint32), wi.view(np.uint32))
                # Rank-bit diagonals as scalars: equal in value, and bit for bit wherever the
                # result is not an exact zero (whose sign may differ); bit for bit otherwise.
                value = np.array_equal(re, wr) and np.array_equal(im, wi) and \
                    np.array_equal(re.view(np.uint32)[wr != 0], wr.view(np.uint32)[wr != 0]) and \
                    np.array_equal(im.view(np.uint32)[wi != 0], wi.view(np.uint32)[wi != 0])
                ok = value if (diag and zeros) else bits
                nmulti = sum(o["kind"] == "swap_multi" for o in ops)
                lines.append(f"{name}|{fuse}|{int(remap)}/{batch}/{int(diag)}|{int(ok)}|{int(same)}|{len(comm)}|"
                             f"{nmulti}")
    finally:
        dist.destroy_process_group()
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write("\n".join(lines) + "\n")


@pytest.mark.parametrize("nranks,q", [(2, 9), (4, 10), (8, 11)])
def test_sharded_plan_replays_bit_exact(nranks, q, tmp_path):
    port = _free_port()
    ctx = torch.multiprocessing.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, nranks, q, port, str(tmp_path))) for r in range(nranks)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for r, p in enumerate(procs):
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0, f"rank {r} exit {p.exitcode}"
    total_comm = total_multi = 0
    for r in range(nranks):
        for line in open(tmp_path / f"r{r}.txt").read().splitlines():
            name, fuse, remap, ok, same, ncomm, nmulti = line.split("|")
            assert ok == "1", f"rank {r}: {name} fuse={fuse} remap/batch/diag={remap}: shard differs"
            assert same == "1", f"{name} fuse={fuse} remap/batch/diag={remap}: a pair of ranks disagree on their steps"
            total_comm += int(ncomm)
            total_multi += int(nmulti)
    assert total_comm > 0
    if nranks >= 4:
        assert total_multi > 0, "batched swap-ins must be exercised"


def test_plan_handle_needs_no_gpu():
    # A plan handle loads and plans with no CUDA device and no NCCL; the fused group limits hold.
    from lyth_b200 import circuit as cc
    from lyth_b200.statevector import Plan

    gates = cc.layered(12, 2, cc.Rng(cc.BENCH_SEED))
    for k in range(1, 7):
        with Plan(12, 0, 1) as p:
            p.set_fusion(k)
            p.apply(gates)
            ops = p.ops()
        assert all(o["kind"] in ("u", "cu", "fused", "swap_local") for o in ops)
        for o in ops:
            if o["kind"] == "fused":
                assert 2 <= len(o["gates"]) <= 48
                assert len({b for t, c, _ in o["gates"] for b in (t, c) if b >= 0}) <= k
        if k == 1:
            assert not any(o["kind"] == "fused" for o in ops)
        # gates run = gates given minus swaps (relabels)
        run = sum(len(o["gates"]) if o["kind"] == "fused" else 1 for o in ops)
        assert run == sum(not isinstance(g, cc.Swap) for g in gates)


def test_readout_permutation_passes_replay_bit_exact():
    # 16 qubits on one rank: the read-out undoes the qubit map with permutation passes (the tile
    # pass's size); replayed with the oracle's gates and numpy, the result is the oracle's.
    import sys

    sys.path.insert(0, ROOT)
    from lyth_b200 import circuit as cc
    from lyth_b200.statevector import Plan
    from oracle import oracle as orc
    from tests.test_gpu_statevector import as_tuples

    q = 16
    gates = cc.layered(q, 3, cc.Rng(cc.BENCH_SEED))
    re0, im0 = orc.random_state(700, q)
    want_r, want_i = orc.run_gates(as_tuples(gates), re0, im0)
    with Plan(q, 0, 1) as p:
        p.apply(gates)
        p.finish()
        ops = p.ops()
    assert any(o["kind"] == "permute" for o in ops)
    re, im = replay(ops, 0, q, re0.copy(), im0.copy())
    assert np.array_equal(re.view(np.uint32), want_r.view(np.uint32))
    assert np.array_equal(im.view(np.uint32), want_i.view(np.uint32))


def _range_worker(rank, world, port, out_dir):
    import sys

    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    import lyth_b200 as lb

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rows = []
        for n in (0, 1, 1000, 1 << 20, (1 << 20) + 3, 1 << 33):
            off, cnt = lb.stream_range(n, rank, world)
            got = [None] * world
            dist.all_gather_object(got, (off, cnt))
            rows.append((n, got))
    finally:
        dist.destroy_process_group()
    import json

    with open(os.path.join(out_dir, f"range{rank}.json"), "w") as f:
        json.dump(rows, f)


@pytest.mark.parametrize("world", [2, 8])
def test_stream_ranges_cover_once(world, tmp_path):
    # Large streams shard as contiguous ranges, one per rank, with no collective on the data
    # path: every rank derives the same partition, which covers [0, n) once, 16-byte aligned.
    import json

    port = _free_port()
    ctx = torch.multiprocessing.get_context("spawn")
    procs = [ctx.Process(target=_range_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for r, p in enumerate(procs):
        assert p.exitcode == 0, r
    tables = [json.load(open(tmp_path / f"range{r}.json")) for r in range(world)]
    for rows in tables[1:]:
        assert rows == tables[0]  # the same partition everywhere
    for n, got in tables[0]:
        pos = 0
        for off, cnt in got:
            assert off == pos and cnt >= 0 and off % 1024 == 0
            pos += cnt
        assert pos == n


def test_diagonal_rank_gates_move_no_data():
    # A diagonal gate on a rank-bit target (a phase, a controlled phase) is a scalar on each shard:
    # no swap-in, no exchange. On the benchmark circuit at 8 ranks only the H gates on the three
    # rank-bit qubits move data: three single swap-ins per layer, one batched one.
    from lyth_b200 import circuit as cc
    from lyth_b200.statevector import Plan

    layers = 6
    gates = cc.layered(33, layers, cc.Rng(cc.BENCH_SEED))
    counts = {}
    for diag in (True, False):
        for batch in (1, 3):
            with Plan(33, 5, 8) as p:
                p.set_diagonal(diag)
                p.set_swap_batch(batch)
                p.apply(gates)
                ops = p.ops()
            counts[diag, batch] = sum(o["kind"] in COMM for o in ops)
    assert counts[True, 1] == 3 * layers
    assert counts[True, 3] == layers
    assert counts[False, 1] > counts[True, 1] and counts[False, 3] > counts[True, 3]
    t = 32  # a rank bit at 8 ranks, before any swap
    for g in ([cc.U(t, cc.phase(0.3))], [cc.CU(0, t, cc.phase(0.3))], [cc.CU(t - 1, t, cc.phase(0.3))],
              [cc.U(t, cc.Z)]):
        for rank in range(8):
            with Plan(33, rank, 8) as p:
                p.apply(g)
                ops = p.ops()
            assert not any(o["kind"] in COMM for o in ops), (g, rank, ops)
