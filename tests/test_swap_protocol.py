"""The swap-in pipeline's ordering (lyth_b200/csrc/sv.cu, physical_swap_multi), modelled on the
host: every rank's compute and communication streams, its events and the cross-GPU flags, issued in
the order the engine issues them for each IPC transport form -- copy-engine pulls into receive
chunks ("ce"), SM peer loads fused with the unpack ("pl"), SM stores into the partners' shards
("ps") -- and consecutive swap-ins that mix the forms as the "mixed" default does. Kernels run one
cell at a time in a random order and interleave with every other stream, so a read that could see
a cell before its writer (or after its overwriter) shows up as a wrong final shard; a wait that
could never end shows up as a deadlock. Each shard, read out on its own compute stream after the
swap-ins, must be what a sequential swap of bits leaves, and a rank's teardown (teardown_ce: streams
drained, its send slots' "pulled" flags awaited, then its memory freed) must never precede a
peer's access to that memory.

The model is a statement of the protocol, not the CUDA code: it follows the engine's issue order,
and the comments name the step of physical_swap_multi each group of ops mirrors."""
import random

import pytest


class Event:
    def __init__(self):
        self.latest = None


class Mem(dict):
    """One rank's device memory (a shard, a chunk slot or a flag block): any access after the rank
    freed it is a use after free by a peer."""
    freed = False

    def _check(self):
        assert not self.freed, "a peer touched memory its owner had freed"

    def __getitem__(self, k):
        self._check()
        return dict.__getitem__(self, k)

    def __setitem__(self, k, v):
        self._check()
        dict.__setitem__(self, k, v)

    def get(self, k, d=None):
        self._check()
        return dict.get(self, k, d)


class World:
    def __init__(self, nranks, nbits, nchunks, seed):
        self.R, self.G, self.N = nranks, nbits, nchunks
        self.rng = random.Random(seed)
        self.state = [Mem({(cls, c): (r, cls, c) for cls in range(1 << nbits) for c in range(nchunks)})
                      for r in range(nranks)]
        self.sre = [[Mem(), Mem()] for _ in range(nranks)]
        self.rre = [[Mem(), Mem()] for _ in range(nranks)]
        self.flags = [Mem() for _ in range(nranks)]
        self.streams = [{"S": [], "M": []} for _ in range(nranks)]
        self.done_records = set()
        self.next_rid = 0
        self.xseq = [0] * nranks
        self.slot_seq = [[0, 0] for _ in range(nranks)]
        self.slot_partners = [[[], []] for _ in range(nranks)]
        self.ev = [{k: Event() for k in ("start", "packed0", "packed1", "recv0", "recv1", "done0", "done1", "drained")}
                   for _ in range(nranks)]

    # ---- ops
    def record(self, r, s, name):
        rid = self.next_rid
        self.next_rid += 1
        self.ev[r][name].latest = rid
        self.streams[r][s].append(("record", rid))

    def wait_event(self, r, s, name):
        self.streams[r][s].append(("wait_event", self.ev[r][name].latest))

    def kernel(self, r, s, cells):
        cells = list(cells)
        self.rng.shuffle(cells)
        self.streams[r][s].append(["kernel", cells])

    def flag_wait(self, r, s, kind, srcs, b, target):
        self.streams[r][s].append(("flag_wait", r, kind, tuple(srcs), b, target))

    def flag_put(self, r, s, kind, dsts, b, value):
        self.streams[r][s].append(("flag_put", r, kind, tuple(dsts), b, value))

    def free(self, r, s):
        self.streams[r][s].append(("free", r))

    def ready(self, op):
        if op[0] == "wait_event":
            return op[1] is None or op[1] in self.done_records
        if op[0] == "flag_wait":
            _, r, kind, srcs, b, target = op
            return all(self.flags[r].get((kind, q, b), 0) >= target for q in srcs)
        return True

    def step(self, op, queue):
        if op[0] == "record":
            self.done_records.add(op[1])
        elif op[0] == "free":
            r = op[1]
            for m in [self.state[r], self.flags[r], *self.sre[r], *self.rre[r]]:
                m.freed = True
        elif op[0] == "flag_put":
            _, r, kind, dsts, b, value = op
            for d in dsts:
                key = (kind, r, b)
                self.flags[d][key] = max(self.flags[d].get(key, 0), value)
        elif op[0] == "kernel":
            op[1].pop()()
            if op[1]:
                return  # the kernel still runs: the stream stays busy
        queue.pop(0)

    def run(self):
        while True:
            live = [(r, s) for r in range(self.R) for s in ("S", "M") if self.streams[r][s]]
            if not live:
                return
            runnable = [(r, s) for r, s in live if self.ready(self.streams[r][s][0])]
            assert runnable, "deadlock: " + "; ".join(f"rank {r} {s}: {self.streams[r][s][0][:2]}" for r, s in live)
            r, s = self.rng.choice(runnable)
            q = self.streams[r][s]
            op = q[0]
            if op[0] in ("wait_event", "flag_wait"):
                q.pop(0)
            else:
                self.step(op, q)


def with_bits(cls, K, pat):
    for j, bit in enumerate(K):
        cls = (cls & ~(1 << bit)) | (((pat >> j) & 1) << bit)
    return cls


def bits_of(x, K):
    return sum(((x >> bit) & 1) << j for j, bit in enumerate(K))


def issue_swap(w, K, form_of):
    """One swap of local class bits K with the same rank bits K on every rank, in the engine's issue
    order. form_of(P) picks the form for a swap with P partners (the transport setting)."""
    k = len(K)
    P = (1 << k) - 1
    N = w.N
    for r in range(w.R):
        qself = bits_of(r, K)
        partners = [with_bits(r, K, q) for q in range(P + 1) if q != qself]
        subsets = [q for q in range(P + 1) if q != qself]
        form = form_of(P)
        seq0 = w.xseq[r]
        others = [cls for cls in range(1 << w.G) if bits_of(cls, K) == 0]

        def cells_of(q):
            return [with_bits(cls, K, q) for cls in others]

        # ev_start: the communication stream starts after the compute stream's earlier work
        w.record(r, "S", "start")
        w.wait_event(r, "M", "start")

        # pack(c): the slot waits for the pulls of its last chunk, pack_multi_kernel, "packed" to
        # every partner (for the push form also "these positions are free"), ev_packed
        def pack(c, r=r, partners=partners, subsets=subsets, form=form, seq0=seq0):
            b = c & 1
            if w.slot_seq[r][b]:
                w.flag_wait(r, "S", "pulled", w.slot_partners[r][b], b, w.slot_seq[r][b])
            ops = []
            for y, q in enumerate(subsets):
                for cls in cells_of(q):
                    def f(r=r, b=b, y=y, cls=cls, c=c):
                        w.sre[r][b][(y, cls)] = w.state[r][(cls, c)]
                    ops.append(f)
            w.kernel(r, "S", ops)
            w.flag_put(r, "S", "packed", partners, b, seq0 + c + 1)
            if form == "ps":
                w.slot_seq[r][b] = 0
                w.slot_partners[r][b] = []
            else:
                w.slot_seq[r][b] = seq0 + c + 1
                w.slot_partners[r][b] = list(partners)
            w.record(r, "S", f"packed{b}")

        pack(0)
        for c in range(N):
            b = c & 1
            seq = seq0 + c + 1
            # receive slot b is free once unpack(c - 2) drained it (copy engines only)
            if c >= 2 and form == "ce":
                w.wait_event(r, "M", f"done{b}")
            # the move on the communication stream: push_kernel / pull_unpack_kernel / the copies
            if form == "ps":
                w.wait_event(r, "M", f"packed{b}")
                w.flag_wait(r, "M", "packed", partners, b, seq)
                ops = []
                for y, p in enumerate(partners):
                    for cls in cells_of(subsets[y]):
                        def f(r=r, b=b, y=y, cls=cls, p=p, c=c, qself=qself):
                            w.state[p][(with_bits(cls, K, qself), c)] = w.sre[r][b][(y, cls)]
                        ops.append(f)
                w.kernel(r, "M", ops)
                w.flag_put(r, "M", "landed", partners, b, seq)
            elif form == "pl":
                w.wait_event(r, "M", f"packed{b}")
                w.flag_wait(r, "M", "packed", partners, b, seq)
                ops = []
                for y, p in enumerate(partners):
                    yp = [with_bits(p, K, q) for q in range(P + 1) if q != bits_of(p, K)].index(r)
                    for cls in cells_of(subsets[y]):
                        def f(r=r, b=b, yp=yp, cls=cls, p=p, c=c, qself=qself):
                            w.state[r][(cls, c)] = w.sre[p][b][(yp, with_bits(cls, K, qself))]
                        ops.append(f)
                w.kernel(r, "M", ops)
                w.flag_put(r, "M", "pulled", partners, b, seq)
            else:
                w.flag_wait(r, "M", "packed", partners, b, seq)
                ops = []
                for y, p in enumerate(partners):
                    yp = [with_bits(p, K, q) for q in range(P + 1) if q != bits_of(p, K)].index(r)
                    for cls in cells_of(subsets[y]):
                        def f(r=r, b=b, y=y, yp=yp, cls=cls, p=p, qself=qself):
                            w.rre[r][b][(y, cls)] = w.sre[p][b][(yp, with_bits(cls, K, qself))]
                        ops.append(f)
                w.kernel(r, "M", ops)
                w.flag_put(r, "M", "pulled", partners, b, seq)
            # ev_recv, pack(c + 1), the compute stream joins, unpack_multi_kernel (copy engines)
            w.record(r, "M", f"recv{b}")
            if c + 1 < N:
                pack(c + 1)
            w.wait_event(r, "S", f"recv{b}")
            if form == "ce":
                ops = []
                for y in range(P):
                    for cls in cells_of(subsets[y]):
                        def f(r=r, b=b, y=y, cls=cls, c=c):
                            w.state[r][(cls, c)] = w.rre[r][b][(y, cls)]
                        ops.append(f)
                w.kernel(r, "S", ops)
                w.record(r, "S", f"done{b}")
        # the push form ends when every partner's last "landed" of both slots has arrived
        if form == "ps":
            bl = (N - 1) & 1
            w.flag_wait(r, "S", "landed", partners, bl, seq0 + N)
            if N >= 2:
                w.flag_wait(r, "S", "landed", partners, bl ^ 1, seq0 + N - 1)
        w.xseq[r] = seq0 + N


def issue_teardown(w, wait_pulled=True):
    """teardown_ce: both streams drained, then every partner has pulled the last chunk of each send
    slot, then the rank's buffers and flag block go."""
    for r in range(w.R):
        w.record(r, "M", "drained")
        w.wait_event(r, "S", "drained")
        for b in range(2):
            if wait_pulled and w.slot_seq[r][b]:
                w.flag_wait(r, "S", "pulled", w.slot_partners[r][b], b, w.slot_seq[r][b])
        w.free(r, "S")


def sequential(state, nbits, K):
    out = [dict() for _ in state]
    for r, shard in enumerate(state):
        for (cls, c), v in shard.items():
            r2 = with_bits(r, K, bits_of(cls, K))
            cls2 = with_bits(cls, K, bits_of(r, K))
            out[r2][(cls2, c)] = v
    return out


FORMS = {
    "ce": lambda P: "ce",
    "pl": lambda P: "pl",
    "ps": lambda P: "ps",
    "mixed": lambda P: "pl" if P > 1 else "ce",
}


def run_case(nbits, nchunks, swaps, transports, seed, teardown_waits=True):
    R = 1 << nbits
    w = World(R, nbits, nchunks, seed)
    want = [dict(s) for s in w.state]
    # the host issues every swap-in before the device runs any of them (the engine is asynchronous)
    for K, t in zip(swaps, transports):
        issue_swap(w, K, FORMS[t])
        want = sequential(want, nbits, K)
    got = [dict(s) for s in w.state]
    # each rank reads its shard out after its own streams have finished the swap-ins
    for r in range(R):
        w.streams[r]["S"].append(("kernel", [lambda r=r: got[r].update(dict.items(w.state[r]))]))
    issue_teardown(w, teardown_waits)
    w.run()
    for r in range(R):
        assert got[r] == want[r], f"rank {r}: shard differs from the sequential swaps"


@pytest.mark.parametrize("form", ["ce", "pl", "ps", "mixed"])
@pytest.mark.parametrize("nbits,nchunks", [(1, 1), (1, 3), (2, 1), (2, 4), (3, 2)])
def test_one_swap_every_interleaving_family(form, nbits, nchunks):
    K = list(range(nbits))
    for seed in range(40):
        run_case(nbits, nchunks, [K], [form], seed)


@pytest.mark.parametrize("nbits", [2, 3])
def test_consecutive_swaps_mix_forms_and_reuse_slots(nbits):
    # pairwise and batched swap-ins back to back, each form following each other form, so the send
    # slots, the flags' sequence numbers and the events carry over between forms
    bitsets = [list(range(nbits)), [0], [nbits - 1], [0, 1]]
    rng = random.Random(7)
    for seed in range(60):
        swaps = [rng.choice(bitsets) for _ in range(4)]
        transports = [rng.choice(list(FORMS)) for _ in swaps]
        run_case(nbits, rng.choice([1, 2, 3]), swaps, transports, seed)


def test_the_model_catches_a_missing_wait():
    # the push form without the wait for the partners' "packed" flags: a push can overwrite a
    # partner's cells before that partner packed them, and some interleaving shows it
    original = World.flag_wait

    def drop_packed_waits_on_m(self, r, s, kind, srcs, b, target):
        if kind == "packed" and s == "M":
            return
        original(self, r, s, kind, srcs, b, target)

    failed = False
    World.flag_wait = drop_packed_waits_on_m
    try:
        for seed in range(40):
            try:
                run_case(1, 2, [[0]], ["ps"], seed)
            except AssertionError:
                failed = True
                break
    finally:
        World.flag_wait = original
    assert failed, "the model did not detect the missing wait"


def test_the_model_catches_a_teardown_that_does_not_wait_for_the_pulls():
    # with peer loads a partner reads this rank's send slot after this rank's own streams are
    # done; freeing without waiting for its "pulled" flags lets that read land on freed memory
    caught = False
    for seed in range(80):
        try:
            run_case(1, 1, [[0]], ["pl"], seed, teardown_waits=False)
        except AssertionError:
            caught = True
            break
    assert caught, "the model did not detect the early free"
