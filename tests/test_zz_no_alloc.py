"""lyth_b200_reduce_noalloc: the whole reduction for callers that cannot give the library device
memory (a host whose device memory belongs to its own arena, a runtime that embeds these kernels
and forbids them to allocate, a loop that cannot afford cudaMalloc's synchronisation). It keeps
its scratch in a fixed array of the library, so it must agree with the workspace entry point
bit for bit, call after call, and refuse sizes past the array's limit.

Collected last on purpose: a failure here leaves every other test already run."""
import ctypes as C

import numpy as np
import pytest
import torch

import lyth_b200 as lb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

MAX_N = 268435456  # LYTH_REDUCE_NOALLOC_MAX_N

_fn = lb.lib.lyth_b200_reduce_noalloc
_fn.restype = C.c_int
_fn.argtypes = [C.c_int, C.c_uint64, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]


def noalloc(op, x, y, out):
    stream = torch.cuda.current_stream().cuda_stream
    return _fn(op, x.numel(), x.data_ptr(), None if y is None else y.data_ptr(), out.data_ptr(), stream)


@pytest.mark.parametrize("op", ["sum", "dot", "max", "min"])
def test_two_calls_in_a_row_match_the_workspace_entry_point(cuda, op):
    code = {"sum": lb.SUM, "dot": lb.SUM, "max": lb.MAX, "min": lb.MIN}[op]
    for call, (seed, n) in enumerate([(91, 3_000_017), (92, 250_001)]):
        x = torch.from_numpy(orc.uniform(seed, n)).to(cuda)
        y = torch.from_numpy(orc.uniform(seed + 7, n)).to(cuda) if op == "dot" else None
        want = lb.reduce(code, x, y)
        got = torch.full((1,), float("nan"), device=cuda)
        assert noalloc(code, x, y, got) == lb.OK
        torch.cuda.synchronize()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert g.view(np.uint32)[0] == w.view(np.uint32)[0], (op, call, g, w)


def test_sizes_past_the_fixed_scratch_are_refused(cuda):
    x = torch.zeros(16, device=cuda)
    out = torch.full((1,), 7.0, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    rc = _fn(lb.SUM, MAX_N + 1, x.data_ptr(), None, out.data_ptr(), stream)
    assert rc == lb.E_UNSUPPORTED
    torch.cuda.synchronize()
    assert out.item() == 7.0  # nothing ran


def test_exact_fill_zero_and_a_small_call_after_a_large_one(cuda):
    # n = the limit fills all 16384 slots; n = 0 is the identity; a small n right after the
    # limit must not read any slot the large call left behind.
    stream = torch.cuda.current_stream().cuda_stream
    big = torch.from_numpy(orc.uniform(93, 1 << 20)).to(cuda).repeat(MAX_N >> 20)  # 1 GiB
    for n in (MAX_N, 0, 1000, 3):
        # n = 0: the sum's identity, +0.0 (the workspace entry point refuses an empty tensor's
        # null pointer, so the bits are compared with the identity directly)
        want = lb.reduce(lb.SUM, big[:n]).cpu().numpy() if n else np.zeros(1, np.float32)
        got = torch.full((1,), float("nan"), device=cuda)
        rc = _fn(lb.SUM, n, big.data_ptr(), None, got.data_ptr(), stream)
        assert rc == lb.OK
        torch.cuda.synchronize()
        assert got.cpu().numpy().view(np.uint32)[0] == want.view(np.uint32)[0], n
    del big
    torch.cuda.empty_cache()


def test_max_with_y_is_refused_and_runs_nothing(cuda):
    x = torch.ones(64, device=cuda)
    out = torch.full((1,), 7.0, device=cuda)
    for op in (lb.MAX, lb.MIN):
        assert noalloc(op, x, x, out) == lb.E_UNSUPPORTED
    torch.cuda.synchronize()
    assert out.item() == 7.0
