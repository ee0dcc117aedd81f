"""Bounded waits that run out are reported, and the context stays usable.

The reference's contract for a failed run is that the executable stays
reusable (test/e2e/program/execution/recovery.test.ts:8-23).  Here the failure
is made on purpose without faulting anything: a test hook makes the decode
qmv's split-K combine wait for one more contributor than exists, with a short
limit, so every shared block's wait gives up after that limit.  The kernel
then records TIMEOUT in its status word and finishes; the host must report it,
and the next normal launch must be correct (the block counters are reset).
"""
import ctypes

import numpy as np
import pytest
import torch

from affon_b200 import _lib, synthetic
from gpu_util import Ctx, dense_desc

pytestmark = pytest.mark.gpu

LIMIT_NS = 20_000_000  # 20 ms


@pytest.fixture(scope="module")
def ctx():
    c = Ctx(0)
    yield c
    c.close()


def _operands(M, N, K, bits, dev, seed):
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=seed)
    return {k: torch.from_numpy(np.ascontiguousarray(data[k]).view(np.int32 if data[k].dtype == np.uint32 else
                                                                    np.int16)).to(dev) for k in ("x", "w", "s", "b")}


@pytest.fixture
def combine_hook():
    L = _lib.lib()
    L.affon_b200_debug_set_combine_wait(LIMIT_NS, 1)
    try:
        yield
    finally:
        L.affon_b200_debug_set_combine_wait(0, 0)


def test_combine_timeout_is_reported_and_next_launch_is_correct(ctx):
    L = _lib.lib()
    M, N, K = 4, 16384, 4096                # split-K: blocks shared by several CTAs
    bufs = _operands(M, N, K, 4, ctx.device, seed=31)
    ptrs = [bufs[k].data_ptr() for k in ("x", "w", "s", "b")]
    d = dense_desc(M, N, K, 4)
    y_ref = torch.empty((M, N), dtype=torch.float32, device=ctx.device)
    sel = ctx.qmm(d, *ptrs, y_ref.data_ptr())
    assert sel.splits > 1, sel.reason
    assert L.affon_b200_ctx_synchronize(ctx.ptr) == _lib.OK

    L.affon_b200_debug_set_combine_wait(LIMIT_NS, 1)
    try:
        y = torch.empty_like(y_ref)
        ctx.qmm(d, *ptrs, y.data_ptr())
        assert L.affon_b200_ctx_synchronize(ctx.ptr) == _lib.TIMEOUT
        assert "bounded wait" in _lib.last_error()
    finally:
        L.affon_b200_debug_set_combine_wait(0, 0)
    assert L.affon_b200_ctx_synchronize(ctx.ptr) == _lib.OK    # reported once, then cleared

    for _ in range(2):                       # the counters were reset: normal launches are exact again
        y = torch.full_like(y_ref, float("nan"))
        ctx.qmm(d, *ptrs, y.data_ptr())
        assert L.affon_b200_ctx_synchronize(ctx.ptr) == _lib.OK
        assert torch.equal(y, y_ref)


def test_noalloc_status_reports_a_timeout(ctx, combine_hook):
    L = _lib.lib()
    M, N, K = 8, 16384, 4096                # split-K: blocks shared by several CTAs
    bufs = _operands(M, N, K, 4, ctx.device, seed=32)
    ptrs = [bufs[k].data_ptr() for k in ("x", "w", "s", "b")]
    d = dense_desc(M, N, K, 4)
    stream = torch.cuda.current_stream(ctx.device).cuda_stream
    y = torch.empty((M, N), dtype=torch.float32, device=ctx.device)
    assert L.affon_b200_qmv_noalloc(ctypes.byref(d), *ptrs, y.data_ptr(), stream) == _lib.OK
    status = ctypes.c_uint32(0)
    assert L.affon_b200_qmv_noalloc_status(stream, ctypes.byref(status)) == _lib.TIMEOUT
    assert status.value == 4
    L.affon_b200_debug_set_combine_wait(0, 0)
    y_ref = torch.empty_like(y)
    ctx.qmm(d, *ptrs, y_ref.data_ptr())
    assert L.affon_b200_qmv_noalloc(ctypes.byref(d), *ptrs, y.data_ptr(), stream) == _lib.OK
    assert L.affon_b200_qmv_noalloc_status(stream, ctypes.byref(status)) == _lib.OK
    assert status.value == 0
    assert torch.equal(y, y_ref)
