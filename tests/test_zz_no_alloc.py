"""The allocation-free decode qmv entry point, affon_b200_qmv_noalloc.

It exists for callers that may not let a library allocate device memory (a
runtime that owns every byte of the GPU in its own arena, a plugin host whose
allocator alone may call the driver): it needs no context and keeps its
scratch in a static device array.  These tests call it through the C ABI and
compare it with the regular context-based entry point on the same inputs,
twice in a row (the array keeps the previous call's contents, so the second
call checks that what must start at zero is cleared).  Both run the same
kernel with the same plan, so the results must be bit-identical; the status
word, read back with affon_b200_qmv_noalloc_status, must say that no bounded
wait gave up.  The file sorts last so that a run stopping at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from affon_b200 import _lib, synthetic
from gpu_util import Ctx, dense_desc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = Ctx(0)
    yield c
    c.close()


def _upload(data, dev):
    return {k: torch.from_numpy(np.ascontiguousarray(data[k]).view(np.int32 if data[k].dtype == np.uint32 else
                                                                    np.int16)).to(dev) for k in ("x", "w", "s", "b")}


@pytest.mark.parametrize("M,N,K,bits,yd", [(16, 4096, 4096, 4, "f32"), (1, 14336, 4096, 4, "bf16"),
                                           (8, 4096, 14336, 8, "f32"), (4, 28672, 4096, 4, "f32"),
                                           (32, 4096, 4096, 4, "f32")])
def test_noalloc_matches_context_entry_twice(ctx, M, N, K, bits, yd):
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=21)
    dev = ctx.device
    bufs = _upload(data, dev)
    ptrs = [bufs[k].data_ptr() for k in ("x", "w", "s", "b")]
    tdt = torch.float32 if yd == "f32" else torch.bfloat16
    d = dense_desc(M, N, K, bits, yd=yd)

    y_ref = torch.full((M, N), float("nan"), dtype=tdt, device=dev)
    sel = ctx.qmm(d, *ptrs, y_ref.data_ptr())
    assert "qmv" in sel.implementation_id.decode()
    torch.cuda.synchronize()
    assert torch.isfinite(y_ref.float()).all()

    stream = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=tdt, device=dev)
        rc = _lib.lib().affon_b200_qmv_noalloc(ctypes.byref(d), *ptrs, y.data_ptr(), stream)
        assert rc == 0, _lib.last_error()
        status = ctypes.c_uint32(7)
        assert _lib.lib().affon_b200_qmv_noalloc_status(stream, ctypes.byref(status)) == 0, _lib.last_error()
        assert status.value == 0
        assert torch.equal(y, y_ref)


def test_noalloc_rejects_shapes_beyond_its_scratch(ctx):
    """M*N beyond the static scratch is refused before any launch, with a message."""
    M, N, K = 16, 128256, 4096
    d = dense_desc(M, N, K, 4)
    y = torch.zeros((M, N), dtype=torch.float32, device=ctx.device)
    dummy = torch.zeros(16, dtype=torch.int32, device=ctx.device).data_ptr()
    rc = _lib.lib().affon_b200_qmv_noalloc(ctypes.byref(d), dummy, dummy, dummy, dummy, y.data_ptr(),
                                           torch.cuda.current_stream(ctx.device).cuda_stream)
    assert rc == _lib.UNSUPPORTED
    assert "scratch" in _lib.last_error()
    assert (y == 0).all()
