"""Prefill qmm with reassociated numerics on tcgen05 (the default
`backend_equivalent` policy, M >= 64) through the C ABI, against the CPU
oracle and float64.

The reference's contract for this path: f32 result, weights never rounded,
class `reassociated` (docs/core/quantized-inference.md:57,119-121,175-177);
its partial-tile cases reach M = 128 (test/e2e/program/operations/
quantized-matmul.test.ts:123-148), BASELINE config 3 reaches M = 8192.
"""
import numpy as np
import pytest
import torch

import oracle
from affon_b200 import _lib, synthetic
from gpu_util import Ctx, dense_desc, f64_reference

pytestmark = pytest.mark.gpu

EXACT = "cuda_quantized_matmul.sm100_qmm_tcgen05_exact_b{}_g64"


@pytest.fixture(scope="module")
def ctx():
    c = Ctx(0)
    yield c
    c.close()


def _run(ctx, data, yd="f32", policy="backend_equivalent"):
    M, N, K, bits = data["M"], data["N"], data["K"], data["bits"]
    dev = ctx.device
    up = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int32 if a.dtype == np.uint32 else np.int16)).to(dev)
    x, w, s, b = (up(data[k]) for k in ("x", "w", "s", "b"))
    y = torch.full((M, N), float("nan"), dtype=torch.float32 if yd == "f32" else torch.bfloat16, device=dev)
    d = dense_desc(M, N, K, bits, yd=yd)
    d.numerical_policy = _lib.POLICY[policy]
    sel = ctx.qmm(d, x.data_ptr(), w.data_ptr(), s.data_ptr(), b.data_ptr(), y.data_ptr())
    assert _lib.lib().affon_b200_ctx_synchronize(ctx.ptr) == 0, _lib.last_error()
    return y.float().cpu().numpy().astype(np.float64), sel.implementation_id.decode()


def _exact_data(M, N, K, bits, seed):
    """Small-integer activations and power-of-two scales with bias
    -2^(bits-1)*s: every product, group sum and total is exact in f32, so the
    result is exactly the oracle's whatever the summation order."""
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=seed)
    rng = np.random.default_rng(seed + 100)
    data["x"] = synthetic.bf16_round_bits(rng.integers(-3, 4, size=(M, K)).astype(np.float32))
    s = (2.0 ** rng.integers(-6, -2, size=data["s"].shape)).astype(np.float32)
    data["s"] = synthetic.bf16_round_bits(s)
    data["b"] = synthetic.bf16_round_bits(-(1 << (bits - 1)) * s)
    return data


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,N,K", [(64, 128, 64), (100, 1000, 576), (300, 200, 960), (256, 384, 1024),
                                   (700, 4096, 1024)])
def test_exact_when_every_sum_is_exact(ctx, bits, M, N, K):
    """Bit-equal to the oracle when all sums are exact: checks the swizzled
    operand layouts, the per-group TMEM double buffer, the bias stages (K = 64
    has one group, 576 and 960 leave zero-padded bias columns), the ragged M
    and N edges and the store mapping."""
    data = _exact_data(M, N, K, bits, seed=5)
    y, impl = _run(ctx, data)
    assert impl == EXACT.format(bits), impl
    ref = oracle.qmm_dense(data["x"], "bf16", data["w"], data["s"], data["b"], "bf16", M, N, K, bits, 64,
                           threads=oracle.cpu_threads())
    np.testing.assert_array_equal(y, ref.astype(np.float64))


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (2048, 1024, 4096), (512, 14336, 4096), (512, 4096, 14336)])
def test_exact_baseline_distributions(ctx, bits, M, N, K):
    """BASELINE config 3 distributions with the reference's default f32
    result: within 1e-5 of the largest |y| of the float64 contraction (the
    qmv's reassociated gate), and a bf16 result within 2e-2."""
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=0)
    rows = np.arange(N) if N <= 1024 else np.linspace(0, N - 1, 1024).astype(np.int64)
    ref, _ = f64_reference(data, rows)
    peak = max(1.0, np.abs(ref).max())
    y32, impl = _run(ctx, data, "f32")
    assert impl == EXACT.format(bits), impl
    assert np.abs(y32[:, rows] - ref).max() <= 1e-5 * peak
    y16, impl = _run(ctx, data, "bf16")
    assert impl == EXACT.format(bits), impl
    assert np.abs(y16[:, rows] - ref).max() / peak <= 2e-2


def test_exact_matches_the_f32_oracle(ctx):
    """Against the oracle itself (fma(s, q, b) per weight, f32 sums in K
    order) on a case it finishes in seconds: both within the same 1e-5 gate
    of float64."""
    M, N, K, bits = 256, 512, 4096, 4
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=8)
    y, impl = _run(ctx, data)
    assert impl == EXACT.format(bits)
    ref32 = oracle.qmm_dense(data["x"], "bf16", data["w"], data["s"], data["b"], "bf16", M, N, K, bits, 64,
                             threads=oracle.cpu_threads()).astype(np.float64)
    ref64, _ = f64_reference(data)
    peak = max(1.0, np.abs(ref64).max())
    assert np.abs(y - ref64).max() <= 1e-5 * peak
    assert np.abs(ref32 - ref64).max() <= 1e-5 * peak
    assert np.abs(y - ref32).max() <= 2e-5 * peak


@pytest.mark.parametrize("N", [4096, 14336])
def test_exact_m8192(ctx, N):
    """BASELINE config 3 at its largest M (8192 rows, 4-bit, K = 4096, f32
    result): 256 sampled weight rows against float64 at the 1e-5 gate, every
    output finite."""
    M, K = 8192, 4096
    data = synthetic.quantized_linear(M, N, K, bits=4, seed=3)
    y, impl = _run(ctx, data)
    assert impl == EXACT.format(4), impl
    assert np.isfinite(y).all()
    rows = np.linspace(0, N - 1, 256).astype(np.int64)
    ref, _ = f64_reference(data, rows)
    assert np.abs(y[:, rows] - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_exact_row_slices_match_one_pass(ctx):
    """Large M is processed in row slices whose group sums fit the workspace;
    a 256-row cap forces four slices of a 1000-row problem, which must give
    the same bits as one pass."""
    M, N, K = 1000, 768, 2048
    data = synthetic.quantized_linear(M, N, K, bits=4, seed=6)
    one, impl = _run(ctx, data)
    assert impl == EXACT.format(4)
    L = _lib.lib()
    assert L.affon_b200_debug_set_slice_rows(256) == 0
    try:
        sliced, _ = _run(ctx, data)
    finally:
        L.affon_b200_debug_set_slice_rows(0)
    np.testing.assert_array_equal(sliced, one)


@pytest.mark.parametrize("bits", [4, 8])
def test_exact_repeated_runs_are_identical(ctx, bits):
    """Pipeline-race guard: a shape with more tiles than SMs (and several
    tiles per CTA) run five times gives the same bits each time, within the
    gate of float64."""
    M, N, K = 512, 14336, 2048
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=2)
    rows = np.linspace(0, N - 1, 512).astype(np.int64)
    ref, _ = f64_reference(data, rows)
    first = None
    for _ in range(5):
        y, impl = _run(ctx, data)
        assert impl == EXACT.format(bits)
        assert np.abs(y[:, rows] - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())
        if first is None:
            first = y
        else:
            np.testing.assert_array_equal(y, first)
