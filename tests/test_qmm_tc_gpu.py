"""Prefill qmm on tcgen05 with bf16-rounded decoded weights (the
`approximate` policy, M >= 64) through the C ABI against the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle
from affon_b200 import _lib, synthetic
from gpu_util import Ctx, dense_desc, f64_reference as _f64

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = Ctx(0)
    yield c
    c.close()


APPROX = "cuda_quantized_matmul.sm100_qmm_tcgen05_b{}_g64"


def _run(ctx, data, yd="bf16", policy="approximate"):
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


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,N,K", [(64, 128, 512), (100, 1000, 512), (256, 384, 4096), (700, 4096, 1024)])
def test_qmm_tc_exact_when_weights_are_bf16_exact(ctx, bits, M, N, K):
    """Power-of-two scales and bias -2^(bits-1)*s make every decoded weight exact
    in bf16, and small-integer activations make all f32 sums exact: the tensor
    -core result must then equal the oracle bit for bit (checks the swizzled
    operand layouts, TMEM addressing and the epilogue mapping)."""
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=4)
    rng = np.random.default_rng(9)
    x = rng.integers(-3, 4, size=(M, K)).astype(np.float32)
    data["x"] = synthetic.bf16_round_bits(x)
    s = (2.0 ** rng.integers(-6, -2, size=data["s"].shape)).astype(np.float32)
    data["s"] = synthetic.bf16_round_bits(s)
    data["b"] = synthetic.bf16_round_bits(-(1 << (bits - 1)) * s)
    y, impl = _run(ctx, data, "f32", "approximate")
    assert impl == APPROX.format(bits), impl
    ref = oracle.qmm_dense(data["x"], "bf16", data["w"], data["s"], data["b"], "bf16", M, N, K, bits, 64,
                           threads=oracle.cpu_threads())
    np.testing.assert_array_equal(y, ref.astype(np.float64))


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (2048, 1024, 4096), (512, 14336, 4096), (512, 4096, 14336)])
def test_qmm_tc_baseline_distributions(ctx, bits, M, N, K):
    """BASELINE config 3 distributions.  bf16 result: max relative error
    <= 2e-2 vs the f32 oracle.  f32 result (approximate policy): within the
    bound of one bf16 rounding per weight, 2^-8 * sum|x||w| per element."""
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=0)
    rows = np.arange(N) if N <= 1024 else np.linspace(0, N - 1, 1024).astype(np.int64)
    ref, mag = _f64(data, rows)
    y16, impl = _run(ctx, data, "bf16")
    assert impl == APPROX.format(bits), impl
    peak = max(1.0, np.abs(ref).max())
    assert np.abs(y16[:, rows] - ref).max() / peak <= 2e-2
    y32, impl = _run(ctx, data, "f32", "approximate")
    assert impl == APPROX.format(bits)
    assert (np.abs(y32[:, rows] - ref) <= 2.0 ** -8 * mag + 1e-6).all()


@pytest.mark.parametrize("N", [4096, 14336])
def test_qmm_tc_m8192(ctx, N):
    """BASELINE config 3 at its largest M (8192 rows, 4-bit, K=4096): 256
    sampled weight rows against float64, bf16 gate 2e-2, and every output
    finite."""
    M, K = 8192, 4096
    data = synthetic.quantized_linear(M, N, K, bits=4, seed=3)
    y, impl = _run(ctx, data, "bf16")
    assert impl == APPROX.format(4), impl
    assert np.isfinite(y).all()
    rows = np.linspace(0, N - 1, 256).astype(np.int64)
    ref, _ = _f64(data, rows)
    peak = max(1.0, np.abs(ref).max())
    assert np.abs(y[:, rows] - ref).max() / peak <= 2e-2


def test_qmm_tc_large_property(ctx):
    """BASELINE qmm shape M=2048, N=128256, K=4096 (4-bit): sampled rows and
    columns against float64, and a checksum of checksums over all outputs."""
    M, N, K = 2048, 128256, 4096
    data = synthetic.quantized_linear(M, N, K, bits=4, seed=1)
    y, impl = _run(ctx, data, "bf16")
    assert impl == APPROX.format(4), impl
    assert np.isfinite(y).all()
    rows = np.linspace(0, N - 1, 256).astype(np.int64)
    ref, _ = _f64(data, rows)
    peak = max(1.0, np.abs(ref).max())
    assert np.abs(y[:, rows] - ref).max() / peak <= 2e-2
    # column sums over all N for a few activation rows (linearity check)
    xs = synthetic.bf16_to_f32(data["x"][:4]).astype(np.float64)
    wsum = np.zeros(K)
    for r0 in range(0, N, 8192):
        codes = data["codes"][r0:r0 + 8192].astype(np.float64)
        s = np.repeat(synthetic.bf16_to_f32(data["s"][r0:r0 + 8192]).astype(np.float64), 64, axis=1)
        b = np.repeat(synthetic.bf16_to_f32(data["b"][r0:r0 + 8192]).astype(np.float64), 64, axis=1)
        wsum += (codes * s + b).sum(axis=0)
    want = xs @ wsum
    got = y[:4].sum(axis=1)
    assert np.abs(got - want).max() <= 2e-2 * np.abs(y[:4]).sum(axis=1).max() / np.sqrt(N) + 1e-3 * np.abs(want).max()


@pytest.mark.parametrize("bits", [4, 8])
def test_qmm_tc_repeated_runs_are_identical_and_bounded(ctx, bits):
    """Pipeline-race guard: a multi-tile shape (more tiles than SMs) run five
    times must give bit-identical results, every element within the
    single-rounding bound of the float64 contraction."""
    M, N, K = 512, 14336, 4096
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=2)
    ref, mag = _f64(data)
    first = None
    for _ in range(5):
        y, impl = _run(ctx, data, "f32", "approximate")
        assert impl == APPROX.format(bits), impl
        assert (np.abs(y - ref) <= 2.0 ** -8 * mag + 1e-6).all()
        if first is None:
            first = y
        else:
            np.testing.assert_array_equal(y, first)
