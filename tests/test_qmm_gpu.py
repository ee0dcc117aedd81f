"""GPU parity of quantized_matmul through the C ABI against the CPU oracle and
the reference's golden vectors (run with -m gpu on a B200)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from affon_b200 import _lib, synthetic
from golden_cases import bf16_tolerance, f32_tolerance, fixture_cells, general_cases, kat_cases
from gpu_util import Ctx, dense_desc, run_case

pytestmark = pytest.mark.gpu

BASELINE_NK = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]


@pytest.fixture(scope="module")
def ctx():
    c = Ctx(0)
    yield c
    c.close()


def test_kats_exact(ctx):
    """quantized-matmul.test.ts asserts toEqual; every KAT must be bit-exact on the GPU too."""
    for case in kat_cases():
        y, impl = run_case(ctx, case)
        assert impl.startswith("cuda_quantized_matmul."), impl
        np.testing.assert_array_equal(y, case.expected, err_msg=f"{case.name} via {impl}")


def test_fixture_cells(ctx):
    """268 CUDA catalog cells (quantized_fixture.py) within the f32 tolerance, and
    bit-identical to the oracle when the generic kernel ran."""
    for case in fixture_cells():
        y, impl = run_case(ctx, case)
        assert np.abs(y - case.expected).max() <= f32_tolerance(case.expected), case.name
        if impl.endswith("sm100_generic"):
            np.testing.assert_array_equal(y.astype(np.float32), oracle.qmm_case(case), err_msg=case.name)


def test_general_cases(ctx):
    """192 seeded cases of check-cuda-quantized-general.py, every element within
    2e-6*max(1,peak), operator and composed (y+y) form."""
    for case in general_cases():
        y, impl = run_case(ctx, case)
        assert np.isfinite(y).all(), case.name
        for factor in (1, 2):
            wanted = case.expected * factor
            assert np.abs(y * factor - wanted).max() <= f32_tolerance(wanted), (case.name, impl)


def _upload(ctx, data):
    dev = ctx.device
    return {k: torch.from_numpy(np.ascontiguousarray(data[k]).view(np.int32 if data[k].dtype == np.uint32 else
                                                                       np.int16)).to(dev)
            for k in ("x", "w", "s", "b")}


def _run_dense(ctx, data, bufs, yd="f32", M=None):
    M = M or data["M"]
    N, K, bits = data["N"], data["K"], data["bits"]
    y = torch.full((M, N), float("nan"), dtype=torch.float32 if yd == "f32" else torch.bfloat16, device=ctx.device)
    d = dense_desc(M, N, K, bits, yd=yd)
    sel = ctx.qmm(d, bufs["x"].data_ptr(), bufs["w"].data_ptr(), bufs["s"].data_ptr(), bufs["b"].data_ptr(),
                  y.data_ptr())
    torch.cuda.synchronize()
    return y, sel


@pytest.mark.parametrize("bits", [4, 8])
def test_codes_bit_exact_through_kernel(ctx, bits):
    """Unpacked codes are bit-exact: one-hot activations with scale 1 and bias 0
    make y[m, n] = q[n, k_m] exactly, for every row n of a full-size weight."""
    M, N, K = 16, 4096, 4096
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=7)
    ks = np.random.default_rng(1).choice(K, size=M, replace=False)
    x = np.zeros((M, K), dtype=np.float32)
    x[np.arange(M), ks] = 1.0
    data["x"] = synthetic.bf16_round_bits(x)
    data["s"] = synthetic.bf16_round_bits(np.ones_like(synthetic.bf16_to_f32(data["s"])))
    data["b"] = np.zeros_like(data["b"])
    y, sel = _run_dense(ctx, data, _upload(ctx, data))
    assert "qmv" in sel.implementation_id.decode()
    codes = oracle.unpack(data["w"], N, K, bits)
    np.testing.assert_array_equal(y.cpu().numpy(), codes[:, ks].T.astype(np.float32))


def _oracle_rows(data, rows, threads):
    """Oracle on a subset of weight rows (all M activation rows)."""
    sub = {k: data[k][rows] for k in ("w", "s", "b")}
    return oracle.qmm_dense(data["x"], "bf16", sub["w"], sub["s"], sub["b"], "bf16", data["M"], len(rows), data["K"],
                            data["bits"], 64, threads=threads), \
        _oracle_rows_f64(data, rows)


def _oracle_rows_f64(data, rows):
    x = synthetic.bf16_to_f32(data["x"]).astype(np.float64)
    codes = data["codes"][rows].astype(np.float64)
    s = np.repeat(synthetic.bf16_to_f32(data["s"][rows]).astype(np.float64), 64, axis=1)
    b = np.repeat(synthetic.bf16_to_f32(data["b"][rows]).astype(np.float64), 64, axis=1)
    return x @ (codes * s + b).T


@pytest.mark.parametrize("N,K", BASELINE_NK)
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [1, 4, 8, 16, 32])
def test_qmv_baseline_shapes(ctx, M, bits, N, K):
    """BASELINE decode sweep (config 2) on seeded inputs vs the oracle.

    f32 result: within 1e-5 * max(1, peak) of the float64 contraction (the
    reference's 2e-6 gate is for K <= 500; at K = 4096..14336 two f32
    summation orders alone differ by more).  bf16 result: max relative error
    <= 2e-2 against the f32 oracle (BASELINE parity gate)."""
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=0)
    bufs = _upload(ctx, data)
    y32, sel = _run_dense(ctx, data, bufs, "f32")
    assert sel.implementation_id.decode() == f"cuda_quantized_matmul.sm100_qmv_b{bits}_g64"
    y16, _ = _run_dense(ctx, data, bufs, "bf16")
    rows = np.arange(N) if N <= 4096 else np.linspace(0, N - 1, 2048).astype(np.int64)
    ref32, ref64 = _oracle_rows(data, rows, threads=oracle.cpu_threads())
    g32 = y32.cpu().numpy()[:, rows].astype(np.float64)
    g16 = y16.float().cpu().numpy()[:, rows].astype(np.float64)
    peak = max(1.0, np.abs(ref64).max())
    assert np.abs(g32 - ref64).max() <= 1e-5 * peak
    assert np.abs(ref32 - ref64).max() <= 1e-5 * peak  # the oracle obeys the same bound
    assert np.abs(g16 - ref32).max() / peak <= 2e-2


def test_split_k_is_deterministic(ctx):
    # N = 16384 is past the warp-split plan (three 16-row tiles per SM), and
    # so is K = 14336: blocks shared by several CTAs, combined across them.
    data = synthetic.quantized_linear(16, 16384, 14336, bits=4, seed=3)
    bufs = _upload(ctx, data)
    y1, sel = _run_dense(ctx, data, bufs)
    assert sel.splits > 1
    y2, _ = _run_dense(ctx, data, bufs)
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("M,N,K,bits,rows", [(16, 4096, 4096, 4, 32), (16, 6144, 4096, 4, 48),
                                              (16, 4096, 7168, 4, 32), (8, 1024, 4096, 8, 16),
                                              (1, 4096, 2048, 4, 32), (13, 4008, 3584, 8, 32),
                                              (5, 7000, 2048, 4, 48)])
def test_qmv_warp_split_blocks(ctx, M, N, K, bits, rows):
    """N up to three 16-row tiles per SM and K up to 32 stages (the
    decoder's QKV and O shapes, the down projection's tensor-parallel shard)
    takes the warp-split plan: one whole-K block per CTA, K split over the
    CTA's warps and added in a fixed order (no combine across CTAs).  Every
    row (including a partial last block) within 1e-5 of float64, and the same
    bits twice."""
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=23)
    bufs = _upload(ctx, data)
    y1, sel = _run_dense(ctx, data, bufs)
    assert f"{rows}-row whole-K blocks" in sel.reason.decode(), sel.reason
    assert sel.splits == 1
    y2, _ = _run_dense(ctx, data, bufs)
    assert torch.equal(y1, y2)
    ref = _oracle_rows_f64(data, np.arange(N))
    assert np.abs(y1.cpu().numpy() - ref).max() <= 1e-5 * max(1, np.abs(ref).max())


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [12, 16])
def test_qmv_whole_k_blocks(ctx, M, bits):
    """The gate/up shape (N = 28672) takes the data-parallel plan: 208-row
    blocks, each streamed over the whole K by one CTA (no split-K combine).
    Sampled rows (including the last, partial block) within 1e-5 of float64,
    and the same bits twice."""
    N, K = 28672, 4096
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=21)
    bufs = _upload(ctx, data)
    y1, sel = _run_dense(ctx, data, bufs)
    assert "over 138 CTAs" in sel.reason.decode(), sel.reason
    y2, _ = _run_dense(ctx, data, bufs)
    assert torch.equal(y1, y2)
    rows = np.concatenate([np.linspace(0, N - 209, 500).astype(np.int64), np.arange(N - 208, N)])
    ref = _oracle_rows_f64(data, rows)
    assert np.abs(y1.cpu().numpy()[:, rows] - ref).max() <= 1e-5 * max(1, np.abs(ref).max())


@pytest.mark.parametrize("M", [17, 33, 63, 64, 100])
def test_qmv_multi_pass(ctx, M):
    """M > 32 below 64 runs qmv passes over 32-row slices; from 64 rows the
    reassociated tcgen05 qmm takes over; both within the same gate."""
    data = synthetic.quantized_linear(M, 1024, 4096, bits=4, seed=5)
    y, sel = _run_dense(ctx, data, _upload(ctx, data))
    assert ("qmv" if M < 64 else "qmm_tcgen05_exact") in sel.implementation_id.decode()
    ref = _oracle_rows_f64(data, np.arange(1024))
    assert np.abs(y.cpu().numpy() - ref).max() <= 1e-5 * max(1, np.abs(ref).max())


@pytest.mark.parametrize("bits,K", [(4, 1792), (4, 3584), (8, 1920)])
def test_qmv_k_not_multiple_of_512_with_padded_parameter_rows(ctx, bits, K):
    """Tensor-parallel shards split K at 64-group boundaries (e.g. 14336/8 =
    1792): K need only be a multiple of one 128-byte packed stage, with the
    scale and bias rows padded to a 16-byte stride (a strided view)."""
    M, N = 16, 2048
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=12)
    bufs = _upload(ctx, data)
    G = K // 64
    Gp = (G + 7) // 8 * 8
    pad = {}
    for k in ("s", "b"):
        t = torch.zeros((N, Gp), dtype=torch.int16, device=ctx.device)
        t[:, :G] = bufs[k]
        pad[k] = t
    d = dense_desc(M, N, K, bits)
    d.s = _lib.View(N, G, Gp, 1, 0)
    d.b = _lib.View(N, G, Gp, 1, 0)
    y = torch.empty((M, N), dtype=torch.float32, device=ctx.device)
    sel = ctx.qmm(d, bufs["x"].data_ptr(), bufs["w"].data_ptr(), pad["s"].data_ptr(), pad["b"].data_ptr(),
                  y.data_ptr())
    torch.cuda.synchronize()
    assert "qmv" in sel.implementation_id.decode(), sel.reason
    ref = _oracle_rows_f64(data, np.arange(N))
    assert np.abs(y.cpu().numpy() - ref).max() <= 1e-5 * max(1, np.abs(ref).max())


def test_host_entry_matches_device_entry(ctx):
    data = synthetic.quantized_linear(4, 4096, 4096, bits=4, seed=11)
    y_dev, _ = _run_dense(ctx, data, _upload(ctx, data))
    d = dense_desc(4, 4096, 4096, 4)
    y = np.full((4, 4096), np.nan, dtype=np.float32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    rc = _lib.lib().affon_b200_qmm_host(ctx.ptr, ctypes.byref(d), p(data["x"]), p(data["w"]), p(data["s"]),
                                        p(data["b"]), p(y))
    assert rc == 0, _lib.last_error()
    np.testing.assert_array_equal(y, y_dev.cpu().numpy())


def test_cyna_signature_known_answer():
    """compute_core_cyna_smoke.zig:970-984 through the GPU entry with the same signature."""
    act = np.array([1, 2, 3, 4, 5, 6, 7, 8, 2, 3, 4, 5, 6, 7, 8, 9], dtype=np.float32)
    w = np.array([0x01010101, 0x01010101, 0x02020202, 0x02020202, 0x03030303, 0x03030303], dtype=np.uint32)
    s, b = np.ones(6, dtype=np.float32), np.zeros(6, dtype=np.float32)
    out = np.full(6, -1, dtype=np.float32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    f = _lib.lib().affon_b200_compute_core_run_quantized_matmul_f32
    assert f(p(act), 16, p(w), 6, p(s), 6, p(b), 6, p(out), 6, 2, 8, 3, 8, 4) == 0
    np.testing.assert_array_equal(out, [36, 72, 108, 44, 88, 132])
    out[:] = -1
    assert f(p(act), 16, p(w), 6, p(s), 6, p(b), 6, p(out), 6, 2, 8, 3, 3, 4) == 1
    assert (out == -1).all()


def test_qmv_strided_activation_rows(ctx):
    """x rows at a stride larger than K (a sliced view) keep the fast path."""
    M, N, K = 8, 4096, 4096
    data = synthetic.quantized_linear(M, N, K, bits=4, seed=2)
    bufs = _upload(ctx, data)
    wide = torch.zeros((M, K + 64), dtype=torch.int16, device=ctx.device)
    wide[:, 32:32 + K] = bufs["x"]
    d = dense_desc(M, N, K, 4)
    d.x = _lib.View(M, K, K + 64, 1, 64)
    y = torch.empty((M, N), dtype=torch.float32, device=ctx.device)
    sel = ctx.qmm(d, wide.data_ptr(), bufs["w"].data_ptr(), bufs["s"].data_ptr(), bufs["b"].data_ptr(), y.data_ptr())
    torch.cuda.synchronize()
    assert "qmv" in sel.implementation_id.decode()
    y_ref, _ = _run_dense(ctx, data, bufs)
    assert torch.equal(y, y_ref)
