"""ctypes binding of the CPU oracle (oracle/qmm_ref.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker.  The product library in
affon_b200/ never imports this module.
"""
import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libaffon_oracle.so"
F32, BF16 = 0, 1
_DT = {"f32": F32, "bf16": BF16}

_lib = None


def build():
    """Compile the oracle with its Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        view = [vp, i64, i64, i64]
        L.affon_oracle_qmm_view_f32.argtypes = (view + [i32]) + view + view + (view + [i32]) + [vp, i64, i64, i64, i32, i64]
        L.affon_oracle_qmm_view_f32.restype = i32
        L.affon_oracle_qmm_view_f64.argtypes = L.affon_oracle_qmm_view_f32.argtypes
        L.affon_oracle_qmm_view_f64.restype = i32
        L.affon_oracle_qmm_dense_f32.argtypes = [vp, i32, vp, vp, vp, i32, vp, i64, i64, i64, i32, i64]
        L.affon_oracle_qmm_dense_f32.restype = i32
        L.affon_oracle_qmm_dense_f32_mt.argtypes = [vp, i32, vp, vp, vp, i32, vp, i64, i64, i64, i32, i64, i32]
        L.affon_oracle_qmm_dense_f32_mt.restype = i32
        L.affon_oracle_unpack.argtypes = [vp, i64, i64, i32, vp]
        L.affon_oracle_unpack.restype = i32
        sz = ctypes.c_size_t
        L.affon_oracle_compute_core_run_quantized_matmul_f32.argtypes = [vp, sz, vp, sz, vp, sz, vp, sz, vp, sz, sz, sz,
                                                                         sz, sz, sz]
        L.affon_oracle_compute_core_run_quantized_matmul_f32.restype = i32
        L.affon_oracle_f32_to_bf16.argtypes = [vp, vp, i64]
        L.affon_oracle_validate.argtypes = [i64, i64, i64, i32, i64]
        L.affon_oracle_validate.restype = i32
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def qmm_case(case, f64=False):
    """Run the oracle on a tests.golden_cases.Case (views honoured). Returns [M,N]."""
    M, N, K = case.mnk
    out = np.zeros((M, N), dtype=np.float64 if f64 else np.float32)
    args = []
    for op, with_dtype in ((case.x, True), (case.w, False), (case.s, False), (case.b, True)):
        args += [_ptr(op.phys), op.row_stride, op.col_stride, op.byte_offset]
        if with_dtype:
            args.append(_DT.get(op.dtype, 0))
    fn = lib().affon_oracle_qmm_view_f64 if f64 else lib().affon_oracle_qmm_view_f32
    rc = fn(*args, _ptr(out), M, N, K, case.bits, case.group_size)
    if rc:
        raise ValueError(f"oracle rejected shape (status {rc})")
    return out


def qmm_dense(x, x_dtype, w, s, b, p_dtype, M, N, K, bits, group, threads=1):
    """Dense oracle: x [M,K] (f32 array or bf16 bits), w u32 [N,K/P], s/b [N,K/group]."""
    y = np.zeros((M, N), dtype=np.float32)
    x, w, s, b = (np.ascontiguousarray(a) for a in (x, w, s, b))
    if threads > 1:
        rc = lib().affon_oracle_qmm_dense_f32_mt(_ptr(x), _DT[x_dtype], _ptr(w), _ptr(s), _ptr(b), _DT[p_dtype], _ptr(y),
                                                 M, N, K, bits, group, threads)
    else:
        rc = lib().affon_oracle_qmm_dense_f32(_ptr(x), _DT[x_dtype], _ptr(w), _ptr(s), _ptr(b), _DT[p_dtype], _ptr(y),
                                              M, N, K, bits, group)
    if rc:
        raise ValueError(f"oracle rejected shape (status {rc})")
    return y


def unpack(w, N, K, bits):
    codes = np.zeros((N, K), dtype=np.uint8)
    w = np.ascontiguousarray(w, dtype=np.uint32)
    if lib().affon_oracle_unpack(_ptr(w), N, K, bits, _ptr(codes)):
        raise ValueError("invalid unpack shape")
    return codes


def cyna_qmm_f32(activation, weights, scales, biases, output, rows, depth, columns, bits, group_size):
    """The reference C-ABI shape (compute_core_cyna.zig:29-45) on the oracle."""
    return lib().affon_oracle_compute_core_run_quantized_matmul_f32(
        _ptr(activation), activation.size, _ptr(weights), weights.size, _ptr(scales), scales.size, _ptr(biases),
        biases.size, _ptr(output), output.size, rows, depth, columns, bits, group_size)


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
