"""ctypes binding of libaffon_b200.so (include/affon_b200.h).

The shared library is built in-tree by affon_b200/csrc/Makefile.  Loading it
never falls back to anything: a missing or unloadable library raises.
"""
import ctypes
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libaffon_b200.so"
HEADER = HERE.parent / "include" / "affon_b200.h"

OK, INVALID_SHAPE, UNSUPPORTED, CUDA_ERROR, TIMEOUT, GUARD_MISMATCH, POLICY_REJECTED, INVALID_ARG, INVALID_DTYPE = range(9)
F32, BF16, U32, U64 = 0, 1, 2, 3
REDUCE_SUM, REDUCE_MAX = 0, 1
TP_ID_BYTES = 144
POLICY = {"backend_equivalent": 0, "exact_only": 1, "approximate": 2}
NUMERICS = {0: "exact", 1: "reassociated", 2: "approximate"}

c_i64, c_i32, c_u32, c_vp, c_sz = ctypes.c_int64, ctypes.c_int32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t


class View(ctypes.Structure):
    _fields_ = [("rows", c_i64), ("cols", c_i64), ("row_stride", c_i64), ("col_stride", c_i64), ("byte_offset", c_i64)]


class QmmDesc(ctypes.Structure):
    _fields_ = [("struct_size", c_u32), ("bits", c_i32), ("group_size", c_i64), ("x_dtype", c_i32),
                ("param_dtype", c_i32), ("y_dtype", c_i32), ("numerical_policy", c_i32), ("dense_inputs", c_i32),
                ("reserved", c_i32), ("x", View), ("w", View), ("s", View), ("b", View), ("y", View)]


class QmvFusion(ctypes.Structure):
    _fields_ = [("struct_size", c_u32), ("x_mode", c_i32), ("epilogue", c_i32), ("act_pair_order", c_i32),
                ("h_out", c_vp), ("ld_h_out", c_i64), ("ss_out", c_vp), ("act", c_vp), ("ld_act", c_i64),
                ("amax", c_vp), ("index_offset", c_i64), ("row_ss", c_vp), ("ss_tiles", c_i32),
                ("eps", ctypes.c_float), ("next_gamma", c_vp), ("next_x", c_vp), ("ld_next_x", c_i64),
                ("next_pair_order", c_i32), ("exchange_region", c_i32)]


class AttnDesc(ctypes.Structure):
    _fields_ = [("struct_size", c_u32), ("batch", c_i32), ("q_heads", c_i32), ("kv_heads", c_i32),
                ("head_dim", c_i32), ("capacity", c_i32), ("scale", ctypes.c_float), ("q_offset", c_i32),
                ("k_offset", c_i32), ("v_offset", c_i32), ("out_pair_order", c_i32), ("ld_qkv", c_i64),
                ("ld_out", c_i64)]


EPI_STORE, EPI_RESID, EPI_SILU_MUL, EPI_ARGMAX, EPI_RESID_AR = 0, 1, 2, 3, 4
SS_WIDTH = 32      # row width of the per-16-column sums of squares ([cols/16][SS_WIDTH] f32)
MAX_QMV_ROWS = 32  # activation rows the decode qmv takes in one pass


class Selection(ctypes.Structure):
    _fields_ = [("implementation_id", ctypes.c_char * 64), ("implementation_version", c_i32),
                ("numerical_class", c_i32), ("splits", c_i32), ("reserved", c_i32), ("reason", ctypes.c_char * 256)]


# Every function include/affon_b200.h declares, with its ctypes signature.
SIGNATURES = {
    "affon_b200_abi_version": ([], c_i32),
    "affon_b200_last_error": ([], ctypes.c_char_p),
    "affon_b200_ctx_create": ([c_i32, c_vp, ctypes.POINTER(c_vp)], c_i32),
    "affon_b200_ctx_destroy": ([c_vp], c_i32),
    "affon_b200_ctx_set_stream": ([c_vp, c_vp], c_i32),
    "affon_b200_ctx_device": ([c_vp], c_i32),
    "affon_b200_ctx_reserve_workspace": ([c_vp, c_sz], c_i32),
    "affon_b200_ctx_synchronize": ([c_vp], c_i32),
    "affon_b200_validate": ([ctypes.POINTER(QmmDesc)], c_i32),
    "affon_b200_select": ([ctypes.POINTER(QmmDesc), ctypes.POINTER(Selection)], c_i32),
    "affon_b200_qmm": ([c_vp, ctypes.POINTER(QmmDesc), c_vp, c_vp, c_vp, c_vp, c_vp], c_i32),
    "affon_b200_qmm_explain": ([c_vp, ctypes.POINTER(QmmDesc), c_vp, c_vp, c_vp, c_vp, c_vp,
                                ctypes.POINTER(Selection)], c_i32),
    "affon_b200_qmm_host": ([c_vp, ctypes.POINTER(QmmDesc), c_vp, c_vp, c_vp, c_vp, c_vp], c_i32),
    "affon_b200_compute_core_run_quantized_matmul_f32": ([c_vp, c_sz, c_vp, c_sz, c_vp, c_sz, c_vp, c_sz, c_vp, c_sz,
                                                          c_sz, c_sz, c_sz, c_sz, c_sz], c_i32),
    "affon_b200_qmv_noalloc": ([ctypes.POINTER(QmmDesc), c_vp, c_vp, c_vp, c_vp, c_vp, c_vp], c_i32),
    "affon_b200_qmv_noalloc_status": ([c_vp, ctypes.POINTER(c_u32)], c_i32),
    "affon_b200_ctx_set_overlap": ([c_vp, c_i32], c_i32),
    "affon_b200_debug_set_combine_wait": ([ctypes.c_uint64, c_u32], c_i32),
    "affon_b200_debug_set_slice_rows": ([ctypes.c_int64], c_i32),
    "affon_b200_qmv_fused": ([c_vp, ctypes.POINTER(QmmDesc), c_vp, c_vp, c_vp, c_vp, c_vp,
                              ctypes.POINTER(QmvFusion)], c_i32),
    "affon_b200_qmv_prep": ([c_vp, c_i32, c_vp, c_i64, c_vp, c_i32, c_vp, ctypes.c_float, c_i32, c_i32, c_i32, c_vp,
                             c_i64], c_i32),
    "affon_b200_resid_norm": ([c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, ctypes.c_float, c_i32, c_i32, c_i32, c_vp,
                               c_i64], c_i32),
    "affon_b200_tp_unique_id": ([c_vp], c_i32),
    "affon_b200_tp_id_check": ([c_vp], c_i32),
    "affon_b200_tp_init": ([c_vp, c_i32, c_i32, c_vp, ctypes.c_double], c_i32),
    "affon_b200_tp_exchange_reserve": ([c_vp, c_i32, c_i64], c_i32),
    "affon_b200_tp_rank": ([c_vp], c_i32),
    "affon_b200_tp_world": ([c_vp], c_i32),
    "affon_b200_tp_allreduce": ([c_vp, c_vp, c_sz, c_i32, c_i32], c_i32),
    "affon_b200_tp_allreduce_bf16": ([c_vp, c_vp, c_sz], c_i32),
    "affon_b200_tp_synchronize": ([c_vp, ctypes.c_double], c_i32),
    "affon_b200_tp_abort": ([c_vp], c_i32),
    "affon_b200_tp_destroy": ([c_vp], c_i32),
    "affon_b200_decode_attention": ([c_vp, ctypes.POINTER(AttnDesc), c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp], c_i32),
    "affon_b200_embed": ([c_vp, c_vp, c_i64, c_i64, c_vp, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i32],
                         c_i32),
    "affon_b200_argmax_finalize": ([c_vp, c_vp, c_i32, c_vp, c_vp, c_i32, c_vp, c_vp], c_i32),
    "affon_b200_launch_count": ([], ctypes.c_uint64),
}

_lib = None


def lib():
    """Load the native library (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `make -C affon_b200/csrc` (or __graft_entry__.build())")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def last_error():
    msg = lib().affon_b200_last_error()
    return msg.decode() if msg else ""
