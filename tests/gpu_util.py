"""Helpers for GPU parity tests: run cases through the C ABI."""
import ctypes

import numpy as np
import torch

from affon_b200 import _lib
from affon_b200.core import check

_DT = {"f32": _lib.F32, "bf16": _lib.BF16, "u32": _lib.U32}


class Ctx:
    def __init__(self, device=0):
        self.ptr = ctypes.c_void_p()
        check(_lib.lib().affon_b200_ctx_create(device, None, ctypes.byref(self.ptr)))
        self.device = torch.device("cuda", device)

    def close(self):
        _lib.lib().affon_b200_ctx_destroy(self.ptr)

    def qmm(self, desc, x, w, s, b, y, stream=None):
        L = _lib.lib()
        check(L.affon_b200_ctx_set_stream(self.ptr, stream if stream is not None else
                                          torch.cuda.current_stream(self.device).cuda_stream))
        sel = _lib.Selection()
        check(L.affon_b200_qmm_explain(self.ptr, ctypes.byref(desc), x, w, s, b, y, ctypes.byref(sel)),
              "affon_b200_qmm")
        return sel


def to_device(phys, device):
    a = np.ascontiguousarray(phys)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    elif a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).to(device)


def case_desc(case, y_dtype="f32", policy="backend_equivalent"):
    d = _lib.QmmDesc()
    d.struct_size = ctypes.sizeof(_lib.QmmDesc)
    d.bits = case.bits
    d.group_size = case.group_size
    d.x_dtype = _DT[case.x.dtype]
    d.param_dtype = _DT[case.s.dtype]
    d.y_dtype = _DT[y_dtype]
    d.numerical_policy = _lib.POLICY[policy]
    for name in "xwsb":
        op = getattr(case, name)
        setattr(d, name, _lib.View(op.shape[0], op.shape[1], op.row_stride, op.col_stride, op.byte_offset))
    M, N, _ = case.mnk
    d.y = _lib.View(M, N, N, 1, 0)
    return d


def run_case(ctx, case, y_dtype="f32"):
    """Run a golden Case (with its views) on the GPU; returns (y float64 [M,N], implementation id)."""
    M, N, _ = case.mnk
    bufs = [to_device(getattr(case, n).phys, ctx.device) for n in "xwsb"]
    y = torch.full((M, N), float("nan"), dtype=torch.float32 if y_dtype == "f32" else torch.bfloat16,
                   device=ctx.device)
    sel = ctx.qmm(case_desc(case, y_dtype), *[t.data_ptr() for t in bufs], y.data_ptr())
    torch.cuda.synchronize(ctx.device)
    return y.double().cpu().numpy(), sel.implementation_id.decode()


def dense_desc(M, N, K, bits, group=64, xd="bf16", pd="bf16", yd="f32", ldy=None):
    per = 32 // bits
    d = _lib.QmmDesc()
    d.struct_size = ctypes.sizeof(_lib.QmmDesc)
    d.bits, d.group_size = bits, group
    d.x_dtype, d.param_dtype, d.y_dtype = _DT[xd], _DT[pd], _DT[yd]
    d.x = _lib.View(M, K, K, 1, 0)
    d.w = _lib.View(N, K // per, K // per, 1, 0)
    d.s = _lib.View(N, K // group, K // group, 1, 0)
    d.b = _lib.View(N, K // group, K // group, 1, 0)
    d.y = _lib.View(M, N, ldy or N, 1, 0)
    return d


def f64_reference(data, rows=None):
    """float64 y = x . (codes*s + b)^T for the given weight rows of a
    synthetic.quantized_linear case, and sum |x||w| (the magnitude a rounding
    bound scales with)."""
    from affon_b200 import synthetic
    x = synthetic.bf16_to_f32(data["x"]).astype(np.float64)
    r = slice(None) if rows is None else rows
    g = data.get("group", 64)
    codes = data["codes"][r].astype(np.float64)
    s = np.repeat(synthetic.bf16_to_f32(data["s"][r]).astype(np.float64), g, axis=1)
    b = np.repeat(synthetic.bf16_to_f32(data["b"][r]).astype(np.float64), g, axis=1)
    w = codes * s + b
    return x @ w.T, np.abs(x) @ np.abs(w).T
