"""`affon:ops` surface for the quantized-linear path.

`quantized_matmul(input, packed, scales, biases, {bits, group_size})` follows
src/js/ops.ts:69-79: all four operands formal (a Program node is emitted) or
all four evaluated in one Session (an immediate one-node Program is compiled
and run, ops.ts:29-34); mixing raises.  Authoring validation restates
src/js/compute/program.ts:481-495 with the same messages; the native library
validates again before any launch.
"""
import ctypes

import torch

from . import _lib
from .core import (AffonError, FormalTensor, Tensor, TensorSpec, base_ptr, check, program, qmm_desc_from_specs,
                   view_of)


def _options(options, kwargs):
    opts = dict(options or {})
    opts.update(kwargs)
    return opts


def validate_quantized_matmul(specs, config):
    """program.ts:482-494 — returns the f32 result spec."""
    if not config or config.get("bits") not in (2, 4, 8):
        raise TypeError("quantized_matmul bits must be 2, 4, or 8")
    g = config.get("group_size")
    if not isinstance(g, int) or isinstance(g, bool) or g <= 0:
        raise TypeError("quantized_matmul group_size must be a positive integer")
    if len(specs) != 4 or any(len(s.shape) != 2 for s in specs):
        raise TypeError("quantized_matmul requires four rank-two tensors")
    x, w, s, b = specs
    if x.dtype not in ("f32", "bf16") or w.dtype != "u32" or s.dtype not in ("f32", "bf16") or b.dtype != s.dtype:
        raise TypeError("quantized_matmul requires f32/bf16 input, u32 weights, and matching f32/bf16 scales and biases")
    rows, inner = x.shape
    outputs = w.shape[0]
    per_word = 32 // config["bits"]
    if (not rows or not inner or not outputs or inner % per_word or inner % g or w.shape[1] != inner // per_word
            or s.shape[0] != outputs or s.shape[1] != inner // g or b.shape[0] != outputs or b.shape[1] != inner // g):
        raise TypeError("quantized_matmul packed or group dimensions do not match input features")
    out_dtype = config.get("out_dtype", "f32")
    if out_dtype not in ("f32", "bf16"):
        raise TypeError("quantized_matmul out_dtype must be f32 or bf16")
    return TensorSpec(out_dtype, (rows, outputs))


def _session_of(values):
    session = values[0].session
    if session.disposed:
        raise AffonError("invalid_arg", "Session has been disposed")
    if any(v.session is not session for v in values):
        raise TypeError("operation tensors must belong to the same Session")
    return session


def _immediate(name, values, author):
    """ops.ts:29-34: author a one-node Program over the evaluated operands and run it."""
    session = _session_of(values)
    specs = [TensorSpec(v.dtype, v.shape) for v in values]
    src = program(f"immediate_{name}", lambda p: author([p.argument(f"input_{i}", s) for i, s in enumerate(specs)]))
    return session.compile(src).run({f"input_{i}": v for i, v in enumerate(values)})


def quantized_matmul(input, packed, scales, biases, options=None, **kwargs):
    """Affine weight-only quantized matmul: y[m,n] = sum_k x[m,k]*(s[n,k/g]*q[n,k] + b[n,k/g]).

    `options` = {"bits": 2|4|8, "group_size": int}; the extension key
    "out_dtype" ("f32" default, "bf16") selects a bf16 result.
    """
    opts = _options(options, kwargs)
    values = [input, packed, scales, biases]
    formal = isinstance(input, FormalTensor)
    if any(isinstance(v, FormalTensor) != formal for v in values):
        raise TypeError("quantized_matmul cannot mix formal and evaluated tensors")
    if formal:
        spec = validate_quantized_matmul([v.spec for v in values], opts)
        return input.program.emit("quantized_matmul", values, spec, dict(opts))
    if any(not isinstance(v, Tensor) for v in values):
        raise TypeError("quantized_matmul operands must be tensors")
    return _immediate("quantized_matmul", values, lambda a: quantized_matmul(*a, opts))


def add(a, b):
    if isinstance(a, FormalTensor) != isinstance(b, FormalTensor):
        raise TypeError("add cannot mix formal and evaluated tensors")
    if isinstance(a, FormalTensor):
        # Same shapes, or b a vector over a's last axis (a layer bias).
        if a.spec.dtype != b.spec.dtype or (a.spec.shape != b.spec.shape and b.spec.shape != a.spec.shape[-1:]):
            raise TypeError("add requires matching shapes and dtypes")
        return a.program.emit("add", [a, b], a.spec)
    return _immediate("add", [a, b], lambda v: add(*v))


def transpose(x, axes):
    if list(axes) != [1, 0]:
        raise TypeError("transpose supports rank-two [1, 0] permutations")
    if isinstance(x, FormalTensor):
        r, c = x.spec.shape
        return x.program.emit("transpose", [x], TensorSpec(x.spec.dtype, (c, r)), {"axes": [1, 0]})
    return Tensor(x.session, x._live().t(), x.dtype)


def slice(x, ranges):
    rng = [(int(r.get("start", 0)), int(r["stop"]), int(r.get("step", 1))) for r in ranges]
    if isinstance(x, FormalTensor):
        shape = tuple(len(range(a, b, s)) for a, b, s in rng)
        return x.program.emit("slice", [x], TensorSpec(x.spec.dtype, shape),
                              {"ranges": [{"start": a, "stop": b, "step": s} for a, b, s in rng]})
    d = x._live()
    (a0, b0, s0), (a1, b1, s1) = rng
    return Tensor(x.session, d[a0:b0:s0, a1:b1:s1], x.dtype)


def _evaluate(session, op, args, options, compile_options):
    """Execute one Program node on evaluated operands."""
    if op == "quantized_matmul":
        return _run_qmm(session, args, options, compile_options)
    if op == "add":
        a, b = args
        return Tensor(session, a._live() + b._live(), a.dtype)
    if op == "transpose":
        return transpose(args[0], options["axes"])
    if op == "slice":
        return slice(args[0], options["ranges"])
    raise AffonError("unsupported_lowering", f"operation {op} has no lowering")


def _run_qmm(session, args, options, compile_options):
    x, w, s, b = args
    specs = [TensorSpec(t.dtype, t.shape) for t in args]
    out_spec = validate_quantized_matmul(specs, options)
    policy = _lib.POLICY[compile_options["numericalPolicy"]]
    desc = qmm_desc_from_specs(specs, options, policy, compile_options["denseInputs"], out_spec.dtype)
    for name, t in zip("xwsb", args):
        setattr(desc, name, view_of(t))
    # The runtime owns output allocation (quantized-inference.md:122-123).
    y = torch.empty(out_spec.shape, dtype=torch.float32 if out_spec.dtype == "f32" else torch.bfloat16,
                    device=session.torch_device)
    sel = _lib.Selection()
    session.launch_qmm(desc, base_ptr(x), base_ptr(w), base_ptr(s), base_ptr(b), y.data_ptr(), sel)
    out = Tensor(session, y, out_spec.dtype)
    out.selection = sel.implementation_id.decode()
    return out
