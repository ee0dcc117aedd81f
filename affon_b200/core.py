"""Host-side mirror of the reference's Session / Program / Executable contract
for the quantized-linear path.

Reference behaviour followed:
* `Session({device})`, `session.tensor(values, {dtype})`, tensors owned by one
  Session (src/js/ops.ts:21-28; test/e2e/program/operations/
  quantized-matmul.test.ts:45-56 "same Session").
* `program(name, p => ...)` with `p.argument(name, spec)` and
  `Tensor.f32/bf16/u32(shape)` specs; `Program.inspect()` lists the authored
  nodes (quantized-matmul.test.ts:58-64).
* `session.compile(program, options)` with normalised options forming the
  cache key (docs/core/optimization-and-profiling.md:124-141), `explain()`
  naming the chosen physical implementation (quantized-matmul.test.ts:66-69),
  `numericalPolicy: 'exact_only'` rejecting quantized candidates (:70),
  `denseInputs` guards failing with GuardMismatch (optimization-and-profiling.md:143-151).
* Views: `transpose` / `slice` keep strides and byte offsets; the native kernel
  reads them directly (docs/core/quantized-inference.md:51-52).

PyTorch provides device memory and the current CUDA stream only; the
quantized contraction always runs in libaffon_b200.so.
"""
import ctypes
import itertools
import json

import numpy as np
import torch

from . import _lib

_ERROR_CODES = {
    _lib.INVALID_SHAPE: "invalid_shape",
    _lib.UNSUPPORTED: "unsupported_lowering",
    _lib.CUDA_ERROR: "internal",
    _lib.TIMEOUT: "timeout",
    _lib.GUARD_MISMATCH: "guard_mismatch",
    _lib.POLICY_REJECTED: "unsupported_lowering",
    _lib.INVALID_ARG: "invalid_arg",
    _lib.INVALID_DTYPE: "invalid_dtype",
}


class AffonError(Exception):
    """Runtime failure with a machine-readable `code` (docs/core/errors.md:1-45)."""

    def __init__(self, code, message):
        super().__init__(message)
        self.code = code
        self.message = message


def check(status, what=""):
    if status != _lib.OK:
        msg = _lib.last_error() or f"status {status}"
        raise AffonError(_ERROR_CODES.get(status, "internal"), f"{what}: {msg}" if what else msg)


_TORCH_DTYPE = {"f32": torch.float32, "bf16": torch.bfloat16, "u32": torch.int32}
_NATIVE_DTYPE = {"f32": _lib.F32, "bf16": _lib.BF16, "u32": _lib.U32}


class TensorSpec:
    __slots__ = ("dtype", "shape")

    def __init__(self, dtype, shape):
        if dtype not in _TORCH_DTYPE:
            raise TypeError(f"unsupported dtype {dtype!r}")
        self.dtype = dtype
        self.shape = tuple(int(d) for d in shape)

    def __repr__(self):
        return f"TensorSpec({self.dtype}, {list(self.shape)})"

    def to_json(self):
        return {"dtype": self.dtype, "shape": list(self.shape)}


class Tensor:
    """An evaluated tensor owned by a Session (device memory via torch)."""

    def __init__(self, session, data, dtype):
        self._session = session
        self.data = data  # torch tensor; u32 values are stored as int32 bit patterns
        self.dtype = dtype
        self._disposed = False

    # Spec constructors, as `Tensor.f32([1, 4])` in the reference.
    @staticmethod
    def f32(shape):
        return TensorSpec("f32", shape)

    @staticmethod
    def bf16(shape):
        return TensorSpec("bf16", shape)

    @staticmethod
    def u32(shape):
        return TensorSpec("u32", shape)

    @staticmethod
    def spec(dtype, shape):
        return TensorSpec(dtype, shape)

    @property
    def shape(self):
        return list(self.data.shape)

    @property
    def session(self):
        return self._session

    def _live(self):
        if self._disposed:
            raise AffonError("invalid_arg", "tensor has been disposed")
        if self._session.disposed:
            raise AffonError("invalid_arg", "Session has been disposed")
        return self.data

    def to_numpy(self):
        d = self._live()
        if self.dtype == "u32":
            return d.cpu().numpy().view(np.uint32)
        return d.float().cpu().numpy()

    def to_array(self):
        """Synchronising readback (docs/runtime/configuration.md:109)."""
        a = self.to_numpy()
        return a.astype(np.int64).tolist() if self.dtype == "u32" else a.astype(np.float64).tolist()

    def item(self):
        a = self.to_numpy().reshape(-1)
        return int(a[0]) if self.dtype == "u32" else float(a[0])

    def dispose(self):
        self._disposed = True
        self.data = None


class Session:
    """A CUDA session on one device; `device` is 'cuda' or 'cuda:N'.

    There is no CPU fallback: other devices fail with `backend unavailable`
    (docs/core/backend-support.md: unsupported combinations fail explicitly).
    """

    def __init__(self, device="cuda", telemetry=False, workspace_bytes=None):
        if not (device == "cuda" or (isinstance(device, str) and device.startswith("cuda:"))):
            raise AffonError("unsupported_lowering", f"backend unavailable: affon_b200 runs on cuda, not {device!r}")
        ordinal = int(device.split(":")[1]) if ":" in device else -1
        L = _lib.lib()
        ctx = ctypes.c_void_p()
        check(L.affon_b200_ctx_create(ordinal, None, ctypes.byref(ctx)), "Session")
        self._ctx = ctx
        self.ordinal = L.affon_b200_ctx_device(ctx)
        self.torch_device = torch.device("cuda", self.ordinal)
        if workspace_bytes:
            check(L.affon_b200_ctx_reserve_workspace(ctx, int(workspace_bytes)), "workspace")
        self.device = device
        self.disposed = False
        self._cache = {}

    # -- tensors ---------------------------------------------------------
    def tensor(self, values, dtype="f32"):
        if isinstance(dtype, dict):
            dtype = dtype.get("dtype", "f32")
        if dtype == "u32":
            arr = np.asarray(values, dtype=np.uint64).astype(np.uint32).view(np.int32)
            data = torch.from_numpy(np.ascontiguousarray(arr)).to(self.torch_device)
        else:
            data = torch.as_tensor(np.asarray(values, dtype=np.float64), dtype=torch.float32).to(_TORCH_DTYPE[dtype])
            data = data.to(self.torch_device)
        return Tensor(self, data, dtype)

    def wrap(self, data, dtype):
        """Adopt an existing device tensor (same device) as a Session tensor."""
        if data.device != self.torch_device:
            raise AffonError("device_mismatch", f"tensor on {data.device}, Session on {self.torch_device}")
        return Tensor(self, data, dtype)

    # -- compilation -----------------------------------------------------
    def compile(self, source, options=None):
        if self.disposed:
            raise AffonError("invalid_arg", "Session has been disposed")
        opts = normalize_options(options)
        key = (id(source), json.dumps(opts, sort_keys=True))
        exe = self._cache.get(key)
        if exe is None or exe.disposed:
            exe = Executable(self, source, opts)
            self._cache[key] = exe
        return exe

    # -- native launches ---------------------------------------------------
    def _stream(self):
        return torch.cuda.current_stream(self.torch_device).cuda_stream

    def launch_qmm(self, desc, x, w, s, b, y, selection=None):
        L = _lib.lib()
        check(L.affon_b200_ctx_set_stream(self._ctx, self._stream()))
        sel = selection if selection is not None else None
        status = L.affon_b200_qmm_explain(self._ctx, ctypes.byref(desc), x, w, s, b, y,
                                          ctypes.byref(sel) if sel is not None else None)
        check(status, "quantized_matmul")

    def dispose(self):
        if not self.disposed:
            for exe in self._cache.values():
                exe.disposed = True
            _lib.lib().affon_b200_ctx_destroy(self._ctx)
            self.disposed = True

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()


_DEFAULT_OPTIONS = {"denseInputs": False, "optimizationLevel": "safe", "numericalPolicy": "backend_equivalent",
                    "optimizationGoal": "balanced", "explanationLevel": "summary", "residualPolicy": "retain"}


def normalize_options(options):
    """CompileOptions normalisation (the executable cache key)."""
    opts = dict(_DEFAULT_OPTIONS)
    for k, v in (options or {}).items():
        if k not in _DEFAULT_OPTIONS and k != "searchLimits":
            raise TypeError(f"unknown compile option {k!r}")
        opts[k] = v
    if opts["numericalPolicy"] not in _lib.POLICY:
        raise TypeError("numericalPolicy must be exact_only, backend_equivalent, or approximate")
    return opts


# ---------------------------------------------------------------------------
# Programs (formal authoring)

class FormalTensor:
    __slots__ = ("program", "node", "spec")

    def __init__(self, program, node, spec):
        self.program = program
        self.node = node
        self.spec = spec

    @property
    def shape(self):
        return list(self.spec.shape)

    @property
    def dtype(self):
        return self.spec.dtype


class Program:
    _ids = itertools.count()

    def __init__(self, name):
        self.name = name
        self.nodes = []
        self.arguments = []
        self.outputs = []
        self.id = next(Program._ids)

    def argument(self, name, spec):
        if not isinstance(spec, TensorSpec):
            raise TypeError("argument requires a tensor spec")
        node = {"kind": "argument", "name": name, "spec": spec}
        self.nodes.append(node)
        self.arguments.append(name)
        return FormalTensor(self, len(self.nodes) - 1, spec)

    def emit(self, op, operands, spec, options=None):
        if any(o.program is not self for o in operands):
            raise TypeError("operation operands must belong to the same Program")
        self.nodes.append({"kind": "operation", "op": op, "inputs": [o.node for o in operands], "spec": spec,
                           "options": options or {}})
        return FormalTensor(self, len(self.nodes) - 1, spec)

    def inspect(self):
        nodes = []
        for i, n in enumerate(self.nodes):
            d = {"index": i, "kind": n["kind"], "spec": n["spec"].to_json()}
            if n["kind"] == "operation":
                d.update(op=n["op"], inputs=list(n["inputs"]), options=dict(n["options"]))
            else:
                d["name"] = n["name"]
            nodes.append(d)
        return {"name": self.name, "nodes": nodes, "outputs": list(self.outputs)}


def program(name, author):
    p = Program(name)
    out = author(p)
    outs = out if isinstance(out, (list, tuple)) else [out]
    if not outs or any(not isinstance(o, FormalTensor) or o.program is not p for o in outs):
        raise TypeError("program author must return formal tensors of the program")
    p.outputs = [o.node for o in outs]
    p._single = not isinstance(out, (list, tuple))
    return p


class Executable:
    """A compiled Program: physical implementation per node, frozen."""

    def __init__(self, session, source, options):
        self.session = session
        self.source = source
        self.options = options
        self.disposed = False
        self.physical = []
        policy = _lib.POLICY[options["numericalPolicy"]]
        for i, n in enumerate(source.nodes):
            if n["kind"] != "operation":
                continue
            if n["op"] == "quantized_matmul":
                desc = qmm_desc_from_specs([source.nodes[j]["spec"] for j in n["inputs"]], n["options"], policy,
                                           options["denseInputs"], n["options"].get("out_dtype", "f32"))
                sel = _lib.Selection()
                check(_lib.lib().affon_b200_select(ctypes.byref(desc), ctypes.byref(sel)), "compile quantized_matmul")
                self.physical.append({"node": i, "action": "kernel", "op": n["op"],
                                      "implementation_id": sel.implementation_id.decode(),
                                      "implementation_version": sel.implementation_version,
                                      "numerical_class": _lib.NUMERICS[sel.numerical_class],
                                      "reason": sel.reason.decode()})
            elif n["op"] in ("transpose", "slice"):
                self.physical.append({"node": i, "action": "view", "op": n["op"],
                                      "view_transform": n["op"], **({"view_permutation": n["options"]["axes"]}
                                                                     if n["op"] == "transpose" else
                                                                     {"view_slice_ranges": n["options"]["ranges"]})})
            elif n["op"] == "add":
                self.physical.append({"node": i, "action": "kernel", "op": "add",
                                      "implementation_id": "cuda_elementwise.add", "implementation_version": 1,
                                      "numerical_class": "exact"})
            else:
                raise AffonError("unsupported_lowering", f"operation {n['op']} has no lowering")

    def explain(self):
        return {"program": self.source.name, "options": dict(self.options),
                "executable": {"physical_nodes": [dict(p) for p in self.physical]}}

    def run(self, inputs):
        if self.disposed:
            raise AffonError("invalid_arg", "executable has been disposed")
        from . import ops
        values = {}
        for i, n in enumerate(self.source.nodes):
            if n["kind"] == "argument":
                if n["name"] not in inputs:
                    raise AffonError("missing_arg", f"missing argument {n['name']!r}")
                t = inputs[n["name"]]
                if not isinstance(t, Tensor) or t.session is not self.session:
                    raise TypeError("operation tensors must belong to the same Session")
                if t.dtype != n["spec"].dtype or tuple(t.shape) != n["spec"].shape:
                    raise AffonError("shape_mismatch", f"argument {n['name']!r} does not match {n['spec']}")
                values[i] = t
            else:
                args = [values[j] for j in n["inputs"]]
                values[i] = ops._evaluate(self.session, n["op"], args, n["options"], self.options)
        outs = [values[j] for j in self.source.outputs]
        return outs[0] if getattr(self.source, "_single", True) else tuple(outs)

    def dispose(self):
        self.disposed = True


def view_of(t):
    """Native view (shape, element strides, byte offset) of an evaluated tensor."""
    d = t.data
    r, c = d.shape
    return _lib.View(r, c, d.stride(0), d.stride(1), d.storage_offset() * d.element_size())


def base_ptr(t):
    d = t.data
    return d.data_ptr() - d.storage_offset() * d.element_size()


def qmm_desc_from_specs(specs, options, policy, dense, out_dtype="f32"):
    x, w, s, b = specs
    desc = _lib.QmmDesc()
    desc.struct_size = ctypes.sizeof(_lib.QmmDesc)
    desc.bits = int(options["bits"])
    desc.group_size = int(options["group_size"])
    desc.x_dtype, desc.param_dtype = _NATIVE_DTYPE[x.dtype], _NATIVE_DTYPE[s.dtype]
    desc.y_dtype = _NATIVE_DTYPE[out_dtype]
    desc.numerical_policy = policy
    desc.dense_inputs = 1 if dense else 0
    for name, sp in zip("xwsb", specs):
        r, c = sp.shape
        setattr(desc, name, _lib.View(r, c, c, 1, 0))
    desc.y = _lib.View(x.shape[0], w.shape[0], w.shape[0], 1, 0)
    return desc
