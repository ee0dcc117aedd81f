"""Checkpoint adapter for affine group-quantized linears (safetensors, U32).

A quantized linear is stored as three ordinary tensors of one prefix:
`prefix.weight` (U32 [out, in*bits/32], codes packed little-endian, low bits
first), `prefix.scales` and `prefix.biases` (BF16 or F32 [out, in/group]) --
the layout the reference's quantized-checkpoint tool reads
(tools/test-quantized-checkpoint.py:21-55) and documents
(docs/core/quantized-inference.md:45-67,108-112).

As that document requires, the scheme is not guessed from dtypes: bits and
group size come from the caller or from the checkpoint's configuration
(a `quantization` object with `bits` and `group_size`, as in MLX's
config.json), a prefix is a quantized linear only when all three tensors are
present, and every shape is checked against the scheme -- mismatches raise
instead of being silently reinterpreted.  Tensors are uploaded as they lie
on disk (no repacking) and bound under the names `affon_b200.nn.
quantized_linear` declares.

safetensors: 8-byte little-endian header length, a JSON header
{name: {"dtype", "shape", "data_offsets": [begin, end]}} (offsets relative to
the data section after the header), then the data.
"""
import json
import struct
from pathlib import Path

import numpy as np
import torch

from .core import AffonError, Tensor

_NP = {"U32": np.uint32, "BF16": np.uint16, "F32": np.float32}
_DT = {"U32": "u32", "BF16": "bf16", "F32": "f32"}


def read_header(path):
    """(header dict without __metadata__, metadata dict, data offset)."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise AffonError("invalid_checkpoint", f"{path}: not a safetensors file")
        (n,) = struct.unpack("<Q", raw)
        if n <= 0 or n > 1 << 28:
            raise AffonError("invalid_checkpoint", f"{path}: bad header length {n}")
        header = json.loads(f.read(n))
    meta = header.pop("__metadata__", {}) or {}
    return header, meta, 8 + n


def write(path, tensors, metadata=None):
    """Write numpy arrays as a safetensors file (dtypes uint32 -> U32,
    uint16 -> BF16 bit patterns, float32 -> F32)."""
    names = {np.dtype(np.uint32): "U32", np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32"}
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr)
        b = a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes()
        header[name] = {"dtype": names[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def scheme_from_config(config_path):
    """(bits, group_size) from a config.json `quantization` object."""
    cfg = json.loads(Path(config_path).read_text())
    q = cfg.get("quantization") or cfg.get("quantization_config")
    if not isinstance(q, dict) or "bits" not in q or "group_size" not in q:
        raise AffonError("invalid_checkpoint", f"{config_path}: no quantization {{bits, group_size}}")
    return int(q["bits"]), int(q["group_size"])


class QuantizedCheckpoint:
    """The quantized linears of one safetensors file under a given scheme."""

    def __init__(self, path, bits, group_size):
        if bits not in (2, 4, 8):
            raise AffonError("invalid_checkpoint", "quantization bits must be 2, 4, or 8")
        if not isinstance(group_size, int) or group_size <= 0:
            raise AffonError("invalid_checkpoint", "quantization group_size must be a positive integer")
        self.path, self.bits, self.group_size = Path(path), bits, group_size
        self.header, self.metadata, self._data = read_header(path)
        self.layers = {}
        for name, spec in self.header.items():
            if not name.endswith(".weight") or spec.get("dtype") != "U32":
                continue
            prefix = name[: -len(".weight")]
            if prefix + ".scales" not in self.header or prefix + ".biases" not in self.header:
                continue                    # a U32 tensor alone is not a quantized linear
            self.layers[prefix] = self._check(prefix)

    def _check(self, prefix):
        w, s, b = (self.header[prefix + k] for k in (".weight", ".scales", ".biases"))
        if s["dtype"] not in ("BF16", "F32") or b["dtype"] != s["dtype"]:
            raise AffonError("invalid_checkpoint", f"{prefix}: scales and biases must both be BF16 or F32")
        if len(w["shape"]) != 2:
            raise AffonError("invalid_checkpoint", f"{prefix}.weight must be rank two")
        out, words = w["shape"]
        in_features = words * (32 // self.bits)
        if in_features % self.group_size:
            raise AffonError("invalid_checkpoint",
                             f"{prefix}: {in_features} input features do not divide into groups of {self.group_size}")
        want = [out, in_features // self.group_size]
        if s["shape"] != want or b["shape"] != want:
            raise AffonError("invalid_checkpoint", f"{prefix}: scales/biases shape {s['shape']} is not {want} for "
                                                   f"{self.bits}-bit codes in groups of {self.group_size}")
        for spec, k in ((w, ".weight"), (s, ".scales"), (b, ".biases")):
            n = int(np.prod(spec["shape"])) * np.dtype(_NP[spec["dtype"]]).itemsize
            lo, hi = spec["data_offsets"]
            if hi - lo != n:
                raise AffonError("invalid_checkpoint", f"{prefix}{k}: data size {hi - lo} bytes, expected {n}")
        return {"out_features": out, "in_features": in_features, "param_dtype": _DT[s["dtype"]]}

    def options(self, prefix):
        """`affon_b200.nn.quantized_linear` options for one layer."""
        lay = self.layers[prefix]
        return {"out_features": lay["out_features"], "bits": self.bits, "group_size": self.group_size,
                "param_dtype": lay["param_dtype"]}

    def array(self, name):
        """One tensor as a numpy array read from disk (little-endian)."""
        spec = self.header[name]
        dt = np.dtype(_NP[spec["dtype"]]).newbyteorder("<")
        lo, hi = spec["data_offsets"]
        mm = np.memmap(self.path, dtype=np.uint8, mode="r", offset=self._data + lo, shape=(hi - lo,))
        return np.frombuffer(mm, dtype=dt).reshape(spec["shape"]).astype(dt.newbyteorder("="))

    def bind(self, session, prefix, name=None):
        """Upload one layer's three tensors to the session's device, keyed by
        the argument names of a quantized_linear instance called `name`
        (default: the checkpoint prefix)."""
        if prefix not in self.layers:
            raise AffonError("invalid_checkpoint", f"{prefix!r} is not a quantized linear of {self.path.name}")
        name = name or prefix
        out = {}
        for key in (".weight", ".scales", ".biases"):
            spec = self.header[prefix + key]
            a = self.array(prefix + key)
            if spec["dtype"] == "U32":
                data = torch.from_numpy(np.ascontiguousarray(a).view(np.int32))
            elif spec["dtype"] == "BF16":
                data = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
            else:
                data = torch.from_numpy(np.ascontiguousarray(a))
            data = data.to(session.torch_device)
            out[name + key] = Tensor(session, data, _DT[spec["dtype"]])
        return out
