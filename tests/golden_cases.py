"""Golden cases for quantized_matmul, materialised as physical buffers + views.

Each case yields four operands (x, w, s, b) as physical numpy arrays with a
logical view (element strides and byte offset), exactly the information the
reference's strided kernels receive (docs/core/quantized-inference.md:51-52).
The fixtures come from tests/golden/ (see make_golden.py there).
"""
import gzip
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def bf16_bits(values):
    """float array -> uint16 bf16 bit patterns, round to nearest even."""
    f = np.ascontiguousarray(np.asarray(values, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7F800000) == 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = (u[nan] >> 16).astype(np.uint16)
    return r


def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class Operand:
    phys: np.ndarray      # physical storage (float32, uint16 bf16 bits, or uint32 words)
    dtype: str            # 'f32' | 'bf16' | 'u32'
    row_stride: int       # element strides of the logical [rows, cols] view
    col_stride: int
    offset: int           # element offset of logical [0,0]
    shape: tuple          # logical shape

    @property
    def byte_offset(self):
        return self.offset * self.phys.itemsize

    def logical_f64(self):
        flat = self.phys.reshape(-1)
        if self.dtype == "bf16":
            flat = bf16_to_f32(flat)
        r, c = self.shape
        idx = self.offset + np.arange(r)[:, None] * self.row_stride + np.arange(c)[None, :] * self.col_stride
        return flat[idx].astype(np.float64) if self.dtype != "u32" else flat[idx]

    def dense_copy(self):
        """A dense, zero-offset copy of the logical view (same dtype)."""
        flat = self.phys.reshape(-1)
        r, c = self.shape
        idx = self.offset + np.arange(r)[:, None] * self.row_stride + np.arange(c)[None, :] * self.col_stride
        return np.ascontiguousarray(flat[idx])


def make_operand(values, dtype, view=None):
    arr = np.asarray(values, dtype=np.float64 if dtype != "u32" else np.uint64)
    if dtype == "u32":
        phys = arr.astype(np.uint32)
    elif dtype == "bf16":
        phys = bf16_bits(arr.astype(np.float32))
    else:
        phys = arr.astype(np.float32)
    rows, cols = phys.shape
    view = view or {}
    if view.get("transpose") or view.get("permutation") == [1, 0]:
        return Operand(phys, dtype, 1, cols, 0, (cols, rows))
    if "slice" in view:
        (r0, r1), (c0, c1) = view["slice"]
        return Operand(phys, dtype, cols, 1, r0 * cols + c0, (r1 - r0, c1 - c0))
    if "slices" in view:
        sr, sc = view["slices"]
        nr = len(range(sr["start"], sr["stop"], sr["step"]))
        nc = len(range(sc["start"], sc["stop"], sc["step"]))
        return Operand(phys, dtype, cols * sr["step"], sc["step"], sr["start"] * cols + sc["start"], (nr, nc))
    return Operand(phys, dtype, cols, 1, 0, (rows, cols))


@dataclass
class Case:
    name: str
    bits: int
    group_size: int
    x: Operand
    w: Operand
    s: Operand
    b: Operand
    expected: np.ndarray   # float64 [M, N]
    exact: bool            # the reference asserts exact equality (toEqual)

    @property
    def mnk(self):
        return self.x.shape[0], self.w.shape[0], self.x.shape[1]


def kat_cases():
    with gzip.open(GOLDEN / "kat.json.gz", "rt") as f:
        raw = json.load(f)
    out = []
    for i, c in enumerate(raw):
        v = c["views"]
        out.append(Case(f"kat{i}:{c['source']}", c["bits"], c["group_size"],
                        make_operand(c["x"], c["x_dtype"], v.get("x")), make_operand(c["w"], "u32", v.get("w")),
                        make_operand(c["s"], c["p_dtype"], v.get("s")), make_operand(c["b"], c["p_dtype"], v.get("b")),
                        np.asarray(c["expected"], dtype=np.float64), True))
    return out


def fixture_cells():
    """Catalog cells of test/parity/catalogs/cuda-metal-parity.json with the
    fixture layouts of quantized_fixture.py:21-33."""
    with gzip.open(GOLDEN / "fixture_cells.json.gz", "rt") as f:
        raw = json.load(f)
    out = []
    for c in raw:
        m, k, n = c["shape"]
        per = 32 // c["bits"]
        dt = c["dtype"]
        transposed = "/transposed/" in c["id"]
        offset = "/offset_" in c["id"]
        if transposed:
            views = {"x": {"transpose": True}, "w": {"slice": [[0, n], [1, 1 + k // per]]}}
        elif offset:
            views = {"x": {"slice": [[1, 1 + m], [1, 1 + k]]}, "w": {"slice": [[1, 1 + n], [1, 1 + k // per]]},
                     "s": {"slice": [[1, 1 + n], [1, 1 + k // c["group_size"]]]},
                     "b": {"slice": [[1, 1 + n], [1, 1 + k // c["group_size"]]]}}
        else:
            views = {}
        expected = np.asarray(c["expected"], dtype=np.float64).reshape(m, n)
        out.append(Case(c["id"], c["bits"], c["group_size"], make_operand(c["x"], dt, views.get("x")),
                        make_operand(c["w"], "u32", views.get("w")), make_operand(c["s"], dt, views.get("s")),
                        make_operand(c["b"], dt, views.get("b")), expected, False))
    return out


def general_cases():
    """Seeded cases of check-cuda-quantized-general.py (seed 20261105)."""
    with gzip.open(GOLDEN / "general_cases.json.gz", "rt") as f:
        raw = json.load(f)
    out = []
    for c in raw["cases"]:
        ops = {}
        for name in ("x", "w", "s", "b"):
            inp = c["inputs"][name]
            view = {}
            if "permutation" in inp:
                view["permutation"] = inp["permutation"]
            if "slices" in inp:
                view["slices"] = inp["slices"]
            ops[name] = make_operand(inp["values"], inp["dtype"], view)
        out.append(Case(c["id"], c["bits"], c["group_size"], ops["x"], ops["w"], ops["s"], ops["b"],
                        np.asarray(c["expected"], dtype=np.float64), False))
    return out


def f32_tolerance(expected):
    """check-cuda-quantized-general.py:110 — 2e-6 * max(1, peak |reference|), every element."""
    return 2e-6 * max(1.0, float(np.abs(expected).max()))


def bf16_tolerance(expected):
    """benchmark-cells-pytorch.py:334-335 peer tolerance for bf16: 0.02 * max(1, peak)."""
    return 2e-2 * max(1.0, float(np.abs(expected).max()))
