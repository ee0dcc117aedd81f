#!/usr/bin/env python3
"""Generate the golden fixtures for the quantized-matmul parity tests.

Run in a container that has the reference checkout (pass its root with
--reference); the fixtures it writes are committed so that the tests never
read the reference at run time.  Three sources, all from the reference's own
test suite for this path:

* kat.json.gz — the known-answer tests of
  test/e2e/program/operations/quantized-matmul.test.ts and the C-ABI smoke
  src/support/compute_core_cyna_smoke.zig:970-977.  Inputs and expected values
  are the test's literals; the analytic cases (:95-122, :123-148, :171-184,
  :187-204) are expanded here with the test's own generator formulas and its
  float64 expected-value reduction.
* fixture_cells.json.gz — every quantized CUDA cell of
  test/parity/catalogs/cuda-metal-parity.json, with inputs and expected values
  produced by importing test/parity/fixtures/quantized_fixture.py
  (`physical_parameters` and `reference`).
* general_cases.json.gz — the 192 seeded cases of
  test/parity/reference/check-cuda-quantized-general.py (`cases(20261105)`),
  with the expected output of its `expected()` (PyTorch CPU float64, then f32).
"""
import argparse
import gzip
import importlib.util
import json
import math
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _bf16(v):
    """Round a Python float to bf16 (round-to-nearest-even) and return it as float."""
    import numpy as np
    f = np.float32(v)
    u = int(f.view(np.uint32))
    if (u & 0x7F800000) == 0x7F800000:
        return float(f)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return float(np.uint32(u).view(np.float32))


def _dense(values):
    return {"shape": [len(values), len(values[0])], "values": values}


def kat_cases():
    """Known answers of quantized-matmul.test.ts (line numbers in `source`)."""
    out = []

    def case(source, x, xd, w, s, b, pd, bits, group, expected, views=None):
        out.append({"source": source, "bits": bits, "group_size": group, "x_dtype": xd, "p_dtype": pd,
                    "x": x, "w": w, "s": s, "b": b, "expected": expected, "views": views or {}})

    # :7-18 low-bit-first U32 words, per-group affine parameters (8-bit, g4, bf16 params).
    case("quantized-matmul.test.ts:7-18", [[1, 2, 3, 4, 5, 6, 7, 8], [1, 1, 1, 1, 1, 1, 1, 1]], "f32",
         [[0x04030201, 0x08070605], [0x00000000, 0xFFFFFFFF]], [[1, 2], [1, 0.5]], [[0, -1], [2, 0]], "bf16",
         8, 4, [[352, 3335], [58, 518]])
    # :31-43 two and four bits, high bits of unsigned words.
    for bits, word, width, expected in ((2, 0xE4E4E4E4, 16, -24), (4, 0x76543210, 8, 48)):
        case("quantized-matmul.test.ts:31-43", [[k + 1 for k in range(width)]], "bf16", [[word]], [[0.5]], [[-1]],
             "f32", bits, width, [[expected]])
    # :58-78 single native operation.
    case("quantized-matmul.test.ts:58-78", [[1, 2, 3, 4]], "f32", [[0x04030201]], [[1]], [[0]], "bf16", 8, 4, [[30]])
    # :80-93 transposed input and sliced weights / parameters with byte offsets.
    case("quantized-matmul.test.ts:80-93", [[1, 1], [2, 1], [3, 1], [4, 1]], "f32", [[0, 0], [0, 0x04030201]],
         [[0, 1]], [[0, -1]], "bf16", 8, 4, [[20], [6]],
         views={"x": {"transpose": True}, "w": {"slice": [[1, 2], [1, 2]]},
                "s": {"slice": [[0, 1], [1, 2]]}, "b": {"slice": [[0, 1], [1, 2]]}})

    # :95-122 groups crossing word boundaries, zero and negative scales (f32 and bf16).
    k, n, m, g = 24, 3, 2, 3
    q = lambda row, col: (row * 5 + col) % 16
    xs = [[((row + col) % 7 - 3) / 8 for col in range(k)] for row in range(m)]
    ss = [[(grp % 3 - 1) / 4 for grp in range(k // g)] for _ in range(n)]
    bs = [[grp % 2 - 0.5 for grp in range(k // g)] for _ in range(n)]
    ws = [[sum(q(row, word * 8 + lane) << (lane * 4) for lane in range(8)) for word in range(k // 8)] for row in range(n)]
    exp = [[sum(a * (ss[row][col // g] * q(row, col) + bs[row][col // g]) for col, a in enumerate(x)) for row in range(n)]
           for x in xs]
    for dt in ("f32", "bf16"):
        case("quantized-matmul.test.ts:95-122", xs, dt, ws, ss, bs, dt, 4, g, exp)

    # :123-148 partial M/N/K tiles across all bit widths (transposed x / offset w for m in {17, 64}).
    for bits in (2, 4, 8):
        for m in (1, 3, 4, 7, 16, 17, 33, 64, 128):
            n, k, g = (64, 96, 16) if m >= 64 else (19, 80, 16)
            per, mask = 32 // bits, (1 << bits) - 1
            xs = [[((r + c) % 7 - 3) / 8 for c in range(k)] for r in range(m)]
            ws = [[sum(((r * 5 + word * per + lane) & mask) << (lane * bits) for lane in range(per))
                   for word in range(k // per)] for r in range(n)]
            ss = [[(grp % 3 - 1) / 4 for grp in range(k // g)] for _ in range(n)]
            bs = [[grp % 2 - 0.5 for grp in range(k // g)] for _ in range(n)]
            exp = [[sum(a * (ss[o][c // g] * ((o * 5 + c) & mask) + bs[o][c // g]) for c, a in enumerate(row))
                    for o in range(n)] for row in xs]
            views = {}
            if m in (17, 64):
                views = {"x": {"transpose": True}, "w": {"slice": [[0, n], [1, 1 + k // per]]}}
                xs_phys = [[xs[r][c] for r in range(m)] for c in range(k)]
                ws_phys = [[0] + row for row in ws]
            else:
                xs_phys, ws_phys = xs, ws
            case("quantized-matmul.test.ts:123-148", xs_phys, "bf16", ws_phys, ss, bs, "bf16", bits, g, exp, views)

    # :171-184 group / dtype specialisations stay distinct.
    m, n, k = 8, 3, 128
    for g in (32, 64, 128):
        for dt in ("f32", "bf16"):
            groups = k // g
            case("quantized-matmul.test.ts:171-184", [[1] * k for _ in range(m)], "bf16",
                 [[0x80808080] * (k // 4) for _ in range(n)],
                 [[(grp + 1) / 128 for grp in range(groups)] for _ in range(n)],
                 [[-1] * groups for _ in range(n)], dt, 8, g,
                 [[g * groups * (groups - 1) / 2] * n for _ in range(m)])

    # :187-204 groups 48 and 64 across K tiles.
    for g in (48, 64):
        m, n, k = 64, 64, (96 if g == 48 else 256)
        for dt in ("f32", "bf16"):
            vals = [[((r + c) % 11 - 5) / 8 for c in range(k)] for r in range(m)]
            ws = [[sum(((r + c * 4 + lane) % 256) << (lane * 8) for lane in range(4)) for c in range(k // 4)]
                  for r in range(n)]
            ss = [[(r % 3 - 1) * (grp + 1) / 128 for grp in range(k // g)] for r in range(n)]
            bs = [[(grp % 3 - 1) / 4 for grp in range(k // g)] for _ in range(n)]
            exp = [[sum(a * (ss[r][c // g] * ((r + c) % 256) + bs[r][c // g]) for c, a in enumerate(row))
                    for r in range(n)] for row in vals]
            case("quantized-matmul.test.ts:187-204", vals, dt, ws, ss, bs, dt, 8, g, exp)

    # compute_core_cyna_smoke.zig:970-977 (C-ABI known answer).
    case("compute_core_cyna_smoke.zig:970-977",
         [[1, 2, 3, 4, 5, 6, 7, 8], [2, 3, 4, 5, 6, 7, 8, 9]], "f32",
         [[0x01010101, 0x01010101], [0x02020202, 0x02020202], [0x03030303, 0x03030303]],
         [[1, 1], [1, 1], [1, 1]], [[0, 0], [0, 0], [0, 0]], "f32", 8, 4,
         [[36, 72, 108], [44, 88, 132]])
    return out


def fixture_cells(ref):
    fx = _load(ref / "test/parity/fixtures/quantized_fixture.py", "quantized_fixture")
    catalog = json.loads((ref / "test/parity/catalogs/cuda-metal-parity.json").read_text())
    cells = []
    for c in catalog["cases"]:
        if c.get("op") != "quantized_matmul":
            continue
        x, w, s, b = fx.physical_parameters(c)
        expected = fx.reference(c)
        cells.append({"id": c["id"], "dtype": c["dtype"], "shape": c["shape"], "bits": c["bits"],
                      "group_size": c["group_size"], "x": x, "w": w, "s": s, "b": b, "expected": expected})
    return cells


def general_cases(ref, seed):
    gen = _load(ref / "test/parity/reference/check-cuda-quantized-general.py", "check_general")
    out = []
    for c in gen.cases(seed):
        expected = gen.expected(c)
        rec = {"id": c["id"], "shape": c["shape"], "bits": c["bits"], "group_size": c["group_size"], "inputs": {}}
        for name, inp in c["inputs"].items():
            vals = inp["values"]
            if inp["dtype"] == "bf16":  # store the values the reference actually multiplies
                vals = [[_bf16(v) for v in row] for row in vals]
            entry = {"dtype": inp["dtype"], "shape": inp["shape"], "values": vals}
            for key in ("permutation", "slices"):
                if key in inp:
                    entry[key] = inp[key]
            rec["inputs"][name] = entry
        rec["expected"] = [[float(v) for v in row] for row in expected.tolist()]
        out.append(rec)
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", type=Path, required=True, help="root of the reference checkout")
    ap.add_argument("--seed", type=int, default=20261105)
    args = ap.parse_args()
    ref = args.reference.resolve()
    with gzip.open(HERE / "kat.json.gz", "wt", compresslevel=9) as f:
        json.dump(kat_cases(), f)
    with gzip.open(HERE / "fixture_cells.json.gz", "wt", compresslevel=9) as f:
        json.dump(fixture_cells(ref), f)
    with gzip.open(HERE / "general_cases.json.gz", "wt", compresslevel=9) as f:
        json.dump({"seed": args.seed, "cases": general_cases(ref, args.seed)}, f)
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".json", ".gz")))


if __name__ == "__main__":
    sys.exit(main())
