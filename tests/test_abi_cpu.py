"""CPU-only checks of the C-ABI library: it loads, exports every symbol the
header declares, and validates / selects exactly as the reference's lowering
contract says (no GPU calls)."""
import ctypes
import re

import pytest

from affon_b200 import _lib
from affon_b200.core import AffonError, Tensor, program, qmm_desc_from_specs
from affon_b200.ops import quantized_matmul, validate_quantized_matmul
from gpu_util import dense_desc


def declared_functions():
    text = _lib.HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(affon_b200_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 14
    for name in names:
        assert hasattr(L, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must cover the header exactly"
    assert L.affon_b200_abi_version() == 1


def test_struct_layouts_match_header_sizes():
    """affon_b200_view is five int64; the descriptor is a 40-byte header then five views."""
    assert ctypes.sizeof(_lib.View) == 40
    assert _lib.QmmDesc.group_size.offset == 8
    assert _lib.QmmDesc.x.offset == 40
    assert ctypes.sizeof(_lib.QmmDesc) == 240
    assert ctypes.sizeof(_lib.Selection) == 64 + 16 + 256


def desc(M=1, N=4096, K=4096, bits=4, group=64, xd="bf16", pd="bf16", yd="f32", policy="backend_equivalent",
         dense=False):
    per = 32 // bits
    specs = [Tensor.spec(xd, [M, K]), Tensor.u32([N, K // per]), Tensor.spec(pd, [N, K // group]),
             Tensor.spec(pd, [N, K // group])]
    return qmm_desc_from_specs(specs, {"bits": bits, "group_size": group}, _lib.POLICY[policy], dense, yd)


def select(d):
    sel = _lib.Selection()
    rc = _lib.lib().affon_b200_select(ctypes.byref(d), ctypes.byref(sel))
    return rc, sel


@pytest.mark.parametrize("M,bits", [(1, 4), (4, 8), (16, 4), (16, 8)])
def test_select_qmv_for_decode(M, bits):
    rc, sel = select(desc(M=M, bits=bits))
    assert rc == 0, _lib.last_error()
    assert sel.implementation_id.decode() == f"cuda_quantized_matmul.sm100_qmv_b{bits}_g64"
    assert _lib.NUMERICS[sel.numerical_class] == "reassociated"
    assert b"cuda_host_" not in sel.implementation_id


@pytest.mark.parametrize("kw", [dict(bits=2), dict(group=32), dict(xd="f32"), dict(pd="f32"), dict(K=4096 + 64)])
def test_select_generic_outside_fast_contract(kw):
    rc, sel = select(desc(M=4, **kw))
    assert rc == 0, _lib.last_error()
    assert sel.implementation_id.decode() == "cuda_quantized_matmul.sm100_generic"


def test_exact_only_rejects_quantized_candidates():
    """quantized-inference.md:175-177 / quantized-matmul.test.ts:70."""
    rc, _ = select(desc(policy="exact_only"))
    assert rc == _lib.POLICY_REJECTED
    assert "exact_only" in _lib.last_error()


@pytest.mark.parametrize("mutate,status", [
    (lambda d: setattr(d, "bits", 3), _lib.INVALID_SHAPE),
    (lambda d: setattr(d, "group_size", 0), _lib.INVALID_SHAPE),
    (lambda d: setattr(d.w, "cols", d.w.cols + 1), _lib.INVALID_SHAPE),
    (lambda d: setattr(d.s, "cols", d.s.cols - 1), _lib.INVALID_SHAPE),
    (lambda d: setattr(d.b, "rows", d.b.rows - 1), _lib.INVALID_SHAPE),
    (lambda d: setattr(d, "x_dtype", _lib.U32), _lib.INVALID_DTYPE),
    (lambda d: setattr(d, "struct_size", 12), _lib.INVALID_ARG),
    (lambda d: setattr(d.y, "rows", 2), _lib.INVALID_SHAPE),
])
def test_native_validation_rules(mutate, status):
    d = desc()
    mutate(d)
    assert _lib.lib().affon_b200_validate(ctypes.byref(d)) == status


def test_dense_inputs_guard():
    """optimization-and-profiling.md:143-151: strided or offset views fail with GuardMismatch."""
    d = desc(dense=True)
    assert _lib.lib().affon_b200_validate(ctypes.byref(d)) == 0
    d.x.byte_offset = 4
    assert _lib.lib().affon_b200_validate(ctypes.byref(d)) == _lib.GUARD_MISMATCH


def test_authoring_validation_messages():
    """program.ts:483-492 messages (quantized-matmul.test.ts:20-29,45-56)."""
    src = lambda p, opts: quantized_matmul(p.argument("x", Tensor.f32([1, 4])), p.argument("w", Tensor.u32([1, 1])),
                                           p.argument("s", Tensor.f32([1, 1])), p.argument("b", Tensor.f32([1, 1])),
                                           opts)
    program("ok", lambda p: src(p, {"bits": 8, "group_size": 4}))
    with pytest.raises(TypeError, match="bits"):
        program("bad", lambda p: src(p, {"bits": 3, "group_size": 4}))
    with pytest.raises(TypeError, match="do not match"):
        program("bad", lambda p: src(p, {"bits": 8, "group_size": 3}))
    with pytest.raises(TypeError, match="do not match"):
        program("bad", lambda p: src(p, {"bits": 4, "group_size": 4}))
    with pytest.raises(TypeError, match="group_size"):
        program("bad", lambda p: src(p, {"bits": 8, "group_size": 0}))


def test_program_authors_single_native_operation():
    """quantized-matmul.test.ts:58-64."""
    source = program("quantized_linear", lambda p: quantized_matmul(
        p.argument("x", Tensor.f32([1, 4])), p.argument("w", Tensor.u32([1, 1])),
        p.argument("s", Tensor.bf16([1, 1])), p.argument("b", Tensor.bf16([1, 1])), {"bits": 8, "group_size": 4}))
    ops = [n["op"] for n in source.inspect()["nodes"] if n["kind"] == "operation"]
    assert ops == ["quantized_matmul"]
    out = source.nodes[source.outputs[0]]["spec"]
    assert out.dtype == "f32" and out.shape == (1, 1)


def test_formal_and_evaluated_cannot_mix():
    with pytest.raises(TypeError, match="mix"):
        program("m", lambda p: quantized_matmul(p.argument("x", Tensor.f32([1, 4])), object(), object(), object(),
                                                {"bits": 8, "group_size": 4}))


def test_validate_spec_helper_matches_reference_spec():
    spec = validate_quantized_matmul([Tensor.bf16([3, 128]), Tensor.u32([5, 16]), Tensor.bf16([5, 2]),
                                      Tensor.bf16([5, 2])], {"bits": 4, "group_size": 64})
    assert spec.dtype == "f32" and spec.shape == (3, 5)


def test_cyna_signature_rejects_bad_shapes_without_gpu():
    """compute_core_cyna.zig:1013-1023: shape errors return 1 before any device work."""
    import numpy as np
    f = np.zeros(16, dtype=np.float32)
    w = np.zeros(6, dtype=np.uint32)
    out = np.full(6, -1, dtype=np.float32)
    L = _lib.lib()
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    assert L.affon_b200_compute_core_run_quantized_matmul_f32(p(f), 16, p(w), 6, p(f), 6, p(f), 6, p(out), 6, 2, 8, 3,
                                                              3, 4) == 1
    assert L.affon_b200_compute_core_run_quantized_matmul_f32(p(f), 16, p(w), 6, p(f), 6, p(f), 6, p(out), 6, 2, 8, 3,
                                                              8, 0) == 1
    assert (out == -1).all()


def test_prefill_selection_by_rows_and_policy():
    """M >= 64 with the default policy selects the reassociated kernel; M = 63
    stays on qmv passes; `approximate` selects the bf16-rounding kernel;
    `exact_only` rejects every quantized candidate."""
    L = _lib.lib()
    for M, policy, want in [(64, "backend_equivalent", "exact_b4"), (63, "backend_equivalent", "qmv_b4"),
                            (512, "approximate", "tcgen05_b4"), (4096, "backend_equivalent", "exact_b4")]:
        d = dense_desc(M, 4096, 4096, 4)
        d.numerical_policy = _lib.POLICY[policy]
        sel = _lib.Selection()
        assert L.affon_b200_select(d, sel) == 0, _lib.last_error()
        impl = sel.implementation_id.decode()
        assert impl.endswith(want + "_g64"), (M, policy, impl)
        assert sel.numerical_class == (2 if policy == "approximate" else 1)
    d = dense_desc(512, 4096, 4096, 4)
    d.numerical_policy = _lib.POLICY["exact_only"]
    assert L.affon_b200_select(d, _lib.Selection()) != 0


def test_qmv_plan_by_shape():
    """Decode plans (148 SMs): N up to three 16-row tiles per SM with K up to 32
    stages takes whole-K blocks split over a CTA's warps (no cross-CTA
    combine: one K segment per tile); longer K, larger N and M > 16 stream K
    across CTAs and combine."""
    L = _lib.lib()
    cases = [((16, 4096, 4096, 4), "32-row whole-K blocks over 128 CTAs"),    # O
             ((16, 6144, 4096, 4), "48-row whole-K blocks over 128 CTAs"),    # QKV
             ((8, 1024, 4096, 8), "16-row whole-K blocks over 64 CTAs"),
             ((16, 4096, 7168, 4), "32-row whole-K blocks"),                  # down shard at TP2
             ((16, 4096, 14336, 4), "stream-K"),                             # down: 56 stages
             ((32, 4096, 4096, 4), "stream-K"),                              # M > 16
             ((16, 16384, 4096, 4), "stream-K")]                             # 7 tiles per SM
    for (M, N, K, bits), want in cases:
        sel = _lib.Selection()
        assert L.affon_b200_select(dense_desc(M, N, K, bits), sel) == 0, _lib.last_error()
        reason = sel.reason.decode()
        assert want in reason, (M, N, K, reason)
        assert (sel.splits == 1) == ("whole-K" in want), (M, N, K, sel.splits, reason)
