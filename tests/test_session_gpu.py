"""The reference's e2e quantized_matmul tests (test/e2e/program/operations/
quantized-matmul.test.ts) restated against the Session / ops mirror on CUDA."""
import pytest

from affon_b200 import AffonError, Session, Tensor, program, quantized_matmul, slice, transpose
from affon_b200.ops import add

pytestmark = pytest.mark.gpu


@pytest.fixture
def session():
    s = Session(device="cuda")
    yield s
    s.dispose()


def test_decodes_low_bit_first_words(session):
    """:7-18"""
    x = session.tensor([[1, 2, 3, 4, 5, 6, 7, 8], [1, 1, 1, 1, 1, 1, 1, 1]])
    w = session.tensor([[0x04030201, 0x08070605], [0x00000000, 0xFFFFFFFF]], dtype="u32")
    s = session.tensor([[1, 2], [1, 0.5]], dtype="bf16")
    b = session.tensor([[0, -1], [2, 0]], dtype="bf16")
    y = quantized_matmul(x, w, s, b, {"bits": 8, "group_size": 4})
    assert y.shape == [2, 2] and y.dtype == "f32"
    assert y.to_array() == [[352, 3335], [58, 518]]


def test_rejects_mismatched_metadata(session):
    """:20-29"""
    x = session.tensor([[1, 2, 3, 4]])
    w = session.tensor([[0x04030201]], dtype="u32")
    s = session.tensor([[1]])
    b = session.tensor([[0]])
    with pytest.raises(TypeError):
        quantized_matmul(x, w, s, b, {"bits": 8, "group_size": 3})
    with pytest.raises(TypeError):
        quantized_matmul(x, w, s, b, {"bits": 4, "group_size": 4})


def test_two_and_four_bits(session):
    """:31-43"""
    for bits, word, width, expected in ((2, 0xE4E4E4E4, 16, -24), (4, 0x76543210, 8, 48)):
        x = session.tensor([[k + 1 for k in range(width)]], dtype="bf16")
        y = quantized_matmul(x, session.tensor([[word]], dtype="u32"), session.tensor([[0.5]]), session.tensor([[-1]]),
                             {"bits": bits, "group_size": width})
        assert y.to_array() == [[expected]]


def test_cross_session_and_bits(session):
    """:45-56"""
    other = Session(device="cuda")
    try:
        x = session.tensor([[1, 2, 3, 4]])
        w = session.tensor([[0xFFFFFFFF]], dtype="u32")
        s = session.tensor([[1]])
        with pytest.raises(TypeError, match="same Session"):
            quantized_matmul(x, w, s, other.tensor([[0]]), {"bits": 8, "group_size": 4})
        with pytest.raises(TypeError, match="bits"):
            quantized_matmul(x, w, s, session.tensor([[0]]), {"bits": 3, "group_size": 4})
    finally:
        other.dispose()


def test_program_selects_native_kernel_and_runs(session):
    """:58-78"""
    source = program("quantized_linear", lambda p: quantized_matmul(
        p.argument("x", Tensor.f32([1, 4])), p.argument("w", Tensor.u32([1, 1])),
        p.argument("s", Tensor.bf16([1, 1])), p.argument("b", Tensor.bf16([1, 1])), {"bits": 8, "group_size": 4}))
    exe = session.compile(source, {"explanationLevel": "detailed"})
    text = str(exe.explain())
    assert "cuda_quantized_matmul" in text and "cuda_host_" not in text
    with pytest.raises(AffonError):
        session.compile(source, {"numericalPolicy": "exact_only"})
    y = exe.run({"x": session.tensor([[1, 2, 3, 4]]), "w": session.tensor([[0x04030201]], dtype="u32"),
                 "s": session.tensor([[1]], dtype="bf16"), "b": session.tensor([[0]], dtype="bf16")})
    assert y.to_array() == [[30]]


def test_transposed_and_sliced_views(session):
    """:80-93"""
    x = transpose(session.tensor([[1, 1], [2, 1], [3, 1], [4, 1]]), [1, 0])
    w = slice(session.tensor([[0, 0], [0, 0x04030201]], dtype="u32"), [{"start": 1, "stop": 2}, {"start": 1, "stop": 2}])
    s = slice(session.tensor([[0, 1]], dtype="bf16"), [{"start": 0, "stop": 1}, {"start": 1, "stop": 2}])
    b = slice(session.tensor([[0, -1]], dtype="bf16"), [{"start": 0, "stop": 1}, {"start": 1, "stop": 2}])
    assert quantized_matmul(x, w, s, b, {"bits": 8, "group_size": 4}).to_array() == [[20], [6]]


def test_dense_inputs_guard(session):
    source = program("dense", lambda p: quantized_matmul(
        p.argument("x", Tensor.f32([2, 4])), p.argument("w", Tensor.u32([1, 1])),
        p.argument("s", Tensor.f32([1, 1])), p.argument("b", Tensor.f32([1, 1])), {"bits": 8, "group_size": 4}))
    exe = session.compile(source, {"denseInputs": True})
    xt = transpose(session.tensor([[1, 1], [2, 1], [3, 1], [4, 1]]), [1, 0])
    with pytest.raises(AffonError) as err:
        exe.run({"x": xt, "w": session.tensor([[0x04030201]], dtype="u32"), "s": session.tensor([[1]]),
                 "b": session.tensor([[0]])})
    assert err.value.code == "guard_mismatch"


def test_composed_program(session):
    """The parity worker's composed form add(result, result) (workers/affon-quantized.ts:61-62)."""
    source = program("composed", lambda p: (lambda r: add(r, r))(quantized_matmul(
        p.argument("x", Tensor.f32([1, 4])), p.argument("w", Tensor.u32([1, 1])),
        p.argument("s", Tensor.f32([1, 1])), p.argument("b", Tensor.f32([1, 1])), {"bits": 8, "group_size": 4})))
    y = session.compile(source).run({"x": session.tensor([[1, 2, 3, 4]]), "w": session.tensor([[0x04030201]],
                                                                                              dtype="u32"),
                                     "s": session.tensor([[1]]), "b": session.tensor([[0]])})
    assert y.to_array() == [[60]]
