"""The CPU oracle against every golden vector the reference holds for this path."""
import numpy as np
import pytest

import oracle
from golden_cases import f32_tolerance, fixture_cells, general_cases, kat_cases

KATS = kat_cases()
CELLS = fixture_cells()
GENERAL = general_cases()


@pytest.mark.parametrize("case", KATS, ids=[c.name for c in KATS])
def test_kat_exact(case):
    """quantized-matmul.test.ts asserts exact equality (toEqual) on these."""
    y = oracle.qmm_case(case)
    assert y.shape == case.expected.shape
    np.testing.assert_array_equal(y.astype(np.float64), case.expected)


def test_fixture_cells_match_reference_fixture():
    """All 268 CUDA quantized catalog cells vs quantized_fixture.reference (f64)."""
    assert len(CELLS) == 268
    for case in CELLS:
        y = oracle.qmm_case(case)
        err = np.abs(y - case.expected).max()
        assert err <= f32_tolerance(case.expected), (case.name, err)


def test_general_cases_within_reference_tolerance():
    """The 192 seeded cases (bits x dtype pairs x 4 shapes x 4 layouts) of
    check-cuda-quantized-general.py:34-59, within 2e-6*max(1,peak) (:110)."""
    assert len(GENERAL) == 192
    for case in GENERAL:
        y = oracle.qmm_case(case)
        err = np.abs(y.astype(np.float64) - case.expected).max()
        assert err <= f32_tolerance(case.expected), (case.name, err)


def test_f64_variant_matches_general_reference():
    for case in GENERAL[::7]:
        y = oracle.qmm_case(case, f64=True)
        assert np.abs(y.astype(np.float32).astype(np.float64) - case.expected).max() <= 1e-6 * max(1, np.abs(case.expected).max())


def test_cyna_abi_known_answer_and_rejections():
    """compute_core_cyna_smoke.zig:970-984: known answer, invalid shapes leave output untouched."""
    act = np.array([1, 2, 3, 4, 5, 6, 7, 8, 2, 3, 4, 5, 6, 7, 8, 9], dtype=np.float32)
    w = np.array([0x01010101, 0x01010101, 0x02020202, 0x02020202, 0x03030303, 0x03030303], dtype=np.uint32)
    s = np.ones(6, dtype=np.float32)
    b = np.zeros(6, dtype=np.float32)
    out = np.full(6, -1, dtype=np.float32)
    assert oracle.cyna_qmm_f32(act, w, s, b, out, 2, 8, 3, 8, 4) == 0
    np.testing.assert_array_equal(out, [36, 72, 108, 44, 88, 132])
    out[:] = -1
    assert oracle.cyna_qmm_f32(act, w, s, b, out, 2, 8, 3, 3, 4) == 1
    assert oracle.cyna_qmm_f32(act, w, s, b, out, 2, 8, 3, 8, 0) == 1
    assert oracle.cyna_qmm_f32(act, w, s, b, out, 2**64 - 1, 8, 3, 8, 4) == 1
    np.testing.assert_array_equal(out, [-1] * 6)


def test_unpack_low_bits_first():
    """quantized-inference.md:59-62: the first logical value is the least significant bits."""
    w = np.array([[0x76543210]], dtype=np.uint32)
    assert oracle.unpack(w, 1, 8, 4).tolist() == [[0, 1, 2, 3, 4, 5, 6, 7]]
    w = np.array([[0xE4E4E4E4]], dtype=np.uint32)
    assert oracle.unpack(w, 1, 16, 2).tolist() == [[0, 1, 2, 3] * 4]
    w = np.array([[0x04030201]], dtype=np.uint32)
    assert oracle.unpack(w, 1, 4, 8).tolist() == [[1, 2, 3, 4]]


@pytest.mark.parametrize("bits,group,K", [(8, 3, 4), (4, 4, 4), (3, 4, 24), (8, 0, 4), (4, 3, 8)])
def test_validation_rules(bits, group, K):
    """program.ts:484-493: bits in {2,4,8}, group>0, K divides into words and groups."""
    assert oracle.lib().affon_oracle_validate(1, 1, K, bits, group) == 1
