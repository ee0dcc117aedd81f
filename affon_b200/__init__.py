"""affon_b200 — B200-native (sm_100a) affine group-quantized matmul for Affon.

The compute lives in libaffon_b200.so (built from affon_b200/csrc); this
package is its host-side mirror of `affon:ops.quantized_matmul` and the
Session / Program / Executable lowering contract.
"""
from ._lib import lib as native_library  # noqa: F401
from .core import AffonError, Executable, FormalTensor, Program, Session, Tensor, TensorSpec, program  # noqa: F401
from .ops import add, quantized_matmul, slice, transpose  # noqa: F401

__all__ = ["AffonError", "Executable", "FormalTensor", "Program", "Session", "Tensor", "TensorSpec", "program",
           "quantized_matmul", "add", "slice", "transpose", "native_library"]
