"""`affon:nn`-level quantized linear layer for the Program mirror.

The reference's dense layer is `nn.linear({out_features, bias})`
(src/js/nn.ts:251-275): a callable over `{x}` bindings that declares the
parameters `${name}.weight` (and `${name}.bias`) and emits a matmul.  Its
quantized-inference notes ask that a quantized model "obtain bits/group_size
from checkpoint configuration, bind the three existing ordinary tensors, and
select quantized linear layers", with names such as `.weight`, `.scales` and
`.biases` belonging to the adapter (docs/core/quantized-inference.md:108-112).

`quantized_linear({out_features, bits, group_size, bias})` is that layer: it
declares `${name}.weight` (u32 [out, in*bits/32]), `${name}.scales` and
`${name}.biases` ([out, in/group_size], the activation's float dtype unless
`param_dtype` is given) as Program arguments and lowers to
`quantized_matmul(x, weight, scales, biases, {bits, group_size})` -- x
[rows, in] times the decoded weight transposed, f32 result -- plus an
optional `${name}.bias` add.  The parameters are bound at run time by name,
e.g. from `affon_b200.checkpoint.QuantizedCheckpoint.bind`.
"""
from .core import Tensor, TensorSpec
from .ops import add, quantized_matmul

_SCALE_DTYPES = ("f32", "bf16")


def _check_options(options):
    if not isinstance(options, dict):
        raise TypeError("quantized_linear expects options")
    out_features = options.get("out_features")
    bits = options.get("bits")
    group = options.get("group_size")
    bias = options.get("bias", False)
    if not isinstance(out_features, int) or isinstance(out_features, bool) or out_features <= 0:
        raise TypeError("quantized_linear out_features must be a positive integer")
    if bits not in (2, 4, 8):
        raise TypeError("quantized_linear bits must be 2, 4, or 8")
    if not isinstance(group, int) or isinstance(group, bool) or group <= 0:
        raise TypeError("quantized_linear group_size must be a positive integer")
    if not isinstance(bias, bool):
        raise TypeError("quantized_linear bias must be boolean")
    pd = options.get("param_dtype")
    if pd is not None and pd not in _SCALE_DTYPES:
        raise TypeError("quantized_linear param_dtype must be f32 or bf16")
    return out_features, bits, group, bias, pd


def quantized_linear(options):
    """A quantized linear layer: `layer({"x": x}, name)` -> FormalTensor."""
    out_features, bits, group, bias, param_dtype = _check_options(options)

    def layer(bindings, name="linear"):
        if not isinstance(name, str) or not name:
            raise TypeError("quantized_linear instance name must be a non-empty string")
        if not isinstance(bindings, dict) or "x" not in bindings:
            raise TypeError("quantized_linear requires an x binding")
        x = bindings["x"]
        in_features = x.spec.shape[-1] if x.spec.shape else None
        if not isinstance(in_features, int) or in_features <= 0:
            raise TypeError("quantized_linear requires a known positive input feature size")
        per_word = 32 // bits
        if in_features % per_word or in_features % group:
            raise TypeError("quantized_linear input features must divide into packed words and groups")
        pd = param_dtype or x.spec.dtype
        p = x.program
        weight = p.argument(f"{name}.weight", Tensor.u32([out_features, in_features // per_word]))
        scales = p.argument(f"{name}.scales", TensorSpec(pd, [out_features, in_features // group]))
        biases = p.argument(f"{name}.biases", TensorSpec(pd, [out_features, in_features // group]))
        y = quantized_matmul(x, weight, scales, biases, {"bits": bits, "group_size": group})
        if bias:
            offset = p.argument(f"{name}.bias", TensorSpec("f32", [out_features]))
            y = add(y, offset)
        return y

    return layer


def parameter_names(name, bias=False):
    """The argument names a quantized_linear instance binds."""
    names = [f"{name}.weight", f"{name}.scales", f"{name}.biases"]
    return names + [f"{name}.bias"] if bias else names
