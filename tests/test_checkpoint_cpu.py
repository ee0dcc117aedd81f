"""The U32 checkpoint adapter and the nn-level quantized linear, without a GPU.

A small safetensors file written here holds two quantized linears, a lone
U32 tensor and a dense tensor; the adapter must find exactly the two layers
(quantized-inference.md:108-112: never treat every U32 tensor as quantized),
read them back bit-exactly, take bits/group_size from the configuration, and
reject shapes that do not fit the scheme.  The nn layer must author one
quantized_matmul with the adapter's parameter names.
"""
import json

import numpy as np
import pytest

from affon_b200 import checkpoint, nn, synthetic
from affon_b200.core import AffonError, Tensor, program


def _layer(N, K, bits, seed):
    d = synthetic.quantized_linear(1, N, K, bits=bits, seed=seed)
    return d["w"], d["s"], d["b"]


@pytest.fixture
def ckpt(tmp_path):
    w1, s1, b1 = _layer(64, 256, 4, 1)
    w2, s2, b2 = _layer(32, 128, 4, 2)
    tensors = {"model.layers.0.mlp.up_proj.weight": w1, "model.layers.0.mlp.up_proj.scales": s1,
               "model.layers.0.mlp.up_proj.biases": b1,
               "lm_head.weight": w2, "lm_head.scales": s2.view(np.uint16), "lm_head.biases": b2,
               "model.rotary.inv_freq_bits": np.arange(8, dtype=np.uint32),        # U32 but not quantized
               "model.norm.weight": np.ones(256, dtype=np.float32)}
    path = tmp_path / "model.safetensors"
    checkpoint.write(path, tensors, metadata={"format": "mlx"})
    (tmp_path / "config.json").write_text(json.dumps({"quantization": {"bits": 4, "group_size": 64}}))
    return path, tensors


def test_adapter_finds_only_complete_quantized_linears(ckpt):
    path, tensors = ckpt
    bits, group = checkpoint.scheme_from_config(path.parent / "config.json")
    ck = checkpoint.QuantizedCheckpoint(path, bits, group)
    assert sorted(ck.layers) == ["lm_head", "model.layers.0.mlp.up_proj"]
    assert ck.layers["model.layers.0.mlp.up_proj"] == {"out_features": 64, "in_features": 256, "param_dtype": "bf16"}
    assert ck.metadata == {"format": "mlx"}
    for name in ("model.layers.0.mlp.up_proj.weight", "lm_head.scales", "lm_head.biases"):
        np.testing.assert_array_equal(ck.array(name), tensors[name])


@pytest.mark.parametrize("bits,group", [(8, 64), (4, 48), (2, 64)])
def test_adapter_rejects_a_scheme_the_shapes_do_not_fit(ckpt, bits, group):
    path, _ = ckpt
    with pytest.raises(AffonError) as e:
        checkpoint.QuantizedCheckpoint(path, bits, group)
    assert e.value.code == "invalid_checkpoint"


def test_adapter_rejects_mismatched_parameter_dtypes(tmp_path):
    w, s, b = _layer(16, 128, 4, 3)
    path = tmp_path / "bad.safetensors"
    checkpoint.write(path, {"x.weight": w, "x.scales": s, "x.biases": synthetic.bf16_to_f32(b)})
    with pytest.raises(AffonError):
        checkpoint.QuantizedCheckpoint(path, 4, 64)


def test_config_without_scheme_is_refused(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"hidden_size": 8}))
    with pytest.raises(AffonError):
        checkpoint.scheme_from_config(tmp_path / "config.json")


def test_nn_quantized_linear_authors_one_quantized_matmul(ckpt):
    path, _ = ckpt
    ck = checkpoint.QuantizedCheckpoint(path, 4, 64)
    layer = nn.quantized_linear(ck.options("model.layers.0.mlp.up_proj"))
    src = program("up", lambda p: layer({"x": p.argument("x", Tensor.bf16([3, 256]))}, "up"))
    nodes = src.inspect()["nodes"]
    ops = [n for n in nodes if n["kind"] == "operation"]
    assert [o["op"] for o in ops] == ["quantized_matmul"]
    assert ops[0]["options"] == {"bits": 4, "group_size": 64}
    assert ops[0]["spec"] == {"dtype": "f32", "shape": [3, 64]}
    names = [n["name"] for n in nodes if n["kind"] == "argument"]
    assert names == ["x"] + nn.parameter_names("up")
    with pytest.raises(TypeError):
        nn.quantized_linear({"out_features": 64, "bits": 3, "group_size": 64})
    with pytest.raises(TypeError):
        program("bad", lambda p: layer({"x": p.argument("x", Tensor.bf16([3, 250]))}, "up"))
