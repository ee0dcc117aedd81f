"""A checkpoint's quantized linears run through the nn-level layer on the GPU.

The adapter binds `.weight/.scales/.biases` from a safetensors file written
here; the layer's Program compiles to the sm_100a kernels (explain names
`cuda_quantized_matmul`) and its output matches the CPU oracle on the same
bytes, with and without a layer bias.
"""
import numpy as np
import pytest
import torch

import oracle
from affon_b200 import Session, checkpoint, nn, synthetic
from affon_b200.core import Tensor, program

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits,N,K,M,bias", [(4, 256, 512, 3, False), (8, 128, 1024, 16, True),
                                             (4, 4096, 4096, 1, False)])
def test_checkpoint_layer_matches_oracle(tmp_path, bits, N, K, M, bias):
    d = synthetic.quantized_linear(M, N, K, bits=bits, seed=40 + bits)
    path = tmp_path / "m.safetensors"
    checkpoint.write(path, {"blk.proj.weight": d["w"], "blk.proj.scales": d["s"], "blk.proj.biases": d["b"]})
    ck = checkpoint.QuantizedCheckpoint(path, bits, 64)
    opts = dict(ck.options("blk.proj"), bias=bias)
    layer = nn.quantized_linear(opts)
    with Session("cuda:0") as sess:
        src = program("proj", lambda p: layer({"x": p.argument("x", Tensor.bf16([M, K]))}, "proj"))
        exe = sess.compile(src)
        assert any(n.get("implementation_id", "").startswith("cuda_quantized_matmul")
                   for n in exe.explain()["executable"]["physical_nodes"])
        inputs = ck.bind(sess, "blk.proj", "proj")
        xt = torch.from_numpy(d["x"].view(np.int16)).view(torch.bfloat16).to(sess.torch_device)
        inputs["x"] = sess.wrap(xt, "bf16")
        bvec = np.linspace(-1, 1, N, dtype=np.float32)
        if bias:
            inputs["proj.bias"] = sess.tensor(bvec, "f32")
        y = exe.run(inputs).to_numpy()
    ref = oracle.qmm_dense(d["x"], "bf16", d["w"], d["s"], d["b"], "bf16", M, N, K, bits, 64)
    if bias:
        ref = ref + bvec
    assert np.abs(y - ref).max() <= 1e-5 * max(1.0, float(np.abs(ref).max()))
