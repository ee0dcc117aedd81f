"""The synthetic quantized Llama decoder (fused qmv epilogues/prologues and
decode attention) against a float32 PyTorch restatement of the same step."""
import math

import numpy as np
import pytest
import torch

from affon_b200.decoder import LlamaConfig, QuantizedDecoder

pytestmark = pytest.mark.gpu

SMALL = LlamaConfig(layers=2, d_model=512, q_heads=4, kv_heads=1, head_dim=128, ffn=1024, vocab=1000)


def bf16(t):
    return t.to(torch.bfloat16).float()


def rms_norm(h, g, eps):
    return bf16(h * torch.rsqrt((h * h).mean(dim=-1, keepdim=True) + eps) * g.float())


def rope(x, cos, sin):  # x [..., 128]; rotate-half pairs (d, d+64)
    a, b = x[..., :64], x[..., 64:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], dim=-1)


def ref_step(dec, tokens, pos, kc, vc):
    """One decode step in float32 (bf16 roundings where the kernels store bf16).
    kc/vc: float32 copies of the caches [L][B][kvh][cap][hd], updated in place."""
    c = dec.cfg
    B, G, hd = dec.B, c.q_heads // c.kv_heads, c.head_dim
    h = dec.embed[tokens.long()].float()
    cos, sin = dec.cos[pos], dec.sin[pos]
    for li, lay in enumerate(dec.layers):
        xn = rms_norm(h, lay["attn_norm"], c.eps)
        qkv = bf16(xn @ lay["qkv"].dequantized().T)
        q = qkv[:, :c.q_heads * hd].reshape(B, c.q_heads, hd)
        k = qkv[:, c.q_heads * hd:(c.q_heads + c.kv_heads) * hd].reshape(B, c.kv_heads, hd)
        v = qkv[:, (c.q_heads + c.kv_heads) * hd:].reshape(B, c.kv_heads, hd)
        qr = rope(q, cos, sin) / math.sqrt(hd)
        kc[li][:, :, pos] = bf16(rope(k, cos, sin))
        vc[li][:, :, pos] = v
        keys = kc[li][:, :, :pos + 1]                                   # [B, kvh, T, hd]
        vals = vc[li][:, :, :pos + 1]
        kq = keys.repeat_interleave(G, dim=1)                           # [B, qh, T, hd]
        vq = vals.repeat_interleave(G, dim=1)
        scores = torch.einsum("bhd,bhtd->bht", qr, kq)
        p = torch.softmax(scores, dim=-1)
        attn = bf16(torch.einsum("bht,bhtd->bhd", p, vq).reshape(B, -1))
        h = h + attn @ lay["o"].dequantized().T
        xn2 = rms_norm(h, lay["ffn_norm"], c.eps)
        gu = xn2 @ lay["gate_up"].dequantized().T                       # interleaved tiles of 8 gate + 8 up rows
        gu = gu.reshape(B, -1, 2, 8)
        gate, up = gu[:, :, 0, :].reshape(B, -1), gu[:, :, 1, :].reshape(B, -1)
        act = bf16(torch.nn.functional.silu(gate) * up)
        h = h + act @ lay["down"].dequantized().T
    xf = rms_norm(h, dec.final_norm, c.eps)
    logits = xf @ dec.lm_head.dequantized().T
    return h, logits


@pytest.fixture(scope="module")
def dec():
    d = QuantizedDecoder(SMALL, batch=4, capacity=256, device="cuda:0", seed=1, max_steps=64)
    yield d
    d.close()


def test_decode_step_matches_float32_reference(dec):
    gen = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, SMALL.vocab, (40, dec.B), generator=gen)
    dec.prefill(prompt)                        # eager steps, positions 0..39
    torch.cuda.synchronize()
    kc = dec.k_cache.float().clone()
    vc = dec.v_cache.float().clone()
    tokens = torch.randint(0, SMALL.vocab, (dec.B,), generator=gen).to(dec.device, torch.int32)
    dec.tokens.copy_(tokens)
    dec.reset(40)
    dec.step_eager()
    torch.cuda.synchronize()
    h_ref, logits = ref_step(dec, tokens, 40, kc, vc)
    peak = float(h_ref.abs().max())
    assert float((dec.h - h_ref).abs().max()) <= 2e-2 * peak
    # the new cache rows
    for li in range(SMALL.layers):
        assert float((dec.k_cache[li][:, :, 40].float() - kc[li][:, :, 40]).abs().max()) <= 2e-2 * max(
            1.0, float(kc[li][:, :, 40].abs().max()))
    # greedy tokens agree wherever the reference's top two logits are separated
    top2 = torch.topk(logits, 2, dim=-1)
    clear = (top2.values[:, 0] - top2.values[:, 1]) > 1e-2 * top2.values[:, 0].abs().clamp(min=1)
    got = dec.tokens.long()
    assert clear.any()
    assert torch.equal(got[clear], top2.indices[clear, 0])
    assert int(dec.pos.item()) == 41


def test_prefill_cache_matches_reference(dec):
    gen = torch.Generator().manual_seed(6)
    T = 24
    prompt = torch.randint(0, SMALL.vocab, (T, dec.B), generator=gen)
    dec.prefill(prompt)
    torch.cuda.synchronize()
    c = SMALL
    kc = torch.zeros_like(dec.k_cache, dtype=torch.float32)
    vc = torch.zeros_like(dec.v_cache, dtype=torch.float32)
    for t in range(T):
        ref_step(dec, prompt[t].to(dec.device), t, kc, vc)
    for li in range(c.layers):
        got = dec.k_cache[li][:, :, :T].float()
        want = kc[li][:, :, :T]
        assert float((got - want).abs().max()) <= 3e-2 * max(1.0, float(want.abs().max()))


def test_graph_replay_equals_eager_steps(dec):
    gen = torch.Generator().manual_seed(7)
    prompt = torch.randint(0, SMALL.vocab, (16, dec.B), generator=gen)
    dec.prefill(prompt)
    start_tokens = dec.tokens.clone()
    k0, v0 = dec.k_cache.clone(), dec.v_cache.clone()
    dec.reset(16)
    for _ in range(3):
        dec.step_eager()
    eager_hist = dec.history[:3].clone()
    eager_h = dec.h.clone()
    # same three steps through the captured graph
    dec.k_cache.copy_(k0)
    dec.v_cache.copy_(v0)
    dec.tokens.copy_(start_tokens)
    dec.reset(16)
    dec.capture()          # capture runs one step; restore and replay
    dec.k_cache.copy_(k0)
    dec.v_cache.copy_(v0)
    dec.tokens.copy_(start_tokens)
    dec.reset(16)
    for _ in range(3):
        dec.replay()
    torch.cuda.synchronize()
    assert torch.equal(dec.history[:3], eager_hist)
    assert torch.equal(dec.h, eager_h)
    assert int(dec.pos.item()) == 19


def _pair_order(x):
    """4-bit qmv column order: within each 8 columns [x0 x4 x1 x5 x2 x6 x3 x7]."""
    r, k = x.shape
    return x.reshape(r, k // 8, 2, 4).transpose(-1, -2).reshape(r, k)


@pytest.mark.parametrize("bits", [4, 8])
def test_qmv_prep_orders_and_normalizes(bits):
    import ctypes
    from affon_b200 import _lib
    from affon_b200.core import check
    dev = torch.device("cuda", 0)
    L = _lib.lib()
    ctx = ctypes.c_void_p()
    check(L.affon_b200_ctx_create(0, None, ctypes.byref(ctx)))
    try:
        check(L.affon_b200_ctx_set_stream(ctx, torch.cuda.current_stream().cuda_stream))
        gen = torch.Generator(device=dev).manual_seed(3)
        M, K = 13, 1024
        x = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
        out = torch.zeros((M, K), dtype=torch.bfloat16, device=dev)
        check(L.affon_b200_qmv_prep(ctx, 0, x.data_ptr(), K, None, 0, None, ctypes.c_float(0.0), M, K, bits,
                                    out.data_ptr(), K))
        want = _pair_order(x) if bits == 4 else x
        torch.cuda.synchronize()
        assert torch.equal(out, want)
        # rmsnorm from an f32 residual stream and its [K/16][16] partial sums of squares
        h = torch.randn((M, K), generator=gen, device=dev) * 3
        ss = torch.zeros((K // 16, 16), device=dev)
        ss[:, :M] = (h * h).reshape(M, K // 16, 16).sum(-1).T
        g = (1 + 0.1 * torch.randn((K,), generator=gen, device=dev)).to(torch.bfloat16)
        check(L.affon_b200_qmv_prep(ctx, 1, h.data_ptr(), K, ss.data_ptr(), K // 16, g.data_ptr(),
                                    ctypes.c_float(1e-5), M, K, bits, out.data_ptr(), K))
        torch.cuda.synchronize()
        ref = rms_norm(h, g, 1e-5)
        ref = _pair_order(ref) if bits == 4 else ref
        assert float((out.float() - ref).abs().max()) <= 1e-2 * float(ref.abs().max())
        assert L.affon_b200_ctx_synchronize(ctx) == 0
    finally:
        L.affon_b200_ctx_destroy(ctx)
