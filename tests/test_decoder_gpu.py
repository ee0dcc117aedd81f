"""The synthetic quantized Llama decoder (fused qmv epilogues/prologues and
decode attention) against a float32 PyTorch restatement of the same step:
small configurations for 4 and 8 query heads per KV head, 8-bit codes and
batch 32 (the one-pass M=32 qmv), and one step of the full Llama-3-8B shape."""
import math

import numpy as np
import pytest
import torch

from affon_b200 import _lib
from affon_b200.core import AffonError
from affon_b200.decoder import LLAMA3_8B, LlamaConfig, QuantizedDecoder

pytestmark = pytest.mark.gpu

SMALL = LlamaConfig(layers=2, d_model=512, q_heads=4, kv_heads=1, head_dim=128, ffn=1024, vocab=1000)
SMALL_G8 = LlamaConfig(layers=2, d_model=1024, q_heads=16, kv_heads=2, head_dim=128, ffn=2048, vocab=1000)
SMALL_8BIT = LlamaConfig(layers=2, d_model=512, q_heads=8, kv_heads=2, head_dim=128, ffn=1536, vocab=1000, bits=8)


def bf16(t):
    return t.to(torch.bfloat16).float()


def rms_norm(h, g, eps):
    return bf16(h * torch.rsqrt((h * h).mean(dim=-1, keepdim=True) + eps) * g.float())


def rope(x, cos, sin):  # x [..., 128]; rotate-half pairs (d, d+64)
    a, b = x[..., :64], x[..., 64:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], dim=-1)


def normed_proj(h, g, lin, eps):
    """RMSNorm fused into a projection as the decoder computes it: the
    projection reads bf16(h * gamma) and its output rows are scaled by
    rsqrt(mean(h^2) + eps)."""
    r = torch.rsqrt((h * h).mean(dim=-1, keepdim=True) + eps)
    return r * (bf16(h * g.float()) @ lin.dequantized().T)


def ref_step(dec, tokens, pos, kc, vc):
    """One decode step in float32 (bf16 roundings where the kernels store bf16).
    kc/vc: float32 copies of the caches [L][B][kvh][cap][hd], updated in place."""
    c = dec.cfg
    B, G, hd = dec.B, c.q_heads // c.kv_heads, c.head_dim
    h = dec.embed[tokens.long()].float()
    cos, sin = dec.cos[pos], dec.sin[pos]
    for li, lay in enumerate(dec.layers):
        qkv = bf16(normed_proj(h, lay["attn_norm"], lay["qkv"], c.eps))
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
        gu = normed_proj(h, lay["ffn_norm"], lay["gate_up"], c.eps)     # interleaved tiles of 8 gate + 8 up rows
        gu = gu.reshape(B, -1, 2, 8)
        gate, up = gu[:, :, 0, :].reshape(B, -1), gu[:, :, 1, :].reshape(B, -1)
        act = bf16(torch.nn.functional.silu(gate) * up)
        h = h + act @ lay["down"].dequantized().T
    logits = normed_proj(h, dec.final_norm, dec.lm_head, c.eps)
    return h, logits


def check_step(dec, pos, seed):
    """Prefill `pos` positions, run one eager step at `pos`, and compare the
    residual stream, the new cache rows and the greedy tokens with ref_step."""
    c = dec.cfg
    gen = torch.Generator().manual_seed(seed)
    prompt = torch.randint(0, c.vocab, (pos, dec.B), generator=gen)
    dec.prefill(prompt)                        # positions 0..pos-1
    torch.cuda.synchronize()
    kc = dec.k_cache.float().clone()
    vc = dec.v_cache.float().clone()
    tokens = torch.randint(0, c.vocab, (dec.B,), generator=gen).to(dec.device, torch.int32)
    dec.tokens.copy_(tokens)
    dec.reset(pos)
    dec.step_eager()
    dec.synchronize()
    h_ref, logits = ref_step(dec, tokens, pos, kc, vc)
    peak = float(h_ref.abs().max())
    assert float((dec.h - h_ref).abs().max()) <= 2e-2 * peak
    for li in range(c.layers):
        for got, want in ((dec.k_cache[li][:, :, pos], kc[li][:, :, pos]), (dec.v_cache[li][:, :, pos], vc[li][:, :, pos])):
            assert float((got.float() - want).abs().max()) <= 2e-2 * max(1.0, float(want.abs().max()))
    # greedy tokens agree wherever the reference's top two logits are separated
    top2 = torch.topk(logits, 2, dim=-1)
    clear = (top2.values[:, 0] - top2.values[:, 1]) > 1e-2 * top2.values[:, 0].abs().clamp(min=1)
    got = dec.tokens.long()
    assert clear.any()
    assert torch.equal(got[clear], top2.indices[clear, 0])
    assert int(dec.pos.item()) == pos + 1


@pytest.fixture(scope="module")
def dec():
    d = QuantizedDecoder(SMALL, batch=4, capacity=256, device="cuda:0", seed=1, max_steps=64)
    yield d
    d.close()


def test_decode_step_matches_float32_reference(dec):
    check_step(dec, 40, seed=5)


@pytest.mark.parametrize("cfg,batch,pos", [(SMALL_G8, 3, 130), (SMALL_8BIT, 5, 33), (SMALL, 32, 20)],
                         ids=["8q-per-kv", "8bit", "batch32"])
def test_decoder_variants_match_float32_reference(cfg, batch, pos):
    d = QuantizedDecoder(cfg, batch=batch, capacity=192, device="cuda:0", seed=2, max_steps=16)
    try:
        check_step(d, pos, seed=8)
    finally:
        d.close()


def test_llama3_8b_shape_step_matches_float32_reference():
    """One decode step of the full BASELINE 8B shape (32 layers, 8 KV heads,
    K=14336 down projections, vocab 128256 argmax), batch 16."""
    d = QuantizedDecoder(LLAMA3_8B, batch=16, capacity=16, device="cuda:0", seed=3, max_steps=16)
    try:
        check_step(d, 5, seed=9)
    finally:
        d.close()


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
    dec.synchronize()
    assert torch.equal(dec.history[:3], eager_hist)
    assert torch.equal(dec.h, eager_h)
    assert int(dec.pos.item()) == 19


def test_overlap_mode_is_bit_identical():
    """Programmatic dependent launch changes only when kernels start, never
    what they compute."""
    outs = []
    for overlap in (False, True):
        d = QuantizedDecoder(SMALL, batch=4, capacity=64, device="cuda:0", seed=4, max_steps=16, overlap=overlap)
        try:
            gen = torch.Generator().manual_seed(11)
            d.prefill(torch.randint(0, SMALL.vocab, (12, d.B), generator=gen))
            d.capture()
            d.reset(12)
            for _ in range(4):
                d.replay()
            d.synchronize()
            outs.append((d.h.clone(), d.history[:4].clone(), d.k_cache.clone()))
        finally:
            d.close()
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_position_beyond_capacity_is_refused_and_reported():
    d = QuantizedDecoder(SMALL, batch=2, capacity=8, device="cuda:0", seed=5, max_steps=4)
    try:
        d.reset(8)
        with pytest.raises(ValueError):
            d.step_eager()                     # the host refuses before launching
        k0 = d.k_cache.clone()
        d.pos.fill_(8)                         # a device position the host did not set
        d._pos_host = 0
        d.step_eager()
        with pytest.raises(AffonError) as err:
            d.synchronize()
        assert err.value.code == "invalid_arg"
        assert torch.equal(d.k_cache, k0)      # no cache row was written
        d.reset(0)                             # the context stays usable
        d.step_eager()
        d.synchronize()
    finally:
        d.close()


def test_embed_rejects_out_of_range_tokens():
    d = QuantizedDecoder(SMALL, batch=2, capacity=8, device="cuda:0", seed=5, max_steps=4)
    try:
        d.reset(0)
        d.tokens.copy_(torch.tensor([3, SMALL.vocab + 5], dtype=torch.int32))
        d.step_eager()
        with pytest.raises(AffonError) as err:
            d.synchronize()
        assert err.value.code == "invalid_arg"
    finally:
        d.close()


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
        M, K = 29, 1024
        x = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
        out = torch.zeros((M, K), dtype=torch.bfloat16, device=dev)
        check(L.affon_b200_qmv_prep(ctx, 0, x.data_ptr(), K, None, 0, None, ctypes.c_float(0.0), M, K, bits,
                                    out.data_ptr(), K))
        want = _pair_order(x) if bits == 4 else x
        torch.cuda.synchronize()
        assert torch.equal(out, want)
        # rmsnorm from an f32 residual stream and its [K/16][32] partial sums of squares
        h = torch.randn((M, K), generator=gen, device=dev) * 3
        ss = torch.zeros((K // 16, _lib.SS_WIDTH), device=dev)
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


@pytest.mark.parametrize("B,kvh,G,cap,pos,pair", [(2, 2, 4, 256, 0, 1), (3, 1, 8, 256, 63, 0), (4, 2, 4, 512, 64, 1),
                                                  (16, 8, 4, 1088, 1030, 1), (2, 1, 8, 2112, 2047, 1),
                                                  (1, 1, 4, 64, 40, 0)])
def test_decode_attention_matches_float32(B, kvh, G, cap, pos, pair):
    """Decode attention alone against float32 attention over the bf16 cache:
    single and split contexts, tile-boundary positions, 4 and 8 query heads
    per KV head.  The new key (rotated) and value must land in the cache."""
    import ctypes
    from affon_b200.core import check
    from affon_b200.decoder import rope_tables
    dev = torch.device("cuda", 0)
    L = _lib.lib()
    ctx = ctypes.c_void_p()
    check(L.affon_b200_ctx_create(0, None, ctypes.byref(ctx)))
    try:
        check(L.affon_b200_ctx_set_stream(ctx, torch.cuda.current_stream().cuda_stream))
        gen = torch.Generator(device=dev).manual_seed(pos + 7 * B)
        qh, hd = kvh * G, 128
        rows = (qh + 2 * kvh) * hd
        qkv = torch.randn((B, rows), generator=gen, device=dev).to(torch.bfloat16)
        kc = torch.randn((B, kvh, cap, hd), generator=gen, device=dev).to(torch.bfloat16)
        vc = torch.randn((B, kvh, cap, hd), generator=gen, device=dev).to(torch.bfloat16)
        k0, v0 = kc.clone(), vc.clone()
        cfg = LlamaConfig(layers=1, d_model=qh * hd, q_heads=qh, kv_heads=kvh, head_dim=hd, ffn=512, vocab=16)
        cos, sin = rope_tables(cfg, cap, dev)
        posd = torch.tensor([pos], dtype=torch.int32, device=dev)
        out = torch.full((B, qh * hd), float("nan"), dtype=torch.bfloat16, device=dev)
        d = _lib.AttnDesc(ctypes.sizeof(_lib.AttnDesc), B, qh, kvh, hd, cap, 1.0 / math.sqrt(hd), 0, qh * hd,
                          (qh + kvh) * hd, pair, rows, qh * hd)
        check(L.affon_b200_decode_attention(ctx, ctypes.byref(d), qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                            cos.data_ptr(), sin.data_ptr(), posd.data_ptr(), out.data_ptr()))
        assert L.affon_b200_ctx_synchronize(ctx) == 0, _lib.last_error()
        q = qkv[:, :qh * hd].float().reshape(B, qh, hd)
        k = qkv[:, qh * hd:(qh + kvh) * hd].float().reshape(B, kvh, hd)
        v = qkv[:, (qh + kvh) * hd:].reshape(B, kvh, hd)
        kref, vref = k0.float(), v0.float()
        kref[:, :, pos] = bf16(rope(k, cos[pos], sin[pos]))
        vref[:, :, pos] = v.float()
        # the cache rows: only position pos changed
        assert torch.equal(kc[:, :, pos].float(), kref[:, :, pos]) and torch.equal(vc[:, :, pos], v)
        mask = torch.ones(cap, dtype=torch.bool, device=dev)
        mask[pos] = False
        assert torch.equal(kc[:, :, mask], k0[:, :, mask]) and torch.equal(vc[:, :, mask], v0[:, :, mask])
        qr = rope(q, cos[pos], sin[pos]) / math.sqrt(hd)
        keys = kref[:, :, :pos + 1].repeat_interleave(G, dim=1)
        vals = vref[:, :, :pos + 1].repeat_interleave(G, dim=1)
        p = torch.softmax(torch.einsum("bhd,bhtd->bht", qr, keys), dim=-1)
        ref = torch.einsum("bht,bhtd->bhd", p, vals).reshape(B, qh * hd)
        if pair:
            ref = _pair_order(ref)
        got = out.float()
        assert torch.isfinite(got).all()
        assert float((got - ref).abs().max()) <= 2e-2 * max(1.0, float(ref.abs().max()))
    finally:
        L.affon_b200_ctx_destroy(ctx)
