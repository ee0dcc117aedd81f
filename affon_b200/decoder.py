"""Synthetic Llama-shaped decoder on the affon_b200 kernels.

Every projection is a 4-bit (or 8-bit) affine group-quantized linear
(`quantized_matmul` layout: codes packed little-endian into u32 along K,
group 64, bf16 scale and bias), run by the decode qmv with the decoder's
residual adds, SiLU-gated product and final argmax fused into its epilogue.
RMSNorm is one small kernel that also writes the normalized activations in
the qmv's column order; attention and the SiLU epilogue write theirs in that
order directly.
Attention is the affon_b200 decode-attention kernel (RoPE and KV-cache
append fused).  The reference has no quantized decoder; the layer structure
follows its Llama program (packages/@affon/models/src/llama/model.ts:64-78:
norm -> q/k/v -> RoPE -> attention -> o + residual -> norm -> gate/up ->
SiLU*mul -> down + residual; final norm -> LM head), untied, with the
BASELINE shapes.

Weights are random (seeded), with the BASELINE code/scale/bias
distributions.  The gate/up projection is stored as one weight whose 16-row
tiles hold 8 gate rows followed by the 8 matching up rows, so the qmv
epilogue sees both halves of each SiLU product in one thread.

A decode step is captured once in a CUDA graph: the current position,
step counter and tokens live in device memory and are advanced by the last
kernel, so replays run back to back with no host work.
"""
import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib
from .core import check


@dataclass(frozen=True)
class LlamaConfig:
    layers: int
    d_model: int
    q_heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    eps: float = 1e-5
    rope_theta: float = 500000.0
    bits: int = 4
    group: int = 64

    @property
    def qkv_rows(self):
        return (self.q_heads + 2 * self.kv_heads) * self.head_dim


LLAMA3_8B = LlamaConfig(layers=32, d_model=4096, q_heads=32, kv_heads=8, head_dim=128, ffn=14336, vocab=128256)
LLAMA3_70B = LlamaConfig(layers=80, d_model=8192, q_heads=64, kv_heads=8, head_dim=128, ffn=28672, vocab=128256)


def linear_param_count(cfg):
    per_layer = cfg.qkv_rows * cfg.d_model + cfg.d_model * cfg.q_heads * cfg.head_dim + 3 * cfg.ffn * cfg.d_model
    return cfg.layers * per_layer + cfg.vocab * cfg.d_model


def weight_bytes(cfg):
    """Packed codes plus bf16 scales and biases of every linear."""
    n = linear_param_count(cfg)
    return n * cfg.bits // 8 + (n // cfg.group) * 4


class QuantLinear:
    """Device tensors of one quantized linear [N, K] (+ its descriptor)."""

    def __init__(self, N, K, bits, group, gen, device):
        per = 32 // bits
        self.N, self.K, self.bits, self.group = N, K, bits, group
        self.w = torch.randint(-2 ** 31, 2 ** 31 - 1, (N, K // per), generator=gen, device=device, dtype=torch.int32)
        s = torch.randn((N, K // group), generator=gen, device=device).abs() * 0.02 + 1e-3
        self.s = s.to(torch.bfloat16)
        self.b = (self.s.float() * -(1 << (bits - 1))).to(torch.bfloat16)

    def desc(self, M, ld_x=None, y_dtype=_lib.BF16, x_dtype=_lib.BF16):
        per = 32 // self.bits
        d = _lib.QmmDesc()
        d.struct_size = ctypes.sizeof(_lib.QmmDesc)
        d.bits, d.group_size = self.bits, self.group
        d.x_dtype, d.param_dtype, d.y_dtype = x_dtype, _lib.BF16, y_dtype
        d.numerical_policy = _lib.POLICY["backend_equivalent"]
        d.x = _lib.View(M, self.K, ld_x or self.K, 1, 0)
        d.w = _lib.View(self.N, self.K // per, self.K // per, 1, 0)
        d.s = d.b = _lib.View(self.N, self.K // self.group, self.K // self.group, 1, 0)
        d.y = _lib.View(M, self.N, self.N, 1, 0)
        return d

    def dequantized(self):
        """float32 [N, K] decoded weight (for reference checks)."""
        per = 32 // self.bits
        words = self.w.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        shifts = torch.arange(per, device=words.device, dtype=torch.int64) * self.bits
        codes = ((words.unsqueeze(-1) >> shifts) & ((1 << self.bits) - 1)).reshape(self.N, self.K).float()
        s = self.s.float().repeat_interleave(self.group, dim=1)
        b = self.b.float().repeat_interleave(self.group, dim=1)
        return codes * s + b


def rope_tables(cfg, capacity, device):
    half = cfg.head_dim // 2
    inv = cfg.rope_theta ** (-torch.arange(half, dtype=torch.float64) * 2.0 / cfg.head_dim)
    ang = torch.arange(capacity, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float().to(device).contiguous(), torch.sin(ang).float().to(device).contiguous()


class QuantizedDecoder:
    """Batch-`batch` greedy decoder with a KV cache of `capacity` positions."""

    def __init__(self, cfg, batch, capacity, device, seed=0, max_steps=4096, workspace_bytes=None):
        if batch > 16:
            raise ValueError("decode qmv handles up to 16 rows per step")
        self.cfg, self.B, self.cap = cfg, batch, capacity
        self.device = torch.device(device)
        dev = self.device
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        c = cfg
        self.embed = (torch.randn((c.vocab, c.d_model), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        gamma = lambda: (1.0 + 0.1 * torch.randn((c.d_model,), generator=gen, device=dev)).to(torch.bfloat16)
        self.layers = []
        for _ in range(c.layers):
            self.layers.append({
                "attn_norm": gamma(),
                "qkv": QuantLinear(c.qkv_rows, c.d_model, c.bits, c.group, gen, dev),
                "o": QuantLinear(c.d_model, c.q_heads * c.head_dim, c.bits, c.group, gen, dev),
                "ffn_norm": gamma(),
                "gate_up": QuantLinear(2 * c.ffn, c.d_model, c.bits, c.group, gen, dev),
                "down": QuantLinear(c.d_model, c.ffn, c.bits, c.group, gen, dev),
            })
        self.final_norm = gamma()
        self.lm_head = QuantLinear(c.vocab, c.d_model, c.bits, c.group, gen, dev)
        kv_shape = (c.layers, batch, c.kv_heads, capacity, c.head_dim)
        self.k_cache = torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev)
        self.cos, self.sin = rope_tables(c, capacity, dev)
        # step state (device)
        self.tokens = torch.zeros((batch,), dtype=torch.int32, device=dev)
        self.pos = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.step_ctr = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.history = torch.zeros((max_steps, batch), dtype=torch.int32, device=dev)
        self.h = torch.zeros((batch, c.d_model), dtype=torch.float32, device=dev)
        self.ss = torch.zeros((c.d_model // 16, 16), dtype=torch.float32, device=dev)
        self.xq = torch.zeros((batch, c.d_model), dtype=torch.bfloat16, device=dev)   # normalized x, qmv order
        self.qkv = torch.zeros((batch, c.qkv_rows), dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros((batch, c.q_heads * c.head_dim), dtype=torch.bfloat16, device=dev)
        self.act = torch.zeros((batch, c.ffn), dtype=torch.bfloat16, device=dev)
        self.amax = torch.zeros((batch,), dtype=torch.int64, device=dev)
        L = _lib.lib()
        self._L = L
        self.ctx = ctypes.c_void_p()
        check(L.affon_b200_ctx_create(dev.index, None, ctypes.byref(self.ctx)), "decoder context")
        if workspace_bytes:
            check(L.affon_b200_ctx_reserve_workspace(self.ctx, int(workspace_bytes)))
        self._build_calls()
        self.graph = None

    # -- launch descriptors --------------------------------------------------
    def _build_calls(self):
        c, B = self.cfg, self.B
        L = self._L
        hd = c.head_dim
        self.attn_desc = _lib.AttnDesc(ctypes.sizeof(_lib.AttnDesc), B, c.q_heads, c.kv_heads, hd, self.cap,
                                       1.0 / math.sqrt(hd), 0, c.q_heads * hd, (c.q_heads + c.kv_heads) * hd, 0,
                                       c.qkv_rows, c.q_heads * hd)
        ptr = lambda t: ctypes.c_void_p(t.data_ptr())
        pair = 1 if c.bits == 4 else 0          # producers write the 4-bit qmv's pair order
        self.attn_desc.out_pair_order = pair
        fz = lambda **kw: _lib.QmvFusion(struct_size=ctypes.sizeof(_lib.QmvFusion), x_mode=1, **kw)
        resid = dict(epilogue=_lib.EPI_RESID, h_out=ptr(self.h), ld_h_out=c.d_model, ss_out=ptr(self.ss))
        xq = ptr(self.xq)
        self.calls = []
        for i, lay in enumerate(self.layers):
            q, o, gu, dn = lay["qkv"], lay["o"], lay["gate_up"], lay["down"]
            self.calls.append(("norm", lay["attn_norm"]))
            self.calls.append(("qmv", q.desc(B), xq, q, ptr(self.qkv), fz(epilogue=_lib.EPI_STORE)))
            self.calls.append(("attn", i))
            self.calls.append(("qmv", o.desc(B), ptr(self.attn), o, None, fz(**resid)))
            self.calls.append(("norm", lay["ffn_norm"]))
            self.calls.append(("qmv", gu.desc(B), xq, gu, None,
                               fz(epilogue=_lib.EPI_SILU_MUL, act=ptr(self.act), ld_act=c.ffn, act_pair_order=pair)))
            self.calls.append(("qmv", dn.desc(B), ptr(self.act), dn, None, fz(**resid)))
        lm = self.lm_head
        self.calls.append(("norm", self.final_norm))
        self.calls.append(("qmv", lm.desc(B), xq, lm, None, fz(epilogue=_lib.EPI_ARGMAX, amax=ptr(self.amax))))
        self._kv_layer = [(self.k_cache[i], self.v_cache[i]) for i in range(c.layers)]

    def launches_per_step(self):
        """Kernels one decode step launches: embed, then one per call, then finalize."""
        return 2 + len(self.calls)

    def _launch_step(self, finalize=True):
        L, ctx = self._L, self.ctx
        c = self.cfg
        check(L.affon_b200_embed(ctx, self.embed.data_ptr(), c.d_model, self.tokens.data_ptr(), self.B, c.d_model,
                                 self.h.data_ptr(), self.ss.data_ptr(), self.amax.data_ptr()), "embed")
        for call in self.calls:
            if call[0] == "norm":
                check(L.affon_b200_qmv_prep(ctx, 1, self.h.data_ptr(), c.d_model, self.ss.data_ptr(), c.d_model // 16,
                                            call[1].data_ptr(), ctypes.c_float(c.eps), self.B, c.d_model, c.bits,
                                            self.xq.data_ptr(), c.d_model), "qmv_prep")
            elif call[0] == "attn":
                kc, vc = self._kv_layer[call[1]]
                check(L.affon_b200_decode_attention(ctx, ctypes.byref(self.attn_desc), self.qkv.data_ptr(),
                                                    kc.data_ptr(), vc.data_ptr(), self.cos.data_ptr(),
                                                    self.sin.data_ptr(), self.pos.data_ptr(), self.attn.data_ptr()),
                      "decode_attention")
            else:
                _, desc, x, lin, y, fus = call
                check(L.affon_b200_qmv_fused(ctx, ctypes.byref(desc), x, lin.w.data_ptr(), lin.s.data_ptr(),
                                             lin.b.data_ptr(), y, ctypes.byref(fus)), "qmv_fused")
        if finalize:
            check(L.affon_b200_argmax_finalize(ctx, self.amax.data_ptr(), self.B, self.tokens.data_ptr(),
                                               self.history.data_ptr(), self.pos.data_ptr(),
                                               self.step_ctr.data_ptr()), "finalize")

    # -- public --------------------------------------------------------------
    def set_stream(self, stream):
        check(self._L.affon_b200_ctx_set_stream(self.ctx, stream.cuda_stream))

    def step_eager(self):
        self.set_stream(torch.cuda.current_stream(self.device))
        self._launch_step()

    def capture(self):
        """Capture one decode step into a CUDA graph (one warm-up run first)."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.set_stream(s)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=s):
                self._launch_step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.set_stream(torch.cuda.current_stream(self.device))
        return self.graph

    def replay(self):
        self.graph.replay()

    def reset(self, pos=0):
        self.pos.fill_(pos)
        self.step_ctr.zero_()

    def prefill(self, prompt):
        """Fill the KV cache from a token sequence [T, B] by running decode
        steps with the prompt forced as input (positions 0..T-1)."""
        T = prompt.shape[0]
        self.reset(0)
        prompt = prompt.to(self.device, torch.int32)
        for t in range(T):
            self.tokens.copy_(prompt[t])
            self.replay() if self.graph is not None else self.step_eager()
        self.step_ctr.zero_()

    def close(self):
        if self.ctx:
            self.graph = None
            self._L.affon_b200_ctx_destroy(self.ctx)
            self.ctx = None

    def step_bytes(self, pos):
        """Algorithmic HBM bytes of one decode step at position `pos`: every
        weight once plus the KV rows read by attention."""
        c = self.cfg
        kv = 2 * self.B * c.kv_heads * (pos + 1) * c.head_dim * 2 * c.layers
        return weight_bytes(c) + kv
