"""Synthetic Llama-shaped decoder on the affon_b200 kernels.

Every projection is a 4-bit (or 8-bit) affine group-quantized linear
(`quantized_matmul` layout: codes packed little-endian into u32 along K,
group 64, bf16 scale and bias), run by the decode qmv with the decoder's
residual adds, SiLU-gated product and final argmax fused into its epilogue.
RMSNorm is fused: the embedding and each residual epilogue write the next
projection's activations as bf16(h * gamma) in the qmv's column order, and
that qmv multiplies each output row by rsqrt(mean(h^2) + eps), computed from
the per-16-column sums of squares the same epilogue leaves; attention and the
SiLU epilogue write their outputs in that order directly.
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

Tensor parallelism (`tp=(rank, world, group_id)`, one process per GPU): the
full model is generated identically on every rank and each rank keeps its
shard (affon_b200.tp describes the split).  QKV, gate/up and the LM head are
column-parallel; O and down are row-parallel.  By default (`tp_reduce="p2p"`)
each row-parallel qmv is fused with its all-reduce: it pushes its f32 rows
into every rank's exchange buffer over NVLink, waits (bounded) for the other
ranks' rows, sums them in rank order and applies the residual epilogue, so a
step has the same five launches per layer as on one GPU.  `tp_reduce="nccl"`
runs an NCCL sum all-reduce of the partial outputs and a residual-add +
RMSNorm kernel instead.  The LM head's local argmax keys carry global
vocabulary indices and an NCCL max all-reduce picks the winner, so every rank
samples the same tokens.

A decode step is captured once in a CUDA graph: the current position,
step counter and tokens live in device memory and are advanced by the last
kernel, so replays run back to back with no host work.  `overlap=True` (the
default) runs the context in overlap mode (programmatic dependent launch:
each kernel of the step may start while the previous one finishes and
stream its weights ahead of the activations it waits for); the captured 8B
step measured 4.26 ms with it and 4.45 ms without.
"""
import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib
from . import tp as tpmod
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
    """Device tensors of one quantized linear [N, K] (+ its descriptor).
    Scales and biases are [N, ld_s] with ld_s >= K/group (16-byte rows)."""

    def __init__(self, N, K, bits, group, gen, device):
        per = 32 // bits
        self.N, self.K, self.bits, self.group = N, K, bits, group
        self.w = torch.randint(-2 ** 31, 2 ** 31 - 1, (N, K // per), generator=gen, device=device, dtype=torch.int32)
        s = torch.randn((N, K // group), generator=gen, device=device).abs() * 0.02 + 1e-3
        self.s = s.to(torch.bfloat16)
        self.b = (self.s.float() * -(1 << (bits - 1))).to(torch.bfloat16)
        self.ld_s = K // group

    def shard(self, rows=None, k=None):
        """A copy holding rows `rows` ((start, stop) segments, concatenated) and
        columns k = (k0, k1) (whole groups); scale rows padded to 16 bytes."""
        w, s, b = self.w, self.s, self.b
        if rows is not None:
            w = torch.cat([w[a:z] for a, z in rows])
            s = torch.cat([s[a:z] for a, z in rows])
            b = torch.cat([b[a:z] for a, z in rows])
        K = self.K
        if k is not None:
            w, s, b = tpmod.slice_linear_k(w, s, b, k[0], k[1], self.bits, self.group)
            K = k[1] - k[0]
        out = object.__new__(QuantLinear)
        out.N, out.K, out.bits, out.group = w.shape[0], K, self.bits, self.group
        out.w = w.contiguous()
        groups = K // self.group
        out.ld_s = tpmod.padded_groups(groups)
        out.s = torch.zeros((out.N, out.ld_s), dtype=torch.bfloat16, device=w.device)
        out.b = torch.zeros_like(out.s)
        out.s[:, :groups] = s
        out.b[:, :groups] = b
        return out

    def desc(self, M, ld_x=None, y_dtype=_lib.BF16, x_dtype=_lib.BF16):
        per = 32 // self.bits
        d = _lib.QmmDesc()
        d.struct_size = ctypes.sizeof(_lib.QmmDesc)
        d.bits, d.group_size = self.bits, self.group
        d.x_dtype, d.param_dtype, d.y_dtype = x_dtype, _lib.BF16, y_dtype
        d.numerical_policy = _lib.POLICY["backend_equivalent"]
        d.x = _lib.View(M, self.K, ld_x or self.K, 1, 0)
        d.w = _lib.View(self.N, self.K // per, self.K // per, 1, 0)
        d.s = d.b = _lib.View(self.N, self.K // self.group, self.ld_s, 1, 0)
        d.y = _lib.View(M, self.N, self.N, 1, 0)
        return d

    def dequantized(self):
        """float32 [N, K] decoded weight (for reference checks)."""
        per = 32 // self.bits
        words = self.w.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        shifts = torch.arange(per, device=words.device, dtype=torch.int64) * self.bits
        codes = ((words.unsqueeze(-1) >> shifts) & ((1 << self.bits) - 1)).reshape(self.N, self.K).float()
        g = self.K // self.group
        s = self.s[:, :g].float().repeat_interleave(self.group, dim=1)
        b = self.b[:, :g].float().repeat_interleave(self.group, dim=1)
        return codes * s + b


def rope_tables(cfg, capacity, device):
    half = cfg.head_dim // 2
    inv = cfg.rope_theta ** (-torch.arange(half, dtype=torch.float64) * 2.0 / cfg.head_dim)
    ang = torch.arange(capacity, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float().to(device).contiguous(), torch.sin(ang).float().to(device).contiguous()


class QuantizedDecoder:
    """Batch-`batch` greedy decoder with a KV cache of `capacity` positions.

    tp: None for one GPU, or (rank, world, group_id[, timeout_s]) to hold this
    rank's shard of a tensor-parallel decoder (group_id from
    affon_b200.tp.unique_id on rank 0, shared with every rank)."""

    def __init__(self, cfg, batch, capacity, device, seed=0, max_steps=4096, workspace_bytes=None, overlap=True,
                 tp=None, tp_reduce="p2p"):
        if batch > _lib.MAX_QMV_ROWS:
            raise ValueError(f"decode qmv handles up to {_lib.MAX_QMV_ROWS} rows per step")
        self.cfg, self.B, self.cap = cfg, batch, capacity
        self.device = torch.device(device)
        rank, world = (tp[0], tp[1]) if tp else (0, 1)
        self.rank, self.world = rank, world
        if world > 1:
            tpmod.check_config(cfg, world)
        dev = self.device
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        c = cfg
        q_l, kv_l = c.q_heads // world, c.kv_heads // world
        self.q_heads_local, self.kv_heads_local = q_l, kv_l
        ko = tpmod.k_split(c.q_heads * c.head_dim, rank, world, c.bits) if world > 1 else None
        f0, f1 = tpmod.even_split(c.ffn, rank, world)
        kd = (f0, f1) if world > 1 else None
        v0, v1 = tpmod.even_split(c.vocab, rank, world)
        self.vocab_offset = v0
        shard = (lambda lin, **kw: lin.shard(**kw)) if world > 1 else (lambda lin, **kw: lin)
        self.embed = (torch.randn((c.vocab, c.d_model), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        gamma = lambda: (1.0 + 0.1 * torch.randn((c.d_model,), generator=gen, device=dev)).to(torch.bfloat16)
        self.layers = []
        for _ in range(c.layers):
            attn_norm = gamma()
            qkv = shard(QuantLinear(c.qkv_rows, c.d_model, c.bits, c.group, gen, dev),
                        rows=tpmod.qkv_row_segments(c, rank, world))
            o = shard(QuantLinear(c.d_model, c.q_heads * c.head_dim, c.bits, c.group, gen, dev), k=ko)
            ffn_norm = gamma()
            gu = shard(QuantLinear(2 * c.ffn, c.d_model, c.bits, c.group, gen, dev), rows=[(2 * f0, 2 * f1)])
            down = shard(QuantLinear(c.d_model, c.ffn, c.bits, c.group, gen, dev), k=kd)
            self.layers.append({"attn_norm": attn_norm, "qkv": qkv, "o": o, "ffn_norm": ffn_norm, "gate_up": gu,
                                "down": down})
        self.final_norm = gamma()
        self.lm_head = shard(QuantLinear(c.vocab, c.d_model, c.bits, c.group, gen, dev), rows=[(v0, v1)])
        kv_shape = (c.layers, batch, kv_l, capacity, c.head_dim)
        self.k_cache = torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev)
        self.cos, self.sin = rope_tables(c, capacity, dev)
        # step state (device)
        self.tokens = torch.zeros((batch,), dtype=torch.int32, device=dev)
        self.pos = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.step_ctr = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.history = torch.zeros((max_steps, batch), dtype=torch.int32, device=dev)  # ring of the last steps
        self.h = torch.zeros((batch, c.d_model), dtype=torch.float32, device=dev)
        self.ss = torch.zeros((c.d_model // 16, _lib.SS_WIDTH), dtype=torch.float32, device=dev)
        self.xq = torch.zeros((batch, c.d_model), dtype=torch.bfloat16, device=dev)   # normalized x, qmv order
        self.qkv = torch.zeros((batch, (q_l + 2 * kv_l) * c.head_dim), dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros((batch, q_l * c.head_dim), dtype=torch.bfloat16, device=dev)
        self.act = torch.zeros((batch, f1 - f0), dtype=torch.bfloat16, device=dev)
        self.amax = torch.zeros((batch,), dtype=torch.int64, device=dev)
        self.y = torch.zeros((batch, c.d_model), dtype=torch.float32, device=dev)     # row-parallel partial sums
        L = _lib.lib()
        self._L = L
        self.ctx = ctypes.c_void_p()
        check(L.affon_b200_ctx_create(dev.index, None, ctypes.byref(self.ctx)), "decoder context")
        if workspace_bytes:
            check(L.affon_b200_ctx_reserve_workspace(self.ctx, int(workspace_bytes)))
        # The step's kernels never write weights, so overlap mode is safe here.
        self._overlap = overlap
        check(L.affon_b200_ctx_set_overlap(self.ctx, 1 if overlap else 0))
        self.tp = None
        if tp_reduce not in ("p2p", "nccl"):
            raise ValueError("tp_reduce must be 'p2p' or 'nccl'")
        self.tp_reduce = tp_reduce if world > 1 else None
        if world > 1:
            self.tp = tpmod.TensorParallel(self.ctx, rank, world, tp[2], *(tp[3:4] or [60.0]))
            if tp_reduce == "p2p":
                check(L.affon_b200_tp_exchange_reserve(self.ctx, batch, c.d_model), "tp_exchange_reserve")
        self._build_calls()
        self.graph = None
        self._pos_host = 0   # host copy of the device position, to refuse steps beyond capacity

    # -- launch descriptors --------------------------------------------------
    def _build_calls(self):
        c, B = self.cfg, self.B
        hd = c.head_dim
        q_l, kv_l = self.q_heads_local, self.kv_heads_local
        self.attn_desc = _lib.AttnDesc(ctypes.sizeof(_lib.AttnDesc), B, q_l, kv_l, hd, self.cap,
                                       1.0 / math.sqrt(hd), 0, q_l * hd, (q_l + kv_l) * hd, 0,
                                       (q_l + 2 * kv_l) * hd, q_l * hd)
        ptr = lambda t: ctypes.c_void_p(t.data_ptr())
        pair = 1 if c.bits == 4 else 0          # producers write the 4-bit qmv's pair order
        self.attn_desc.out_pair_order = pair
        fz = lambda **kw: _lib.QmvFusion(struct_size=ctypes.sizeof(_lib.QmvFusion), x_mode=1, **kw)
        # RMSNorm fused into the consumer: x = bf16(h * gamma) written by the
        # embedding or the previous residual epilogue, and the consumer qmv
        # scales each output row by rsqrt(mean(h^2) + eps) from the sums of
        # squares (row-scale mode).
        scaled = dict(row_ss=ptr(self.ss), ss_tiles=c.d_model // 16, eps=c.eps)
        silu = dict(epilogue=_lib.EPI_SILU_MUL, act=ptr(self.act), ld_act=self.act.shape[1], act_pair_order=pair)
        xq = ptr(self.xq)
        self.calls = []
        tp = self.world > 1
        nccl = self.tp_reduce == "nccl"
        resid = lambda gamma, region=None: dict(
            epilogue=_lib.EPI_RESID if region is None else _lib.EPI_RESID_AR, h_out=ptr(self.h), ld_h_out=c.d_model,
            ss_out=ptr(self.ss), next_gamma=ptr(gamma), next_x=xq, ld_next_x=c.d_model, next_pair_order=pair,
            exchange_region=region or 0)
        self.embed_gamma = self.layers[0]["attn_norm"]
        for i, lay in enumerate(self.layers):
            q, o, gu, dn = lay["qkv"], lay["o"], lay["gate_up"], lay["down"]
            nxt = self.layers[i + 1]["attn_norm"] if i + 1 < len(self.layers) else self.final_norm
            # QKV and gate/up read bf16(h * gamma) and apply the row scale,
            # except after an NCCL all-reduce (resid_norm writes normalised x)
            qkv_scaled = (not nccl) or i == 0
            self.calls.append(("qmv", q.desc(B), xq, q, ptr(self.qkv),
                               fz(epilogue=_lib.EPI_STORE, **(scaled if qkv_scaled else {}))))
            self.calls.append(("attn", i))
            if nccl:
                self.calls.append(("qmv", o.desc(B, y_dtype=_lib.F32), ptr(self.attn), o, ptr(self.y),
                                   fz(epilogue=_lib.EPI_STORE)))
                self.calls.append(("allreduce", self.y, "sum"))
                self.calls.append(("resid_norm", lay["ffn_norm"]))
                self.calls.append(("qmv", gu.desc(B), xq, gu, None, fz(**silu)))
                self.calls.append(("qmv", dn.desc(B, y_dtype=_lib.F32), ptr(self.act), dn, ptr(self.y),
                                   fz(epilogue=_lib.EPI_STORE)))
                self.calls.append(("allreduce", self.y, "sum"))
                self.calls.append(("resid_norm", nxt))
            else:
                # row-parallel O and down fused with their all-reduce under
                # tensor parallelism (exchange regions alternate)
                self.calls.append(("qmv", o.desc(B), ptr(self.attn), o, None,
                                   fz(**resid(lay["ffn_norm"], 0 if tp else None))))
                self.calls.append(("qmv", gu.desc(B), xq, gu, None, fz(**silu, **scaled)))
                self.calls.append(("qmv", dn.desc(B), ptr(self.act), dn, None,
                                   fz(**resid(nxt, 1 if tp else None))))
        lm = self.lm_head
        self.calls.append(("qmv", lm.desc(B), xq, lm, None,
                           fz(epilogue=_lib.EPI_ARGMAX, amax=ptr(self.amax), index_offset=self.vocab_offset,
                              **({} if nccl else scaled))))
        if tp:
            self.calls.append(("allreduce", self.amax, "max"))
        self._kv_layer = [(self.k_cache[i], self.v_cache[i]) for i in range(c.layers)]

    def launches_per_step(self):
        """affon_b200 kernels one decode step launches: embed, one per call
        except the NCCL all-reduces, finalize."""
        return 2 + sum(1 for cl in self.calls if cl[0] != "allreduce")

    def _launch_step(self, finalize=True, events=None):
        L, ctx = self._L, self.ctx
        c = self.cfg
        stream = torch.cuda.current_stream(self.device) if events else None
        mark = (lambda i: events[i].record(stream)) if events else (lambda i: None)
        check(L.affon_b200_embed(ctx, self.embed.data_ptr(), c.d_model, c.vocab, self.tokens.data_ptr(), self.B,
                                 c.d_model, self.h.data_ptr(), self.ss.data_ptr(), self.amax.data_ptr(),
                                 self.embed_gamma.data_ptr(), self.xq.data_ptr(), c.d_model,
                                 1 if c.bits == 4 else 0), "embed")
        mark(1)
        for ci, call in enumerate(self.calls):
            kind = call[0]
            if kind == "norm":
                check(L.affon_b200_qmv_prep(ctx, 1, self.h.data_ptr(), c.d_model, self.ss.data_ptr(), c.d_model // 16,
                                            call[1].data_ptr(), ctypes.c_float(c.eps), self.B, c.d_model, c.bits,
                                            self.xq.data_ptr(), c.d_model), "qmv_prep")
            elif kind == "resid_norm":
                check(L.affon_b200_resid_norm(ctx, self.h.data_ptr(), c.d_model, self.y.data_ptr(), c.d_model,
                                              call[1].data_ptr(), ctypes.c_float(c.eps), self.B, c.d_model, c.bits,
                                              self.xq.data_ptr(), c.d_model), "resid_norm")
            elif kind == "allreduce":
                self.tp.allreduce(call[1], call[2])
            elif kind == "attn":
                kc, vc = self._kv_layer[call[1]]
                check(L.affon_b200_decode_attention(ctx, ctypes.byref(self.attn_desc), self.qkv.data_ptr(),
                                                    kc.data_ptr(), vc.data_ptr(), self.cos.data_ptr(),
                                                    self.sin.data_ptr(), self.pos.data_ptr(), self.attn.data_ptr()),
                      "decode_attention")
            else:
                _, desc, x, lin, y, fus = call
                check(L.affon_b200_qmv_fused(ctx, ctypes.byref(desc), x, lin.w.data_ptr(), lin.s.data_ptr(),
                                             lin.b.data_ptr(), y, ctypes.byref(fus)), "qmv_fused")
            mark(ci + 2)
        if finalize or events:
            check(L.affon_b200_argmax_finalize(ctx, self.amax.data_ptr(), self.B, self.tokens.data_ptr(),
                                               self.history.data_ptr(), self.history.shape[0], self.pos.data_ptr(),
                                               self.step_ctr.data_ptr()), "finalize")
            mark(len(self.calls) + 2)

    # -- public --------------------------------------------------------------
    def set_stream(self, stream):
        check(self._L.affon_b200_ctx_set_stream(self.ctx, stream.cuda_stream))

    def _advance(self):
        if self._pos_host >= self.cap:
            raise ValueError(f"KV cache full: position {self._pos_host} of capacity {self.cap}")
        self._pos_host += 1

    def step_eager(self):
        self._advance()
        self.set_stream(torch.cuda.current_stream(self.device))
        self._launch_step()

    def capture(self):
        """Capture one decode step into a CUDA graph."""
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
        self._advance()
        self.graph.replay()

    def reset(self, pos=0):
        if not 0 <= pos <= self.cap:
            raise ValueError(f"position {pos} outside the KV cache (capacity {self.cap})")
        self.pos.fill_(pos)
        self.step_ctr.zero_()
        self._pos_host = pos

    def synchronize(self, timeout=0.0):
        """Wait for the step's stream and raise if a kernel reported a device-side
        failure (a bounded wait that gave up, a position or token out of range)
        or, under tensor parallelism, the group failed or timed out."""
        if self.tp is not None:
            self.tp.synchronize(timeout)
        else:
            check(self._L.affon_b200_ctx_synchronize(self.ctx), "decoder")

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

    def fill_kv_random(self, T, seed=0):
        """Synthetic KV cache: positions 0..T-1 of every layer hold N(0,1)
        bf16 keys and values (for throughput runs that do not need the cache
        a real prompt would leave), and the position moves to T."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        for t in (self.k_cache, self.v_cache):
            for li in range(t.shape[0]):
                t[li, :, :, :T].normal_(generator=g)
        self.reset(T)

    def _roles(self):
        names = []
        for call in self.calls:
            if call[0] == "qmv":
                lin = call[3]
                role = "lm_head" if lin is self.lm_head else next(k for k in ("qkv", "o", "gate_up", "down")
                                                                    if any(l[k] is lin for l in self.layers))
                names.append(role)
            else:
                names.append(call[0])
        return names

    def _role_launch(self, role, lins):
        """A launch function for one kernel role (rotating over layers)."""
        L, ctx, c = self._L, self.ctx, self.cfg
        idx = [0]

        def nxt(seq):
            v = seq[idx[0] % len(seq)]
            idx[0] += 1
            return v
        if role == "attn":
            return lambda: check(L.affon_b200_decode_attention(
                ctx, ctypes.byref(self.attn_desc), self.qkv.data_ptr(), *[t.data_ptr() for t in nxt(self._kv_layer)],
                self.cos.data_ptr(), self.sin.data_ptr(), self.pos.data_ptr(), self.attn.data_ptr()))
        if role == "norm":
            gammas = [l["attn_norm"] for l in self.layers]
            return lambda: check(L.affon_b200_qmv_prep(
                ctx, 1, self.h.data_ptr(), c.d_model, self.ss.data_ptr(), c.d_model // 16, nxt(gammas).data_ptr(),
                ctypes.c_float(c.eps), self.B, c.d_model, c.bits, self.xq.data_ptr(), c.d_model))
        if role == "resid_norm":
            gammas = [l["ffn_norm"] for l in self.layers]
            zero = torch.zeros_like(self.y)
            return lambda: check(L.affon_b200_resid_norm(
                ctx, self.h.data_ptr(), c.d_model, zero.data_ptr(), c.d_model, nxt(gammas).data_ptr(),
                ctypes.c_float(c.eps), self.B, c.d_model, c.bits, self.xq.data_ptr(), c.d_model))
        if role == "allreduce":
            return lambda: self.tp.allreduce(self.y, "sum")
        if role == "embed":
            return lambda: check(L.affon_b200_embed(ctx, self.embed.data_ptr(), c.d_model, c.vocab,
                                                    self.tokens.data_ptr(), self.B, c.d_model, self.h.data_ptr(),
                                                    self.ss.data_ptr(), self.amax.data_ptr(),
                                                    self.embed_gamma.data_ptr(), self.xq.data_ptr(), c.d_model,
                                                    1 if c.bits == 4 else 0))
        if role == "finalize":
            def fin():
                check(L.affon_b200_argmax_finalize(ctx, self.amax.data_ptr(), self.B, self.tokens.data_ptr(), None, 0,
                                                   self._scratch_pos.data_ptr(), self._scratch_step.data_ptr()))
            return fin
        call = next(cl for cl in self.calls if cl[0] == "qmv" and cl[3] is lins[0])
        _, desc, x, _, y, fus = call
        return lambda: (lambda lin: check(L.affon_b200_qmv_fused(ctx, ctypes.byref(desc), x, lin.w.data_ptr(),
                                                                 lin.s.data_ptr(), lin.b.data_ptr(), y,
                                                                 ctypes.byref(fus))))(nxt(lins))

    def role_time_ms(self, role, reps=32):
        """Average device time of one launch of a step kernel, from a CUDA
        graph of `reps` back-to-back launches that rotate over the layers'
        weights (or KV caches), so each launch reads HBM; overlap mode off.
        Roles: qkv, o, gate_up, down, lm_head, attn, norm, resid_norm,
        allreduce, embed, finalize.  Leaves the decoder's state as it was."""
        L = self._L
        lins = ([self.lm_head] if role == "lm_head" else
                [l[role] for l in self.layers] if role in ("qkv", "o", "gate_up", "down") else None)
        self._scratch_pos = self.pos.clone()
        self._scratch_step = self.step_ctr.clone()
        saved = [t.clone() for t in (self.h, self.ss, self.xq, self.qkv, self.attn, self.act, self.amax, self.y,
                                     self.tokens)]
        launch = self._role_launch(role, lins)
        if role == "lm_head":
            reps = 8
        dev = self.device
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        check(L.affon_b200_ctx_set_overlap(self.ctx, 0))
        try:
            with torch.cuda.stream(s):
                self.set_stream(s)
                launch()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for _ in range(reps):
                        launch()
            torch.cuda.current_stream(dev).wait_stream(s)
            self.set_stream(torch.cuda.current_stream(dev))
            g.replay()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize(dev)
            del g
            return e0.elapsed_time(e1) / reps
        finally:
            check(L.affon_b200_ctx_set_overlap(self.ctx, 1 if self._overlap else 0))
            self.set_stream(torch.cuda.current_stream(dev))
            for t, v in zip((self.h, self.ss, self.xq, self.qkv, self.attn, self.act, self.amax, self.y,
                             self.tokens), saved):
                t.copy_(v)

    def launches_by_role(self):
        """How many launches of each role one decode step makes."""
        counts = {"embed": 1, "finalize": 1}
        for r in self._roles():
            counts[r] = counts.get(r, 0) + 1
        return counts

    def step_breakdown(self):
        """Per-role device time of one decode step: each role's launch time
        alone (role_time_ms) times its launches per step, in ms."""
        counts = self.launches_by_role()
        return {r: (self.role_time_ms(r) * n, n) for r, n in counts.items()}

    def close(self):
        if self.ctx:
            self.graph = None
            if self.tp is not None:
                self.tp.destroy()
                self.tp = None
            self._L.affon_b200_ctx_destroy(self.ctx)
            self.ctx = None

    def step_bytes(self, pos):
        """Algorithmic HBM bytes of one decode step at position `pos` on this
        rank: its shard of every weight once plus the KV rows its attention reads."""
        c = self.cfg
        kv = 2 * self.B * self.kv_heads_local * (pos + 1) * c.head_dim * 2 * c.layers
        return weight_bytes(c) // self.world + kv
