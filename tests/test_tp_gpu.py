"""Tensor-parallel decoder on 2 GPUs (one process per GPU, NCCL), against
the same model on one GPU.

Skipped when fewer than two GPUs are visible.  A rank only ever leaves
between steps, with nothing of its own in flight; the other rank learns of
it through the store before its next launch (no collective is left waiting
on a dead peer).  NVLS is off in these child processes.
"""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL_TP = dict(layers=2, d_model=512, q_heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=1024)


def _gpus():
    try:
        return torch.cuda.device_count()
    except Exception:
        return 0


needs2 = pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, *args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(fn, r, port, q, args)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + 240
    while len(out) < 2 and time.time() < deadline:
        try:
            r, res = q.get(timeout=1)
            out[r] = res
        except Exception:
            if not any(p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def _numpy(obj):
    """Results cross the process boundary by value (a torch tensor would be
    shared through a handle that dies with the child)."""
    if isinstance(obj, dict):
        return {k: _numpy(v) for k, v in obj.items()}
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu().numpy()
    return obj


def _entry(fn, rank, port, q, args):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import traceback
    try:
        q.put((rank, _numpy(fn(rank, port, *args))))
    except Exception as e:  # report, do not hang the parent
        q.put((rank, ("error", type(e).__name__, str(e), traceback.format_exc()[-2000:])))


def _group(rank, port):
    import torch.distributed as dist
    from affon_b200 import tp as tpmod
    torch.cuda.set_device(rank)
    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=datetime.timedelta(seconds=60),
                          wait_for_workers=False)
    uid = tpmod.bootstrap_id(store, rank, 2, timeout=60.0)
    return store, uid


def _finish(store, rank):
    store.add("done", 1)
    if rank == 0:
        deadline = time.monotonic() + 60
        while store.add("done", 0) < 2 and time.monotonic() < deadline:
            time.sleep(0.01)


def _tp_vs_single(rank, port, reduce):
    from affon_b200.decoder import LlamaConfig, QuantizedDecoder
    cfg = LlamaConfig(**SMALL_TP)
    store, uid = _group(rank, port)
    dev = torch.device("cuda", rank)
    gen = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, cfg.vocab, (12, 4), generator=gen)
    dec = QuantizedDecoder(cfg, 4, 64, dev, seed=1, max_steps=16, tp=(rank, 2, uid, 60.0), tp_reduce=reduce)
    try:
        dec.prefill(prompt)                         # eager steps, positions 0..11
        dec.synchronize(30.0)
        k_tp = dec.k_cache[:, :, :, :12].float().cpu()
        dec.capture()
        dec.tokens.copy_(prompt[-1].to(dev, torch.int32))
        dec.reset(11)                               # redo position 11 through the graph (teacher-forced)
        dec.replay()
        dec.synchronize(30.0)
        h_tp = dec.h.cpu()
        tok_tp = dec.tokens.cpu()
        for _ in range(2):
            dec.replay()
        dec.synchronize(30.0)
        hist_tp = dec.history[:3].cpu()
    finally:
        dec.close()
    res = {"k": k_tp, "h": h_tp, "tok": tok_tp, "hist": hist_tp}
    if rank == 0:                                   # the same model on one GPU
        ref = QuantizedDecoder(cfg, 4, 64, dev, seed=1, max_steps=16)
        try:
            ref.prefill(prompt)
            ref.capture()
            ref.tokens.copy_(prompt[-1].to(dev, torch.int32))
            ref.reset(11)
            ref.replay()
            ref.synchronize()
            res["ref_h"], res["ref_tok"] = ref.h.cpu(), ref.tokens.cpu()
            res["ref_k"] = ref.k_cache[:, :, :, :12].float().cpu()
            for _ in range(2):
                ref.replay()
            ref.synchronize()
            res["ref_hist"] = ref.history[:3].cpu()
        finally:
            ref.close()
    _finish(store, rank)
    return res


def _peer_leaves(rank, port):
    from affon_b200.core import AffonError
    from affon_b200.decoder import LlamaConfig, QuantizedDecoder
    cfg = LlamaConfig(**SMALL_TP)
    store, uid = _group(rank, port)
    dev = torch.device("cuda", rank)
    dec = QuantizedDecoder(cfg, 2, 16, dev, seed=2, max_steps=8, tp=(rank, 2, uid, 20.0))
    try:
        dec.reset(0)
        dec.step_eager()
        dec.synchronize(20.0)
        store.add("stepped", 1)
        if rank == 1:                               # leave between steps, nothing in flight:
            store.set("left/1", b"1")               # announce it, then abort the group (a rank that
            dec.tp.abort()                          # leaves alone does not finalize with its peers)
            dec.close()
            _finish(store, rank)
            return "left"
        # rank 0: before launching the next step, check the peers on the host
        deadline = time.monotonic() + 20
        while not store.check(["left/1"]) and time.monotonic() < deadline:
            time.sleep(0.01)
        try:
            if store.check(["left/1"]):
                raise AffonError("peer_lost", "tensor-parallel rank 1 left the group")
            dec.step_eager()
            dec.synchronize(10.0)
            return "stepped"
        except AffonError as e:
            dec.tp.abort()                          # nothing of ours is waiting on the peer
            return ("error", e.code)
    finally:
        dec.close()
        if rank == 0:
            _finish(store, rank)


def _fused_allreduce(rank, port):
    """One row-parallel qmv fused with its all-reduce (epilogue 4) on a K
    shard per rank, against the unsharded product on one GPU."""
    import ctypes
    import numpy as np
    from affon_b200 import _lib, synthetic
    from affon_b200 import tp as tpmod
    from affon_b200.core import check
    store, uid = _group(rank, port)
    dev = torch.device("cuda", rank)
    L = _lib.lib()
    ctx = ctypes.c_void_p()
    check(L.affon_b200_ctx_create(rank, None, ctypes.byref(ctx)))
    tpg = tpmod.TensorParallel(ctx, rank, 2, uid, 30.0)
    res = {}
    try:
        check(L.affon_b200_ctx_set_stream(ctx, torch.cuda.current_stream(dev).cuda_stream))
        M, N, K = 16, 4096, 4096
        check(L.affon_b200_tp_exchange_reserve(ctx, M, N))
        d = synthetic.quantized_linear(M, N, K, bits=4, seed=77)
        k0, k1 = tpmod.k_split(K, rank, 2, 4)
        w, sc, b = tpmod.slice_linear_k(d["w"], d["s"], d["b"], k0, k1, 4)
        up = lambda a, t: torch.from_numpy(np.ascontiguousarray(a).view(t)).to(dev)
        x = up(d["x"][:, k0:k1], np.int16)
        wt, st, bt = up(w, np.int32), up(sc, np.int16), up(b, np.int16)
        h = torch.linspace(-1, 1, M * N, device=dev).reshape(M, N).contiguous()
        h0 = h.clone()
        ss = torch.zeros((N // 16, 32), device=dev)
        desc = _lib.QmmDesc()
        desc.struct_size = ctypes.sizeof(_lib.QmmDesc)
        desc.bits, desc.group_size = 4, 64
        desc.x_dtype = desc.param_dtype = desc.y_dtype = _lib.BF16
        Kl = k1 - k0
        desc.x = _lib.View(M, Kl, Kl, 1, 0)
        desc.w = _lib.View(N, Kl // 8, Kl // 8, 1, 0)
        desc.s = desc.b = _lib.View(N, Kl // 64, Kl // 64, 1, 0)
        desc.y = _lib.View(M, N, N, 1, 0)
        for region in (0, 1, 0):                      # three calls: regions alternate, flags reset
            fz = _lib.QmvFusion(struct_size=ctypes.sizeof(_lib.QmvFusion), x_mode=0, epilogue=_lib.EPI_RESID_AR,
                                h_out=h.data_ptr(), ld_h_out=N, ss_out=ss.data_ptr(), exchange_region=region)
            check(L.affon_b200_qmv_fused(ctx, ctypes.byref(desc), x.data_ptr(), wt.data_ptr(), st.data_ptr(),
                                         bt.data_ptr(), None, ctypes.byref(fz)))
        tpg.synchronize(30.0)
        res["h"] = h.cpu()
        res["h0"] = h0.cpu()
        res["ss"] = ss.cpu()
    finally:
        tpg.destroy()
        L.affon_b200_ctx_destroy(ctx)
    if rank == 0:
        import oracle
        d = synthetic.quantized_linear(16, 4096, 4096, bits=4, seed=77)
        res["ref"] = torch.from_numpy(oracle.qmm_dense(d["x"], "bf16", d["w"], d["s"], d["b"], "bf16", 16, 4096,
                                                       4096, 4, 64, threads=oracle.cpu_threads()))
    _finish(store, rank)
    return res


@needs2
def test_tp2_fused_row_parallel_allreduce():
    out = _spawn(_fused_allreduce)
    for r in (0, 1):
        assert not (isinstance(out.get(r), tuple) and out[r][0] == "error"), out.get(r)
    r0, r1 = out[0], out[1]
    np.testing.assert_array_equal(r0["h"], r1["h"])          # replicated, bit for bit
    np.testing.assert_array_equal(r0["ss"], r1["ss"])
    want = r0["h0"] + 3 * r0["ref"]
    assert float(np.abs(r0["h"] - want).max()) <= 1e-4 * max(1.0, float(np.abs(want).max()))


@needs2
@pytest.mark.parametrize("reduce", ["p2p", "nccl"])
def test_tp2_decoder_matches_single_gpu(reduce):
    out = _spawn(_tp_vs_single, reduce)
    for r in (0, 1):
        assert not (isinstance(out.get(r), tuple) and out[r][0] == "error"), out.get(r)
    r0, r1 = out[0], out[1]
    # replicated state is identical on both ranks (same all-reduced sums)
    np.testing.assert_array_equal(r0["h"], r1["h"])
    np.testing.assert_array_equal(r0["hist"], r1["hist"])
    # each rank holds its KV head of the single-GPU cache
    ref_k = r0["ref_k"]
    for r, res in ((0, r0), (1, r1)):
        want = ref_k[:, :, r:r + 1]
        assert float(np.abs(res["k"] - want).max()) <= 2e-2 * max(1.0, float(np.abs(want).max()))
    peak = float(np.abs(r0["ref_h"]).max())
    assert float(np.abs(r0["h"] - r0["ref_h"]).max()) <= 2e-2 * peak
    assert (r0["tok"] == r0["ref_tok"]).mean() >= 0.75


@needs2
def test_tp2_peer_leaving_between_steps_is_detected_on_the_host():
    out = _spawn(_peer_leaves)
    assert out[1] == "left", out
    assert out[0] == ("error", "peer_lost"), out
