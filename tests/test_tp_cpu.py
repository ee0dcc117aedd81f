"""Tensor-parallel host logic on CPU ranks (gloo, world size 2).

No GPU is involved: the group bootstrap runs over a TCP store with
deadlines (a rank that never joins and a corrupted group id must end in an
error, not a hang), and the sharding plan the decoder uses is checked on the
CPU oracle: row-parallel K shards summed by a gloo all-reduce reproduce the
unsharded product, and column-parallel shards concatenate to it exactly.
"""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from affon_b200 import synthetic
from affon_b200 import tp as tpmod
from affon_b200.core import AffonError
from affon_b200.decoder import LLAMA3_8B, LLAMA3_70B, LlamaConfig


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _store(rank, port, timeout=10.0):
    return dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=datetime.timedelta(seconds=timeout),
                         wait_for_workers=False)


def _run(fn, *args):
    """Run fn(rank, port, queue, *args) on two spawned CPU ranks; return
    {rank: result} (exceptions come back as (code, message))."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(fn, r, port, q, args)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + 60
    while len(out) < 2 and time.time() < deadline:
        try:
            r, res = q.get(timeout=1)
            out[r] = res
        except Exception:
            if not any(p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    return out


def _entry(fn, rank, port, q, args):
    try:
        q.put((rank, fn(rank, port, *args)))
    except AffonError as e:
        q.put((rank, ("error", e.code, e.message)))


def _finish(store, rank, world=2, timeout=10.0):
    """Keep rank 0 (the store's server) alive until every rank is done with it."""
    store.add("done", 1)
    if rank == 0:
        deadline = time.monotonic() + timeout
        while store.add("done", 0) < world and time.monotonic() < deadline:
            time.sleep(0.01)


def _good_id():
    return tpmod.seal_id(os.urandom(128))


def _bad_id():
    sealed = bytearray(_good_id())
    sealed[20] ^= 0x40
    return bytes(sealed)


# ------------------------------------------------------------------ rank bodies

def _agree(rank, port):
    store = _store(rank, port)
    try:
        return tpmod.bootstrap_id(store, rank, 2, timeout=10.0, make_id=_good_id).hex()
    finally:
        _finish(store, rank)


def _drop(rank, port):
    if rank == 1:
        return "left"                     # never joins the group
    store = _store(rank, port)
    t0 = time.monotonic()
    try:
        tpmod.bootstrap_id(store, rank, 2, timeout=1.5, make_id=_good_id)
    except AffonError as e:
        return ("error", e.code, e.message, time.monotonic() - t0)
    return "joined"


def _corrupt(rank, port):
    store = _store(rank, port)
    try:
        tpmod.bootstrap_id(store, rank, 2, timeout=5.0, make_id=_bad_id)
        return "accepted"
    finally:
        _finish(store, rank)


def _sharded(rank, port, M, K, N, bits):
    """Row-parallel partials summed over gloo, and column shards gathered."""
    import oracle
    store = _store(rank, port)
    dist.init_process_group("gloo", rank=rank, world_size=2, store=store)
    try:
        data = synthetic.quantized_linear(M, N, K, bits=bits, seed=17)
        x, w, s, b = data["x"], data["w"], data["s"], data["b"]
        k0, k1 = tpmod.k_split(K, rank, 2, bits)
        wk, sk, bk = tpmod.slice_linear_k(w, s, b, k0, k1, bits)
        part = oracle.qmm_dense(np.ascontiguousarray(x[:, k0:k1]), "bf16", np.ascontiguousarray(wk),
                                np.ascontiguousarray(sk), np.ascontiguousarray(bk), "bf16", M, N, k1 - k0, bits, 64)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)                               # the sum exchange the decoder does with NCCL
        n0, n1 = tpmod.even_split(N, rank, 2, 16)
        col = oracle.qmm_dense(x, "bf16", np.ascontiguousarray(w[n0:n1]), np.ascontiguousarray(s[n0:n1]),
                               np.ascontiguousarray(b[n0:n1]), "bf16", M, n1 - n0, K, bits, 64)
        cols = [torch.zeros((M, n1 - n0)) for _ in range(2)]
        dist.all_gather(cols, torch.from_numpy(col.copy()))
        return t.numpy(), torch.cat(cols, dim=1).numpy()
    finally:
        dist.destroy_process_group()


# ----------------------------------------------------------------------- tests

def test_sealed_id_is_checked():
    uid = _good_id()
    tpmod.check_id(uid)                                  # the library's check accepts the Python seal
    with pytest.raises(AffonError) as e:
        tpmod.check_id(_bad_id())
    assert e.value.code == "invalid_arg"
    with pytest.raises(AffonError):
        tpmod.check_id(uid[:100])


def test_bootstrap_two_ranks_agree():
    out = _run(_agree)
    assert set(out) == {0, 1}
    assert out[0] == out[1]


def test_bootstrap_dropped_rank_times_out_without_hanging():
    out = _run(_drop)
    assert out[1] == "left"
    kind, code, msg, waited = out[0]
    assert (kind, code) == ("error", "timeout")
    assert "1" in msg and "did not join" in msg
    assert 1.4 <= waited < 10


def test_bootstrap_rejects_corrupted_id_on_every_rank():
    out = _run(_corrupt)
    for r in (0, 1):
        assert out[r][0] == "error" and out[r][1] == "invalid_arg", out


@pytest.mark.parametrize("bits", [4, 8])
def test_sharded_projection_reproduces_unsharded_oracle(bits):
    import oracle
    M, K, N = 3, 1024, 96
    out = _run(_sharded, M, K, N, bits)
    data = synthetic.quantized_linear(M, N, K, bits=bits, seed=17)
    full = oracle.qmm_dense(data["x"], "bf16", data["w"], data["s"], data["b"], "bf16", M, N, K, bits, 64)
    peak = max(1.0, float(np.abs(full).max()))
    for r in (0, 1):
        row_sum, cols = out[r]
        assert np.abs(row_sum - full).max() <= 1e-5 * peak     # K split: f32 partial sums, reassociated
        np.testing.assert_array_equal(cols, full)              # N split: every output computed alone


def test_shard_plans_of_the_baseline_models():
    for cfg in (LLAMA3_8B, LLAMA3_70B):
        for world in (1, 2, 4, 8):
            tpmod.check_config(cfg, world)
            segs = [tpmod.qkv_row_segments(cfg, r, world) for r in range(world)]
            rows = sorted(i for sg in segs for a, z in sg for i in (a, z))
            assert sum(z - a for sg in segs for a, z in sg) == cfg.qkv_rows
            ks = [tpmod.k_split(cfg.ffn, r, world, cfg.bits) for r in range(world)]
            assert ks[0][0] == 0 and ks[-1][1] == cfg.ffn and all(a % 64 == 0 for a, _ in ks)
            assert rows[0] == 0
    with pytest.raises(AffonError):
        tpmod.check_config(LLAMA3_8B, 3)
    with pytest.raises(AffonError):
        tpmod.check_config(LlamaConfig(layers=1, d_model=512, q_heads=4, kv_heads=1, head_dim=128, ffn=1024,
                                       vocab=1000), 2)
