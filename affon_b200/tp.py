"""Tensor parallelism for the quantized decoder: one process per GPU.

Sharding (per decoder layer; W ranks, rank r):
  * column-parallel (N split, no exchange): QKV by whole heads (query heads
    [r*q/W, (r+1)*q/W) and the matching KV heads), gate/up by SwiGLU column
    (each 16-row tile holds 8 gate rows and their 8 up rows, so a contiguous
    run of tiles is a contiguous slice of both), and the LM head by vocabulary
    rows (the argmax key carries the global row index);
  * row-parallel (K split at 64-group boundaries): O over the local heads'
    columns and down over the local SwiGLU columns, followed by a sum
    all-reduce of the f32 partial outputs.
The packed codes split along K at whole words (64 codes = 8 or 16 words) and
the scales/biases at whole groups; their row stride is padded to 16 bytes so
the decode qmv's tensor maps stay legal (e.g. 14336/8 = 1792 columns = 28
groups, stored 32 wide).

Group set-up: rank 0 creates a sealed NCCL id (library), publishes it
through a key-value store, every rank announces itself and waits for the
others against a deadline; a missing rank or a corrupted id raises
AffonError instead of hanging.  The reference has no multi-device contract
(docs/core/backend-support.md:82); its layer order is
packages/@affon/models/src/llama/model.ts:64-78.
"""
import ctypes
import struct
import time

from . import _lib
from .core import AffonError, check

ID_KEY = "affon_b200/tp/id"
JOIN_KEY = "affon_b200/tp/joined/{}"
_ID_MAGIC = 0x50544641
_ID_VERSION = 1


# ---------------------------------------------------------------------------
# sealed ids

def fnv1a64(data):
    h = 1469598103934665603
    for byte in data:
        h ^= byte
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def seal_id(nccl_id):
    """The sealed form of a 128-byte NCCL unique id (the layout
    affon_b200_tp_unique_id writes): magic, version, id, FNV-1a hash."""
    if len(nccl_id) != 128:
        raise ValueError("an NCCL unique id has 128 bytes")
    head = struct.pack("<II", _ID_MAGIC, _ID_VERSION) + bytes(nccl_id)
    return head + struct.pack("<Q", fnv1a64(head))


def unique_id():
    """A new sealed group id from the library (rank 0 calls this)."""
    buf = ctypes.create_string_buffer(_lib.TP_ID_BYTES)
    check(_lib.lib().affon_b200_tp_unique_id(buf), "tp_unique_id")
    return buf.raw


def check_id(uid):
    """Raise AffonError('invalid_arg') unless `uid` is an intact sealed id."""
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != _lib.TP_ID_BYTES:
        raise AffonError("invalid_arg", f"tp: a group id has {_lib.TP_ID_BYTES} bytes")
    buf = ctypes.create_string_buffer(bytes(uid), len(uid))
    check(_lib.lib().affon_b200_tp_id_check(buf), "tp")


def bootstrap_id(store, rank, world, timeout=30.0, make_id=unique_id, poll=0.01):
    """Agree on a group id through `store` (a torch.distributed Store).

    Rank 0 publishes a sealed id; every rank announces that it joined; each
    waits for the id and for all `world` announcements until `timeout`
    seconds have passed, then raises AffonError('timeout') naming the ranks
    that never came.  A corrupted id raises AffonError('invalid_arg')."""
    if not 0 <= rank < world:
        raise AffonError("invalid_arg", f"tp: rank {rank} outside a group of {world}")
    deadline = time.monotonic() + timeout
    if rank == 0:
        store.set(ID_KEY, make_id())
    store.set(JOIN_KEY.format(rank), b"1")

    def wait_keys(keys, what):
        pending = list(keys)
        while pending:
            pending = [k for k in pending if not store.check([k])]
            if not pending:
                return
            if time.monotonic() > deadline:
                raise AffonError("timeout", f"tp bootstrap: {what(pending)} within {timeout:.1f} s")
            time.sleep(poll)

    wait_keys([ID_KEY], lambda p: "rank 0 published no group id")
    uid = store.get(ID_KEY)
    check_id(uid)
    joins = [JOIN_KEY.format(r) for r in range(world)]
    wait_keys(joins, lambda p: "ranks " + ",".join(k.rsplit("/", 1)[1] for k in p) + " did not join")
    return bytes(uid)


class TensorParallel:
    """This rank's NCCL group, attached to an affon_b200 context (its device
    and stream).  Every wait is bounded by `timeout` seconds."""

    def __init__(self, ctx, rank, world, uid, timeout=60.0):
        self.ctx, self.rank, self.world, self.timeout = ctx, rank, world, timeout
        check_id(uid)
        buf = ctypes.create_string_buffer(bytes(uid), len(uid))
        check(_lib.lib().affon_b200_tp_init(ctx, rank, world, buf, ctypes.c_double(timeout)), "tp_init")

    def allreduce(self, tensor, op="sum"):
        """In place on the context's stream: f32/bf16 sum or int64 (u64) max."""
        import torch
        dt = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.int64: _lib.U64}[tensor.dtype]
        check(_lib.lib().affon_b200_tp_allreduce(self.ctx, tensor.data_ptr(), tensor.numel(), dt,
                                                 _lib.REDUCE_SUM if op == "sum" else _lib.REDUCE_MAX), "tp_allreduce")

    def synchronize(self, timeout=0.0):
        check(_lib.lib().affon_b200_tp_synchronize(self.ctx, ctypes.c_double(timeout)), "tp_synchronize")

    def abort(self):
        _lib.lib().affon_b200_tp_abort(self.ctx)

    def destroy(self):
        if self.ctx:
            _lib.lib().affon_b200_tp_destroy(self.ctx)
            self.ctx = None


# ---------------------------------------------------------------------------
# sharding plan (used by the decoder and checked on the CPU oracle)

def even_split(total, rank, world, multiple=1):
    """[start, stop) of this rank's equal share of `total`, in units of `multiple`."""
    if total % (world * multiple):
        raise AffonError("invalid_shape", f"tp: {total} does not split into {world} shares of whole {multiple}s")
    share = total // world
    return rank * share, (rank + 1) * share


def check_config(cfg, world):
    """The BASELINE decoders shard at TP 1/2/4/8: heads, SwiGLU columns and the
    vocabulary must split evenly, and K shards must stay whole 128-byte
    packed stages of the decode qmv."""
    stage = 256 if cfg.bits == 4 else 128
    if cfg.kv_heads % world or cfg.q_heads % world:
        raise AffonError("invalid_shape", f"tp: {cfg.kv_heads} KV heads do not split over {world} ranks")
    if (cfg.ffn // world) % max(stage, 16) or cfg.ffn % world:
        raise AffonError("invalid_shape", f"tp: ffn {cfg.ffn} does not split into whole qmv stages over {world}")
    if (cfg.q_heads // world * cfg.head_dim) % stage:
        raise AffonError("invalid_shape", "tp: the O projection's K shard is not a whole qmv stage")
    if cfg.vocab % (16 * world):
        raise AffonError("invalid_shape", f"tp: vocab {cfg.vocab} does not split into 16-row tiles over {world}")


def qkv_row_segments(cfg, rank, world):
    """Rows of the full [q; k; v] projection that this rank holds, as
    (start, stop) segments: its query heads, then its KV heads' keys and values."""
    hd = cfg.head_dim
    q0, q1 = even_split(cfg.q_heads, rank, world)
    k0, k1 = even_split(cfg.kv_heads, rank, world)
    qn, kn = cfg.q_heads * hd, cfg.kv_heads * hd
    return [(q0 * hd, q1 * hd), (qn + k0 * hd, qn + k1 * hd), (qn + kn + k0 * hd, qn + kn + k1 * hd)]


def k_split(K, rank, world, bits, group=64):
    """This rank's [k0, k1) of a row-parallel projection, at group and word boundaries."""
    return even_split(K, rank, world, multiple=max(group, 32 // bits))


def slice_linear_k(w, s, b, k0, k1, bits, group=64):
    """Packed codes and parameters of columns [k0, k1) (views, no copy)."""
    per = 32 // bits
    return w[:, k0 // per:k1 // per], s[:, k0 // group:k1 // group], b[:, k0 // group:k1 // group]


def padded_groups(groups):
    """Row stride (in bf16 elements) for `groups` scales: a multiple of 8 (16 bytes)."""
    return (groups + 7) // 8 * 8
