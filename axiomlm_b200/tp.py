"""Tensor parallelism of the quantized decoder over NVLink.

The 8B-shaped decoder runs column-parallel QKV (by heads: each rank owns
n_head / world query heads and n_kv_head / world KV heads, so attention needs
no exchange), column-parallel gate_up (by FFN rows) and lm_head (by vocab
rows), and row-parallel o / down projections whose fp32 partial sums meet in
one NCCL allreduce each (two per layer), inside the runner's CUDA graph.  The
greedy token is the max over ranks of packed (logit, -index) keys: the lowest
index wins a tie, as ``torch.argmax``.  RMSNorm, the residual stream and the
embedding table are replicated.

The reference has no inference-time parallelism (its only collective is a
training ``all_reduce``, axiomlm/train.py:296); this module is the B200
build's own multi-GPU mode, next to batch-sharded replicas.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L

ID_BYTES = 128


class TensorParallel:
    """One rank's NCCL communicator for tensor-parallel decode (current CUDA
    device).  Build it with ``from_process_group`` under ``torch.distributed``
    or directly from a shared 128-byte unique id."""

    def __init__(self, rank: int, world: int, unique_id: bytes):
        if len(unique_id) != ID_BYTES:
            raise ValueError(f"unique id must be {ID_BYTES} bytes")
        self.rank, self.world = rank, world
        buf = (C.c_char * ID_BYTES).from_buffer_copy(unique_id)
        h = C.c_void_p()
        L.call("axb_tp_comm_create", C.cast(buf, C.c_void_p), world, rank, C.byref(h))
        self._comm = h

    @staticmethod
    def new_unique_id() -> bytes:
        buf = (C.c_char * ID_BYTES)()
        L.call("axb_tp_unique_id", C.cast(buf, C.c_void_p))
        return bytes(buf)

    @classmethod
    def from_process_group(cls, group=None, id_fn=None) -> "TensorParallel":
        """Rank 0 of ``group`` makes the unique id and broadcasts it (any
        torch.distributed backend, gloo included)."""
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        obj = [(id_fn or cls.new_unique_id)() if rank == 0 else None]
        src = 0 if group is None else dist.get_global_rank(group, 0)
        dist.broadcast_object_list(obj, src=src, group=group)
        return cls(rank, world, obj[0])

    @property
    def comm(self) -> int:
        return self._comm.value or 0

    def all_reduce_(self, t: torch.Tensor, op: str = "sum") -> torch.Tensor:
        """In-place allreduce on the current stream: fp32 / fp16 sum, uint64
        (int64 storage) max."""
        if not t.is_cuda or not t.is_contiguous():
            raise RuntimeError("all_reduce_ needs a contiguous CUDA tensor")
        code = {("sum", torch.float32): L.TP_SUM_F32, ("sum", torch.float16): L.TP_SUM_F16,
                ("max", torch.int64): L.TP_MAX_U64}.get((op, t.dtype))
        if code is None:
            raise ValueError(f"unsupported allreduce ({op}, {t.dtype})")
        L.call("axb_tp_allreduce", self._comm, C.c_void_p(t.data_ptr()), t.numel(), code,
               C.c_void_p(torch.cuda.current_stream().cuda_stream))
        return t

    def abort(self):
        """Abandon the communicator (a peer is gone); pending collectives end."""
        if self._comm:
            L.call("axb_tp_comm_abort", self._comm)
            self._comm = C.c_void_p()

    def close(self):
        if self._comm:
            L.call("axb_tp_comm_destroy", self._comm)
            self._comm = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def local_dims(cfg: dict, world: int) -> dict:
    """This rank's shard sizes; every sharded dimension must divide evenly."""
    H, Hkv, F, V = cfg["n_head"], cfg["n_kv_head"], cfg["ffn"], cfg["vocab"]
    for name, v in (("n_head", H), ("n_kv_head", Hkv), ("ffn", F), ("vocab", V)):
        if v % world:
            raise ValueError(f"{name}={v} is not divisible by the tensor-parallel world {world}")
    if (F // world) % 64:
        raise ValueError(f"ffn / world = {F // world} must be a multiple of 64")
    return dict(cfg, n_head=H // world, n_kv_head=Hkv // world, ffn=F // world, vocab=V // world,
                head_dim=cfg["d_model"] // H)


def shard_weights(cfg: dict, W: dict, rank: int, world: int) -> dict:
    """Slice fp32 master weights (c_attn rows [q; k; v], c_proj, w_gate, w_up,
    w_down, lm_head; the layout of ``tests/golden/model_weights``) to this
    rank's shard.  The embedding and the norms stay whole."""
    d, H, Hkv, F, V = cfg["d_model"], cfg["n_head"], cfg["n_kv_head"], cfg["ffn"], cfg["vocab"]
    hd = d // H
    hl, kl, fl, vl = H // world, Hkv // world, F // world, V // world
    out = {"wte": W["wte"], "ln_f": W["ln_f"], "layers": []}
    for lw in W["layers"]:
        qkv = lw["c_attn"]
        q = qkv[rank * hl * hd:(rank + 1) * hl * hd]
        k = qkv[H * hd + rank * kl * hd:H * hd + (rank + 1) * kl * hd]
        v = qkv[(H + Hkv) * hd + rank * kl * hd:(H + Hkv) * hd + (rank + 1) * kl * hd]
        out["layers"].append(dict(
            c_attn=torch.cat([q, k, v], 0).contiguous(),
            c_proj=lw["c_proj"][:, rank * hl * hd:(rank + 1) * hl * hd].contiguous(),
            w_gate=lw["w_gate"][rank * fl:(rank + 1) * fl].contiguous(),
            w_up=lw["w_up"][rank * fl:(rank + 1) * fl].contiguous(),
            w_down=lw["w_down"][:, rank * fl:(rank + 1) * fl].contiguous(),
            ln_1=lw["ln_1"], ln_2=lw["ln_2"]))
    lm = W.get("lm_head")
    out["lm_head"] = None if lm is None else lm[rank * vl:(rank + 1) * vl].contiguous()
    return out


def argmax_key(value: float, index: int) -> int:
    """The packed key the ranks' winners meet in (max): ordered fp32 bits of
    the fp16 logit, then the complement of the global index."""
    import struct

    bits = struct.unpack("<I", struct.pack("<f", float(value)))[0]
    bits = (~bits & 0xFFFFFFFF) if bits & 0x80000000 else (bits | 0x80000000)
    return (bits << 32) | (0xFFFFFFFF - index)
