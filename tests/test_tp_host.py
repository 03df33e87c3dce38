"""Host-side logic of the tensor-parallel decoder (no GPU): weight sharding,
the argmax key rule, and the unique-id exchange over a gloo process group of
two CPU ranks."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from model_weights import make_weights

MID = dict(n_layer=2, d_model=256, n_head=8, n_kv_head=4, ffn=512, vocab=1024, eps=1e-5, theta=10000.0,
           block_size=256)


@pytest.mark.parametrize("world", [2, 4])
def test_shards_reassemble_the_model(world):
    from axiomlm_b200.tp import local_dims, shard_weights

    W = make_weights(MID, 3)
    shards = [shard_weights(MID, W, r, world) for r in range(world)]
    loc = local_dims(MID, world)
    d, H, Hkv = MID["d_model"], MID["n_head"], MID["n_kv_head"]
    hd = d // H
    for li, lw in enumerate(W["layers"]):
        parts = [s["layers"][li] for s in shards]
        q = torch.cat([p["c_attn"][: loc["n_head"] * hd] for p in parts], 0)
        k = torch.cat([p["c_attn"][loc["n_head"] * hd: (loc["n_head"] + loc["n_kv_head"]) * hd] for p in parts], 0)
        v = torch.cat([p["c_attn"][(loc["n_head"] + loc["n_kv_head"]) * hd:] for p in parts], 0)
        assert torch.equal(torch.cat([q, k, v], 0), lw["c_attn"])
        assert torch.equal(torch.cat([p["c_proj"] for p in parts], 1), lw["c_proj"])
        assert torch.equal(torch.cat([p["w_gate"] for p in parts], 0), lw["w_gate"])
        assert torch.equal(torch.cat([p["w_up"] for p in parts], 0), lw["w_up"])
        assert torch.equal(torch.cat([p["w_down"] for p in parts], 1), lw["w_down"])
        assert all(p["ln_1"] is lw["ln_1"] for p in parts)
    assert torch.equal(torch.cat([s["lm_head"] for s in shards], 0), W["lm_head"])
    assert all(s["wte"] is W["wte"] for s in shards)


def test_local_dims_reject_uneven_shards():
    from axiomlm_b200.tp import local_dims

    with pytest.raises(ValueError):
        local_dims(dict(MID, n_kv_head=3), 2)
    with pytest.raises(ValueError):
        local_dims(MID, 16)  # ffn / world = 32 is not a multiple of 64


def test_argmax_key_rule():
    from axiomlm_b200.tp import argmax_key

    # larger logit wins; equal logits: the lower global index wins (torch.argmax)
    assert argmax_key(1.5, 10) > argmax_key(1.25, 3)
    assert argmax_key(-0.5, 7) > argmax_key(-0.75, 2)
    assert argmax_key(0.25, 3) > argmax_key(0.25, 9)
    vals = [(-3.0, 0), (2.0, 5), (2.0, 1), (-1.0, 4)]
    best = max(vals, key=lambda t: argmax_key(*t))
    assert best == (2.0, 1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _exchange(rank, world, port, out):
    import torch.distributed as dist

    from axiomlm_b200.tp import TensorParallel

    class Probe(TensorParallel):
        def __init__(self, r, w, uid):  # records the id instead of creating a communicator
            self.rank, self.world, self.uid = r, w, uid

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t = Probe.from_process_group(id_fn=lambda: bytes(range(128)))
        out[rank] = (t.rank, t.world, t.uid)
    finally:
        dist.destroy_process_group()


def test_unique_id_reaches_every_rank():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_exchange, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        assert out[0] == (0, 2, bytes(range(128)))
        assert out[1] == (1, 2, bytes(range(128)))
