"""Tensor-parallel decode on 2 GPUs against the single-GPU decoder on the
same weights and teacher-forced tokens: the gathered vocab shards of the
logits within the model tolerance, and the same greedy token at every step
(apart from near-ties).  Needs two CUDA devices; skipped otherwise."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

MID = dict(n_layer=2, d_model=1024, n_head=8, n_kv_head=2, ffn=2048, vocab=4096, eps=1e-5, theta=10000.0,
           block_size=1024)
REL_TOL = 1.5e-2  # fp8 KV: codes can flip on last-ulp differences of K / V
TIE = 2e-3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, steps, out):
    import datetime

    import torch.distributed as dist

    from axiomlm_b200.model import QuantizedDecoder
    from axiomlm_b200.tp import TensorParallel
    from model_weights import make_weights

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    tp = TensorParallel.from_process_group()
    try:
        W = make_weights(MID, 11, ln_random=True)
        kw = dict(kv_dtype="fp8", kv_group=128, max_seq=512, rope_len=1024)
        dec = QuantizedDecoder.from_weights(MID, W, "q4_g128_sym", tp=tp, **kw)
        g = torch.Generator().manual_seed(5)
        prompt = torch.randint(0, MID["vocab"], (1, 40), generator=g)
        forced = torch.randint(0, MID["vocab"], (steps, 1, 1), generator=g)
        dec.prefill(prompt.cuda())
        logits, tokens = [], []
        for i in range(steps):
            lg = dec.decode_step(forced[i].cuda())[0, 0].float().cpu()
            parts = [torch.empty_like(lg) for _ in range(world)]
            dist.all_gather(parts, lg)
            logits.append(torch.cat(parts))
            tokens.append(int(dec.argmax(1)[0]))
        assert dec.status() == 0
        dec.close()
        if rank == 0:
            ref = QuantizedDecoder.from_weights(MID, W, "q4_g128_sym", **kw)
            ref.prefill(prompt.cuda())
            res = []
            for i in range(steps):
                a = ref.decode_step(forced[i].cuda())[0, 0].float().cpu()
                res.append((a, int(ref.argmax(1)[0])))
            ref.close()
            out["ref"] = res
            out["tp"] = list(zip(logits, tokens))
        dist.barrier()
    finally:
        tp.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two CUDA devices")
def test_tp2_decode_matches_single_gpu():
    steps = 8
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, steps, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=600)
            assert p.exitcode == 0, f"rank exited with {p.exitcode}"
        ref, tp = out["ref"], out["tp"]
    for i, ((a, ta), (b, tb)) in enumerate(zip(ref, tp)):
        rel = float((a - b).abs().max() / a.abs().max())
        assert rel < REL_TOL, f"step {i}: rel {rel:.2e}"
        assert tb == int(b.argmax()), f"step {i}: the tp argmax is not the argmax of the gathered logits"
        if ta != tb:
            top = a.topk(2).values
            assert float(top[0] - top[1]) / float(a.abs().max()) < TIE, f"step {i}: {ta} != {tb}"
