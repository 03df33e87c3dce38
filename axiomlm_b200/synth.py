"""Seeded synthetic models at the BASELINE shapes (random N(0, 0.02) weights
packed on the GPU, uniform-random token ids), shared by the benchmark and the
op micro-benchmarks.  There are no checkpoints or datasets on this path: the
weights only have to have the right shapes, formats and value distribution."""

from __future__ import annotations

import torch

# Llama-3-8B shape
CFG_8B = dict(n_layer=32, d_model=4096, n_head=32, n_kv_head=8, ffn=14336, vocab=128256, eps=1e-5, theta=10000.0,
              block_size=8192)


def build_decoder(cfg, batch, ctx, kv, seed=0, tp=None, max_tokens=1, extra_slots=1024, ring_buffer=False):
    """Random N(0, 0.02) weights packed Q4 group-128 symmetric on the GPU, and
    a decoder with room for ``ctx + extra_slots`` cached tokens.  With ``tp``
    (tensor parallel) this rank packs only its shard: H / N query heads,
    Hkv / N KV heads, F / N FFN rows, V / N vocab rows; the embedding and the
    norms, replicated, come from the same seed on every rank."""
    from . import ops
    from .model import QuantizedDecoder

    world = tp.world if tp is not None else 1
    g = torch.Generator(device="cuda").manual_seed(seed + (tp.rank if tp is not None else 0))
    dev = torch.device("cuda")

    def rn(*shape):
        return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * 0.02

    d, H, Hkv, F, V = cfg["d_model"], cfg["n_head"], cfg["n_kv_head"], cfg["ffn"], cfg["vocab"]
    hd = d // H
    H, Hkv, F, V_l = H // world, Hkv // world, F // world, V // world
    layers = []
    for _ in range(cfg["n_layer"]):
        layers.append(dict(
            qkv=ops.pack_q4t(rn((H + 2 * Hkv) * hd, d), 128, True), o=ops.pack_q4t(rn(d, H * hd), 128, True),
            gu=ops.pack_q4t(rn(2 * F, d), 128, True, gate_up=True), down=ops.pack_q4t(rn(d, F), 128, True),
            ln_1=torch.ones(d, device=dev), ln_2=torch.ones(d, device=dev), qkv_b=None))
        torch.cuda.synchronize()
    gr = torch.Generator(device="cuda").manual_seed(seed + 7919)  # replicated tensors: same on every rank
    wte = torch.randn(V, d, generator=gr, device=dev, dtype=torch.float32) * 0.02
    emb_w, emb_s = ops.pack_q8_g64(wte)
    del wte
    lm = ops.pack_q4t(rn(V_l, d), 128, True)
    packed = dict(layers=layers, emb_w=emb_w, emb_s=emb_s, lm_head=lm, ln_f=torch.ones(d, device=dev))
    torch.cuda.synchronize()
    kv_dtype, kv_group = kv
    return QuantizedDecoder(cfg, packed, kv_dtype=kv_dtype, kv_group=kv_group, max_batch=batch,
                            max_seq=ctx + extra_slots, max_tokens=max_tokens, rope_len=cfg["block_size"], tp=tp,
                            ring_buffer=ring_buffer)


def fill_context(dec, batch, ctx, seed=1):
    """ctx random token ids per sequence, run through the decoder one token at
    a time (the decode path the benchmark times)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    toks = torch.randint(0, dec.cfg["vocab"], (batch, ctx), generator=g, device="cuda")
    for t in range(ctx):
        dec.decode_step(toks[:, t:t + 1])
    torch.cuda.synchronize()
