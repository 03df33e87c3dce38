"""Seeded synthetic models at the benchmark shapes (random N(0, 0.02) weights
packed on the GPU, uniform-random token ids), shared by the benchmark and the
op micro-benchmarks.  There are no checkpoints or datasets on this path: the
weights only have to have the right shapes, formats and value distribution."""

from __future__ import annotations

import torch

# Llama-3-8B shape (the decode, tree-verification and long-context benchmarks)
CFG_8B = dict(n_layer=32, d_model=4096, n_head=32, n_kv_head=8, ffn=14336, vocab=128256, eps=1e-5, theta=10000.0,
              block_size=8192)


def _q2t_random(fmt, N, K, g):
    """A 2-bit projection with random codes at the benchmark's value
    distribution: uniform bytes give each 2-bit ternary field +1 and -1 with
    p = .25 and 0 with p = .5; the scales are those of N(0, 0.02) weights
    (per-tensor absmean 0.016; K-quant d, dmin about range / 15)."""
    from . import _lib as L
    from . import ops

    dev = torch.device("cuda")
    codes = torch.randint(0, 256, (N, K // 4), generator=g, device=dev, dtype=torch.uint8)
    if fmt == L.W_TERNARY_PT:
        return ops.q2t_from_ref(fmt, codes, torch.full((1,), 0.016, device=dev, dtype=torch.float16), None, K)
    sub = torch.randint(0, 256, (N, K // 16), generator=g, device=dev, dtype=torch.uint8)
    dm = (torch.rand(N, K // 256, 2, generator=g, device=dev) * 0.004).half()
    return ops.q2t_from_ref(fmt, codes, sub, dm, K)


def build_decoder(cfg, batch, ctx, kv, seed=0, tp=None, max_tokens=1, extra_slots=1024, ring_buffer=False,
                  weights="q4_g128", ring=0):
    """Random N(0, 0.02) weights packed Q4 group-128 symmetric on the GPU, and
    a decoder with room for ``ctx + extra_slots`` cached tokens.  With ``tp``
    (tensor parallel) this rank packs only its shard: H / N query heads,
    Hkv / N KV heads, F / N FFN rows, V / N vocab rows; the embedding and the
    norms, replicated, come from the same seed on every rank.

    ``weights="ternary_pt" | "q2k"``: the projections and the lm_head in that
    2-bit benchmark-only layout (random codes, ``_q2t_random``).  ``ring``: a ring
    cache of that many slots (the sliding window) instead of ``ctx +
    extra_slots``; positions run on to ``ctx + extra_slots``."""
    from . import _lib as L
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
    lowbit = {"ternary_pt": L.W_TERNARY_PT, "q2k": L.W_Q2K_SB256}.get(weights)
    if lowbit is None and weights != "q4_g128":
        raise ValueError(f"unknown weights {weights!r}")
    if lowbit is not None and tp is not None and tp.world > 1:
        raise ValueError("2-bit weights are served without tensor parallelism")

    def proj(N, K, gate_up=False):
        if lowbit is not None:
            return _q2t_random(lowbit, N, K, g)
        return ops.pack_q4t(rn(N, K), 128, True, gate_up=gate_up)

    layers = []
    for _ in range(cfg["n_layer"]):
        layers.append(dict(
            qkv=proj((H + 2 * Hkv) * hd, d), o=proj(d, H * hd), gu=proj(2 * F, d, gate_up=True), down=proj(d, F),
            ln_1=torch.ones(d, device=dev), ln_2=torch.ones(d, device=dev), qkv_b=None))
        torch.cuda.synchronize()
    gr = torch.Generator(device="cuda").manual_seed(seed + 7919)  # replicated tensors: same on every rank
    wte = torch.randn(V, d, generator=gr, device=dev, dtype=torch.float32) * 0.02
    emb_w, emb_s = ops.pack_q8_g64(wte)
    del wte
    lm = proj(V_l, d)
    packed = dict(layers=layers, emb_w=emb_w, emb_s=emb_s, lm_head=lm, ln_f=torch.ones(d, device=dev))
    torch.cuda.synchronize()
    kv_dtype, kv_group = kv
    return QuantizedDecoder(cfg, packed, kv_dtype=kv_dtype, kv_group=kv_group, max_batch=batch,
                            max_seq=ring or ctx + extra_slots, max_tokens=max_tokens,
                            rope_len=max(cfg["block_size"], ctx + extra_slots), tp=tp,
                            ring_buffer=ring_buffer or bool(ring))


def fill_context(dec, batch, ctx, seed=1):
    """ctx random token ids per sequence, run through the decoder one token at
    a time (the decode path the benchmark times).  With a ring cache of W <
    ctx slots only the last W tokens stay cached, and a step's cost depends on
    that window alone: the position counters start at ctx - W, and the last W
    tokens are decoded into the window."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    c = dec.cache
    t0 = 0
    if c.ring_buffer and ctx > c.max_seq_len:
        t0 = ctx - c.max_seq_len
        c.advance(t0)
    toks = torch.randint(0, dec.cfg["vocab"], (batch, ctx), generator=g, device="cuda")
    for t in range(t0, ctx):
        dec.decode_step(toks[:, t:t + 1])
    torch.cuda.synchronize()
