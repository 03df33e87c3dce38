"""Seeded fp32 master weights for the parity models.

Shared by ``make_golden.py`` (which feeds them to the reference, in this
container only) and by the GPU parity tests (which pack them with the CUDA
packers).  ``torch.Generator`` on the CPU is deterministic for a fixed seed
and torch build, so both sides see identical weights.
"""

from __future__ import annotations

import torch

SMALL = dict(n_layer=2, d_model=256, n_head=4, n_kv_head=2, ffn=512, vocab=1024,
             eps=1e-5, theta=10000.0, block_size=256)
# BASELINE config 1 (the reference's CPU-runnable case).
TINY = dict(n_layer=12, d_model=768, n_head=12, n_kv_head=12, ffn=2048, vocab=32000,
            eps=1e-5, theta=10000.0, block_size=512)


def make_weights(cfg: dict, seed: int, ln_random: bool = False, tied: bool = False) -> dict:
    """N(0, 0.02) projections / embeddings; RMSNorm weights are ones, or
    1 + 0.1*N(0,1) when ``ln_random`` (to exercise the norm multiply)."""
    g = torch.Generator().manual_seed(seed)
    d, H, Hkv, F, V = cfg["d_model"], cfg["n_head"], cfg["n_kv_head"], cfg["ffn"], cfg["vocab"]
    hd = d // H
    qkv = H * hd + 2 * Hkv * hd

    def rn(*shape):
        return torch.randn(*shape, generator=g, dtype=torch.float32) * 0.02

    def ln():
        if ln_random:
            return 1.0 + 0.1 * torch.randn(d, generator=g, dtype=torch.float32)
        return torch.ones(d, dtype=torch.float32)

    w = {"wte": rn(V, d), "layers": []}
    for _ in range(cfg["n_layer"]):
        w["layers"].append(dict(
            c_attn=rn(qkv, d), c_proj=rn(d, H * hd), w_gate=rn(F, d), w_up=rn(F, d),
            w_down=rn(d, F), ln_1=ln(), ln_2=ln()))
    w["ln_f"] = ln()
    w["lm_head"] = None if tied else rn(V, d)
    return w


def make_prompt(n: int, vocab: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (1, n), generator=g, dtype=torch.int64)
