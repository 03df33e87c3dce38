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
# The reference's CPU-runnable tiny model.
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


# A tiny Hugging Face-format checkpoint (Llama / Qwen2 tensor names, half-split
# q / k rows, bf16 tensors), written from a seed.  Shared by make_golden.py,
# which feeds it to the reference's importer, and by the importer tests.
HF_TINY = dict(num_hidden_layers=2, hidden_size=64, num_attention_heads=4, num_key_value_heads=2,
               intermediate_size=128, vocab_size=96, rms_norm_eps=1e-5, rope_theta=500000.0,
               max_position_embeddings=2048, architectures=["LlamaForCausalLM"])


def make_hf_checkpoint(path, seed: int, bias: bool = False, tied: bool = False, shards: int = 1) -> dict:
    import json
    import os

    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    c = dict(HF_TINY, tie_word_embeddings=tied)
    d, H, Hkv, F, V = (c["hidden_size"], c["num_attention_heads"], c["num_key_value_heads"], c["intermediate_size"],
                       c["vocab_size"])
    hd = d // H

    def rn(*shape):
        return (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16)

    t = {"model.embed_tokens.weight": rn(V, d), "model.norm.weight": (1 + rn(d)).to(torch.bfloat16)}
    if not tied:
        t["lm_head.weight"] = rn(V, d)
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}"
        t.update({f"{p}.self_attn.q_proj.weight": rn(H * hd, d), f"{p}.self_attn.k_proj.weight": rn(Hkv * hd, d),
                  f"{p}.self_attn.v_proj.weight": rn(Hkv * hd, d), f"{p}.self_attn.o_proj.weight": rn(d, H * hd),
                  f"{p}.mlp.gate_proj.weight": rn(F, d), f"{p}.mlp.up_proj.weight": rn(F, d),
                  f"{p}.mlp.down_proj.weight": rn(d, F), f"{p}.input_layernorm.weight": (1 + rn(d)),
                  f"{p}.post_attention_layernorm.weight": (1 + rn(d))})
        if bias:
            t.update({f"{p}.self_attn.q_proj.bias": rn(H * hd), f"{p}.self_attn.k_proj.bias": rn(Hkv * hd),
                      f"{p}.self_attn.v_proj.bias": rn(Hkv * hd)})
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(c, f)
    names = sorted(t)
    if shards == 1:
        save_file({k: t[k].contiguous() for k in names}, os.path.join(path, "model.safetensors"))
    else:
        wmap = {}
        for s in range(shards):
            fn = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
            part = names[s::shards]
            save_file({k: t[k].contiguous() for k in part}, os.path.join(path, fn))
            wmap.update({k: fn for k in part})
        with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
            json.dump({"weight_map": wmap}, f)
    return c
