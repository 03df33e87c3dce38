"""Hugging Face safetensors checkpoints into the decoder (drop-in for
``axiomlm/utils/hf_importer.py``: ``load_hf_safetensors`` :199-305,
``build_model_config_from_hf`` :96-152).

Llama-3 / SmolLM2 / Qwen2.5 checkpoints (``LlamaForCausalLM`` /
``Qwen2ForCausalLM``) are read from a local directory: ``config.json`` and
``model.safetensors``, or shards listed in ``model.safetensors.index.json``,
or every ``*.safetensors`` file.  There is no hub download here (no network
on the serving side): pass a directory.

Hugging Face stores each q / k head's rows half-split (dims [0, hd/2) then
[hd/2, hd)), for its rotate-half RoPE; the reference's RoPE rotates
interleaved pairs (x[2i], x[2i + 1]), so the importer interleaves the rows of
q_proj / k_proj (and Qwen2's q / k biases) the same way the reference does
(hf_importer.py:23-63).  q, k, v are fused into one c_attn matrix.  Tensors
are read in the reference's load dtype (fp16 by default, the value the
reference quantizes from) and handed to the packers as fp32.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import torch


def permute_hf_rope_weight(w: torch.Tensor, n_heads: int, head_dim: int) -> torch.Tensor:
    """Rows of a half-split RoPE projection (HF) in interleaved-pair order:
    per head, row j of the first half then row j of the second half
    (hf_importer.py:23-35)."""
    return w.reshape(n_heads, 2, head_dim // 2, -1).transpose(1, 2).reshape(n_heads * head_dim, -1).contiguous()


def unpermute_hf_rope_weight(w: torch.Tensor, n_heads: int, head_dim: int) -> torch.Tensor:
    """The inverse of ``permute_hf_rope_weight`` (hf_importer.py:38-50)."""
    return w.reshape(n_heads, head_dim // 2, 2, -1).transpose(1, 2).reshape(n_heads * head_dim, -1).contiguous()


def permute_hf_rope_bias(b: torch.Tensor, n_heads: int, head_dim: int) -> torch.Tensor:
    """``permute_hf_rope_weight`` for a bias vector (hf_importer.py:53-63)."""
    return b.reshape(n_heads, 2, head_dim // 2).transpose(1, 2).reshape(n_heads * head_dim).contiguous()


def hf_config(hf_cfg: dict[str, Any], has_qkv_bias: bool = False, max_seq_len: int | None = None) -> dict:
    """A Hugging Face ``config.json`` as the decoder's cfg dict, with the
    reference's defaults (build_model_config_from_hf, hf_importer.py:96-152):
    eps 1e-6, theta 10000, tied embeddings unless stated, and a block size of
    ``max_seq_len`` or min(max_position_embeddings, 4096)."""
    n_head = int(hf_cfg["num_attention_heads"])
    rope_params = hf_cfg.get("rope_parameters") or {}
    theta = float(hf_cfg.get("rope_theta", rope_params.get("rope_theta", 10000.0)))
    rope_scaling = hf_cfg.get("rope_scaling")
    if rope_scaling is None and isinstance(rope_params, dict) and rope_params.get("rope_type") not in (None, "default"):
        rope_scaling = rope_params
    max_pos = int(hf_cfg.get("max_position_embeddings", 4096))
    return dict(
        n_layer=int(hf_cfg["num_hidden_layers"]), d_model=int(hf_cfg["hidden_size"]), n_head=n_head,
        n_kv_head=int(hf_cfg.get("num_key_value_heads", n_head)), ffn=int(hf_cfg["intermediate_size"]),
        vocab=int(hf_cfg["vocab_size"]), eps=float(hf_cfg.get("rms_norm_eps", 1e-6)), theta=theta,
        rope_scaling=rope_scaling, block_size=max_seq_len if max_seq_len is not None else min(max_pos, 4096),
        tied=bool(hf_cfg.get("tie_word_embeddings", True)),
        qkv_bias=bool(has_qkv_bias or hf_cfg.get("attention_bias", False) or hf_cfg.get("qkv_bias", False)))


class SafetensorsDir:
    """Lazy tensor access over a checkpoint directory's safetensors files
    (one file, an index of shards, or every ``*.safetensors``; the
    reference's _SafetensorsReader, hf_importer.py:155-196)."""

    def __init__(self, model_dir: str | Path):
        from safetensors import safe_open

        self._open = lambda p: safe_open(str(p), framework="pt", device="cpu")
        self.dir = Path(model_dir)
        self._handles: dict[str, Any] = {}
        self.weight_map: dict[str, str] = {}
        index = self.dir / "model.safetensors.index.json"
        if index.exists():
            self.weight_map = dict(json.loads(index.read_text(encoding="utf-8"))["weight_map"])
            return
        files = [self.dir / "model.safetensors"] if (self.dir / "model.safetensors").exists() \
            else sorted(self.dir.glob("*.safetensors"))
        if not files:
            raise FileNotFoundError(f"no .safetensors files in {self.dir}")
        for f in files:
            h = self._handles[f.name] = self._open(f)
            for k in h.keys():
                self.weight_map[k] = f.name

    def __contains__(self, key: str) -> bool:
        return key in self.weight_map

    def get(self, key: str, dtype: torch.dtype) -> torch.Tensor:
        if key not in self.weight_map:
            raise KeyError(f"tensor {key!r} not in the checkpoint")
        shard = self.weight_map[key]
        if shard not in self._handles:
            self._handles[shard] = self._open(self.dir / shard)
        return self._handles[shard].get_tensor(key).to(dtype)


def read_hf_checkpoint(model_dir: str | Path, dtype: torch.dtype = torch.float16,
                       max_seq_len: int | None = None) -> tuple[dict, dict]:
    """(cfg, weights) of a local Hugging Face checkpoint, ``weights`` in the
    layout ``QuantizedDecoder.from_weights`` packs: ``wte``, ``lm_head`` (None
    when tied), ``ln_f`` and per layer ``c_attn`` (q, k rows interleaved for
    the pair RoPE, then v), ``c_attn_b`` (or None), ``c_proj``, ``w_gate``,
    ``w_up``, ``w_down``, ``ln_1``, ``ln_2``; fp32 tensors holding the values
    of ``dtype`` (load_hf_safetensors, hf_importer.py:199-305)."""
    d = Path(model_dir)
    if not d.is_dir():
        raise FileNotFoundError(f"{model_dir} is not a local checkpoint directory (no hub download here)")
    cfg_path = d / "config.json"
    if not cfg_path.exists():
        raise FileNotFoundError(f"missing config.json in {d}")
    hf_cfg = json.loads(cfg_path.read_text(encoding="utf-8"))
    st = SafetensorsDir(d)
    has_bias = "model.layers.0.self_attn.q_proj.bias" in st
    if "lm_head.weight" in st and not bool(hf_cfg.get("tie_word_embeddings", True)):
        hf_cfg["tie_word_embeddings"] = False
    cfg = hf_config(hf_cfg, has_qkv_bias=has_bias, max_seq_len=max_seq_len)
    H, Hkv = cfg["n_head"], cfg["n_kv_head"]
    hd = cfg["d_model"] // H

    def get(key):
        return st.get(key, dtype).float()

    w = {"wte": get("model.embed_tokens.weight"), "ln_f": get("model.norm.weight"),
         "lm_head": get("lm_head.weight") if not cfg["tied"] and "lm_head.weight" in st else None, "layers": []}
    if w["lm_head"] is None:
        cfg["tied"] = True
    for i in range(cfg["n_layer"]):
        p = f"model.layers.{i}"
        wq = permute_hf_rope_weight(get(f"{p}.self_attn.q_proj.weight"), H, hd)
        wk = permute_hf_rope_weight(get(f"{p}.self_attn.k_proj.weight"), Hkv, hd)
        wv = get(f"{p}.self_attn.v_proj.weight")
        bias = None
        if cfg["qkv_bias"] and f"{p}.self_attn.q_proj.bias" in st:
            bias = torch.cat([permute_hf_rope_bias(get(f"{p}.self_attn.q_proj.bias"), H, hd),
                              permute_hf_rope_bias(get(f"{p}.self_attn.k_proj.bias"), Hkv, hd),
                              get(f"{p}.self_attn.v_proj.bias")])
        w["layers"].append(dict(
            c_attn=torch.cat([wq, wk, wv], 0), c_attn_b=bias, c_proj=get(f"{p}.self_attn.o_proj.weight"),
            w_gate=get(f"{p}.mlp.gate_proj.weight"), w_up=get(f"{p}.mlp.up_proj.weight"),
            w_down=get(f"{p}.mlp.down_proj.weight"), ln_1=get(f"{p}.input_layernorm.weight"),
            ln_2=get(f"{p}.post_attention_layernorm.weight")))
    return cfg, w
