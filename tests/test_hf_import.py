"""Hugging Face checkpoint import and the packed-weight cache (host logic).

The importer's output is compared with the reference's own
``load_hf_safetensors`` run on the same seeded checkpoints
(tests/golden/make_golden.py --hf-only -> hf_import.npz): every parameter
bit-identical.  The RoPE row permutation is also checked against its meaning:
the pair RoPE of the permuted projection equals the permuted rotate-half RoPE
of the original one.
"""

import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from model_weights import make_hf_checkpoint

from axiomlm_b200.hf_import import (hf_config, permute_hf_rope_bias, permute_hf_rope_weight, read_hf_checkpoint,
                                    unpermute_hf_rope_weight)


def _f16_bits(t):
    return torch.as_tensor(t).to(torch.float16).numpy().view(np.uint16)


@pytest.mark.parametrize("tag,seed,bias,tied,shards", [("llama", 71, False, False, 1), ("qwen", 72, True, True, 2)])
def test_import_matches_reference_importer(tmp_path, tag, seed, bias, tied, shards):
    fx = np.load(os.path.join(GOLDEN, "hf_import.npz"))
    make_hf_checkpoint(str(tmp_path), seed, bias=bias, tied=tied, shards=shards)
    cfg, w = read_hf_checkpoint(tmp_path)
    assert cfg["block_size"] == int(fx[f"{tag}_block_size"])
    assert cfg["theta"] == float(fx[f"{tag}_theta"])
    assert cfg["tied"] == tied and cfg["qkv_bias"] == bias
    assert np.array_equal(_f16_bits(w["wte"]), fx[f"{tag}_wte"].view(np.uint16))
    assert np.array_equal(_f16_bits(w["ln_f"]), fx[f"{tag}_ln_f"].view(np.uint16))
    lmh = w["wte"] if w["lm_head"] is None else w["lm_head"]
    assert (w["lm_head"] is None) == tied
    assert np.array_equal(_f16_bits(lmh), fx[f"{tag}_lm_head"].view(np.uint16))
    for i, ly in enumerate(w["layers"]):
        for k in ("c_attn", "c_proj", "w_gate", "w_up", "w_down", "ln_1", "ln_2"):
            assert np.array_equal(_f16_bits(ly[k]), fx[f"{tag}_{i}_{k}"].view(np.uint16)), (i, k)
        if bias:
            assert np.array_equal(_f16_bits(ly["c_attn_b"]), fx[f"{tag}_{i}_c_attn_b"].view(np.uint16))
        else:
            assert ly["c_attn_b"] is None


def _rope_half_split(q, ang):
    """Hugging Face rotate-half RoPE on (heads, hd): dims i and i + hd/2 share angle i."""
    h = q.shape[-1] // 2
    cos, sin = torch.cos(ang), torch.sin(ang)
    a, b = q[..., :h], q[..., h:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], -1)


def _rope_pairs(q, ang):
    """The reference's RoPE: pairs (x[2i], x[2i + 1]) rotated by angle i."""
    a, b = q[..., 0::2], q[..., 1::2]
    cos, sin = torch.cos(ang), torch.sin(ang)
    return torch.stack([a * cos - b * sin, a * sin + b * cos], -1).flatten(-2)


def test_rope_permutation_carries_the_half_split_rope_to_the_pair_rope():
    g = torch.Generator().manual_seed(5)
    H, hd, d = 3, 16, 24
    W = torch.randn(H * hd, d, generator=g, dtype=torch.float64)
    bvec = torch.randn(H * hd, generator=g, dtype=torch.float64)
    x = torch.randn(d, generator=g, dtype=torch.float64)
    ang = 7.0 * 10000.0 ** (-torch.arange(hd // 2, dtype=torch.float64) * 2 / hd)
    q_hf = _rope_half_split((W @ x + bvec).view(H, hd), ang)
    q_ax = _rope_pairs((permute_hf_rope_weight(W, H, hd) @ x + permute_hf_rope_bias(bvec, H, hd)).view(H, hd), ang)
    # the same vector, its halves interleaved
    assert torch.allclose(q_ax, permute_hf_rope_bias(q_hf.reshape(-1), H, hd).view(H, hd), atol=1e-12)
    assert torch.equal(unpermute_hf_rope_weight(permute_hf_rope_weight(W, H, hd), H, hd), W)


def test_hf_config_defaults_and_rope_parameters():
    base = dict(num_attention_heads=8, hidden_size=512, num_hidden_layers=2, intermediate_size=1024, vocab_size=100)
    c = hf_config(base)
    assert (c["eps"], c["theta"], c["tied"], c["block_size"], c["n_kv_head"], c["qkv_bias"]) == \
        (1e-6, 10000.0, True, 4096, 8, False)
    rp = {"rope_type": "llama3", "rope_theta": 500000.0, "factor": 8.0}
    c = hf_config(dict(base, rope_parameters=rp, max_position_embeddings=131072, attention_bias=True), max_seq_len=512)
    assert c["theta"] == 500000.0 and c["rope_scaling"] == rp and c["block_size"] == 512 and c["qkv_bias"]


def test_import_rejects_missing_directory(tmp_path):
    with pytest.raises(FileNotFoundError):
        read_hf_checkpoint(tmp_path / "absent")
    os.makedirs(tmp_path / "empty")
    with open(tmp_path / "empty" / "config.json", "w") as f:
        json.dump({}, f)
    with pytest.raises(FileNotFoundError):
        read_hf_checkpoint(tmp_path / "empty")


def test_packed_cache_round_trip_on_host(tmp_path):
    from safetensors.torch import save_file

    from axiomlm_b200 import _lib as L
    from axiomlm_b200 import ops
    from axiomlm_b200.model import QuantizedDecoder, packed_to_tensors, read_packed

    g = torch.Generator().manual_seed(9)

    def words(n):
        return torch.randint(-2 ** 31, 2 ** 31 - 1, (n,), generator=g, dtype=torch.int32)

    def halfs(*s):
        return torch.randn(*s, generator=g).half()

    q4 = ops.Q4TWeight(words(512), halfs(64), 32, 128, 128, L.W_Q4T_SYM, True)
    q8 = ops.Q8Weight(words(32 * 32).view(32, 32), halfs(32, 2, 2), 32, 128)
    q2 = ops.Q2TWeight(torch.randint(0, 255, (256,), generator=g, dtype=torch.uint8), None, None, halfs(1), 32, 128,
                       L.W_TERNARY_PT)
    layer = dict(qkv=q4, o=q4, gu=q4, down=q2, ln_1=torch.randn(128, generator=g), ln_2=torch.randn(128, generator=g),
                 qkv_b=None)
    packed = dict(layers=[layer, dict(layer, qkv_b=halfs(32))], emb_w=words(64).view(16, 4), emb_s=halfs(16, 1, 2),
                  lm_head=q8, ln_f=torch.randn(128, generator=g))
    cfg = dict(n_layer=2, d_model=128, n_head=2, n_kv_head=1, ffn=128, vocab=32, eps=1e-5, theta=1e4)
    tensors, meta = packed_to_tensors(packed)
    meta.update(cfg=json.dumps(cfg), format=QuantizedDecoder._PACKED_FORMAT)
    path = tmp_path / "packed.safetensors"
    save_file(tensors, str(path), metadata=meta)
    cfg2, p2 = read_packed(path, "cpu")
    assert cfg2 == cfg

    def same(a, b):
        if a is None or b is None:
            return a is None and b is None
        if isinstance(a, torch.Tensor):
            return a.dtype == b.dtype and torch.equal(a, b)
        return type(a) is type(b) and all(same(getattr(a, f), getattr(b, f)) if isinstance(getattr(a, f), torch.Tensor)
                                          or getattr(a, f) is None else getattr(a, f) == getattr(b, f)
                                          for f in a.__dataclass_fields__)

    for k in ("emb_w", "emb_s", "lm_head", "ln_f"):
        assert same(packed[k], p2[k]), k
    for a, b in zip(packed["layers"], p2["layers"]):
        for k in a:
            assert same(a[k], b[k]), k
    # a tied lm_head (the embedding matrix itself) is stored once and shared again
    tied = dict(packed, lm_head=ops.Q8Weight(packed["emb_w"], packed["emb_s"], 16, 16))
    tensors, meta = packed_to_tensors(tied)
    assert not any(k.startswith("lm_head") for k in tensors)
    meta.update(cfg=json.dumps(cfg), format=QuantizedDecoder._PACKED_FORMAT)
    save_file(tensors, str(tmp_path / "tied.safetensors"), metadata=meta)
    _, p3 = read_packed(tmp_path / "tied.safetensors", "cpu")
    assert p3["lm_head"].words.data_ptr() == p3["emb_w"].data_ptr() and torch.equal(p3["emb_w"], packed["emb_w"])
    bad = tmp_path / "other.safetensors"
    save_file({"x": torch.zeros(1)}, str(bad), metadata={"format": "something else"})
    with pytest.raises(ValueError):
        read_packed(bad, "cpu")
