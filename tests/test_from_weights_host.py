"""``QuantizedDecoder.from_weights`` packing, run on the host up to the GPU
relayout: the relayout (``ops.q4t_from_q4g64``, tested on the GPU against
the oracle) and the decoder constructor are replaced by stand-ins that keep
what they are given.  In the reference's "q4" mode every projection and the
lm_head then dequantize to exactly what the reference's own quantize("q4")
packs of the same model dequantize to (tests/golden/small_q4.npz); in
"q4_k_m" the Q4 projections do (small_q4km.npz), and w_down and the lm_head
go to the Q8 packer."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from model_weights import SMALL, make_weights
from oracle import axb_oracle as O


@pytest.fixture
def captured(monkeypatch):
    from axiomlm_b200 import model as M
    from axiomlm_b200 import ops

    cap = {}

    def relayout(words, sb, n_out=None, gate_up=False):
        return ("q4g64", words.clone(), sb.clone(), gate_up)

    def q8(w):  # the Q8_G64 packer is round-to-nearest; its CUDA kernel is tested against the oracle
        p, s = O.pack_q8_g64(w.numpy())
        return torch.from_numpy(p), torch.from_numpy(s)

    def init(self, cfg, packed, **kw):
        cap["cfg"], cap["packed"] = cfg, packed

    monkeypatch.setattr(ops, "q4t_from_q4g64", relayout)
    monkeypatch.setattr(ops, "pack_q8_g64", q8)
    monkeypatch.setattr(M.QuantizedDecoder, "__init__", init)
    return cap


def _same_values(ours, ref_p, ref_s, K, N):
    kind, words, sb, _ = ours
    assert kind == "q4g64"
    a = O.dequant_q4_g64(words.numpy(), sb.numpy(), K)
    b = O.dequant_q4_marlin(ref_p, ref_s, K, N)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))


@pytest.mark.parametrize("name,mode", [("small_q4", "q4"), ("small_q4km", "q4_k_m")])
def test_from_weights_packs_like_the_reference(captured, name, mode):
    from axiomlm_b200 import ops
    from axiomlm_b200.model import QuantizedDecoder

    fx = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    W = make_weights(SMALL, int(fx["seed"]), ln_random=bool(fx["ln_random"]))
    QuantizedDecoder.from_weights(SMALL, W, mode, device="cpu")
    packed = captured["packed"]
    d, F = SMALL["d_model"], SMALL["ffn"]
    qkv_dim = (SMALL["n_head"] + 2 * SMALL["n_kv_head"]) * (d // SMALL["n_head"])
    for i, ly in enumerate(packed["layers"]):
        _same_values(ly["qkv"], fx[f"pk_c_attn_p_{i}"], fx[f"pk_c_attn_s_{i}"], d, qkv_dim)
        _same_values(ly["o"], fx[f"pk_c_proj_p_{i}"], fx[f"pk_c_proj_s_{i}"], d, d)
        _same_values(ly["gu"], fx[f"pk_gu_p_{i}"], fx[f"pk_gu_s_{i}"], d, 2 * F)
        assert ly["gu"][3] is True  # gate_up rows are interleaved for the SwiGLU epilogue
        if mode == "q4":
            _same_values(ly["down"], fx[f"pk_wd_p_{i}"], fx[f"pk_wd_s_{i}"], F, d)
        else:
            assert isinstance(ly["down"], ops.Q8Weight) and ly["down"].K == F
    if mode == "q4":
        _same_values(packed["lm_head"], fx["pk_lmh_p"], fx["pk_lmh_sb"], d, SMALL["vocab"])
    else:
        assert isinstance(packed["lm_head"], ops.Q8Weight) and packed["lm_head"].N == SMALL["vocab"]


@pytest.mark.parametrize("fmt,oracle_pack", [("ternary", "pack_ternary"), ("q2_k", "pack_q2"),
                                             ("ternary_pt", "ternary_pt_pack"), ("q2k", "q2k_pack")])
def test_from_weights_lowbit_packs(monkeypatch, captured, fmt, oracle_pack):
    """The 2-bit formats: every projection (gate_up as cat(w_gate, w_up), the
    reference's row order) and the untied lm_head reach the q2t relayout as
    the oracle packs them (the oracle's ternary / Q2 G64 packers are pinned to
    the reference's)."""
    from axiomlm_b200 import ops
    from axiomlm_b200.model import QuantizedDecoder

    seen = []
    monkeypatch.setattr(ops, "q2t_from_ref", lambda f, c, s1, s2=None, K=None: seen.append((f, c, s1, s2, K)) or
                        ops.Q2TWeight(c, None, None, None, c.shape[0], K, f))
    W = make_weights(SMALL, 7, ln_random=True)
    QuantizedDecoder.from_weights(SMALL, W, fmt, device="cpu")
    mats = []
    for lw in W["layers"]:
        # from_weights packs a layer's w_down first, then c_attn, c_proj and gate_up
        mats += [lw["w_down"], lw["c_attn"], lw["c_proj"], torch.cat([lw["w_gate"], lw["w_up"]], 0)]
    mats.append(W["lm_head"])
    assert len(seen) == len(mats)
    for (f, c, s1, s2, K), w in zip(seen, mats):
        ref = getattr(O, oracle_pack)(w.numpy())
        assert K == w.shape[1] and np.array_equal(c.numpy(), ref[0])
        assert np.array_equal(s1.numpy().view(np.uint8), np.asarray(ref[1]).view(np.uint8))
        if s2 is not None:
            assert np.array_equal(s2.numpy().view(np.uint8), np.asarray(ref[2]).view(np.uint8))


def test_from_hf_carries_bias_and_config(tmp_path, captured):
    """from_hf on a Qwen2-style checkpoint (q / k / v biases, tied
    embeddings): the fused, RoPE-interleaved bias reaches the packed layers in
    fp16 as the reference's importer builds it, the embedding is the Q8
    lm_head, and the model config comes through."""
    from model_weights import make_hf_checkpoint

    from axiomlm_b200 import ops
    from axiomlm_b200.model import QuantizedDecoder

    make_hf_checkpoint(str(tmp_path), 72, bias=True, tied=True, shards=2)
    QuantizedDecoder.from_hf(tmp_path, weight_format="q4", device="cpu")
    fx = np.load(os.path.join(GOLDEN, "hf_import.npz"))
    cfg, packed = captured["cfg"], captured["packed"]
    assert cfg["theta"] == float(fx["qwen_theta"]) and cfg["tied"]
    for i, ly in enumerate(packed["layers"]):
        assert ly["qkv_b"].dtype == torch.float16
        assert np.array_equal(ly["qkv_b"].numpy().view(np.uint16), fx[f"qwen_{i}_c_attn_b"].view(np.uint16))
    lm = packed["lm_head"]
    assert isinstance(lm, ops.Q8Weight) and lm.words is packed["emb_w"]


@pytest.mark.parametrize("fmt", ["q4_rtn", "q4_legacy", "q4_g128_sym", "q8", "q4", "q4_k_m", "ternary", "q2_k",
                                 "ternary_pt", "q2k"])
def test_from_weights_every_format_on_host(monkeypatch, captured, fmt):
    """Every weight format builds its packed model on the host (GPU calls
    replaced by stand-ins): each projection and the lm_head in the format's
    kind, with the right (N, K); gate_up as one (2F, d) matrix."""
    from axiomlm_b200 import model as M
    from axiomlm_b200 import ops

    monkeypatch.setattr(ops, "pack_q4t", lambda w, group=128, symmetric=True, gate_up=False:
                        ops.Q4TWeight(torch.zeros(1, dtype=torch.int32), torch.zeros(1).half(), w.shape[0], w.shape[1],
                                      group, 1 if symmetric else 2, gate_up))
    monkeypatch.setattr(ops, "q2t_from_ref", lambda f, c, s1, s2=None, K=None:
                        ops.Q2TWeight(c, None, None, None, c.shape[0], K, f))
    W = make_weights(SMALL, 9, ln_random=True)
    M.QuantizedDecoder.from_weights(SMALL, W, fmt, device="cpu")
    packed = captured["packed"]
    d, F, V = SMALL["d_model"], SMALL["ffn"], SMALL["vocab"]
    qkv = (SMALL["n_head"] + 2 * SMALL["n_kv_head"]) * (d // SMALL["n_head"])

    def nk(w):
        if isinstance(w, tuple):  # the q4g64 relayout stand-in: (kind, words (N, K/8), ...)
            return w[1].shape[0], w[1].shape[1] * 8
        return w.N, w.K

    q8_down = fmt in ("q8", "q4_k_m")
    for ly in packed["layers"]:
        assert [nk(ly[k]) for k in ("qkv", "o", "gu", "down")] == [(qkv, d), (d, d), (2 * F, d), (d, F)]
        assert isinstance(ly["down"], ops.Q8Weight) == q8_down
        assert isinstance(ly["qkv"], ops.Q8Weight) == (fmt == "q8")
        assert isinstance(ly["qkv"], ops.Q2TWeight) == (fmt in ("ternary", "q2_k", "ternary_pt", "q2k"))
    assert nk(packed["lm_head"]) == (V, d)
    assert isinstance(packed["lm_head"], ops.Q8Weight) == q8_down
