"""The oracle reproduces the reference's own outputs (fixtures made by
tests/golden/make_golden.py from the reference's CPU path)."""

import json
import os

import numpy as np
import pytest
import torch

import oracle as O
from conftest import GOLDEN


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_q4_marlin_rtn_pack_bit_exact():
    g = _load("quant.npz")
    w, sb = O.pack_q4_marlin_rtn(g["W"])
    assert np.array_equal(w, g["q4m_w"])
    assert np.array_equal(sb.view(np.uint16), g["q4m_sb"].view(np.uint16))


@pytest.mark.parametrize("pfx", ["q4m", "q4m_clip"])
def test_q4_marlin_dequant_bit_exact(pfx):
    g = _load("quant.npz")
    dq = O.dequant_q4_marlin(g[f"{pfx}_w"], g[f"{pfx}_sb"], 256, 40)
    assert np.array_equal(dq.view(np.uint16), g[f"{pfx}_dq"].view(np.uint16))


def test_torch_restatement_of_marlin_dequant_matches():
    g = _load("quant.npz")
    dq = O.dequant_q4_marlin_torch(torch.from_numpy(g["q4m_clip_w"]), torch.from_numpy(g["q4m_clip_sb"]), 256, 40)
    assert np.array_equal(dq.numpy().view(np.uint16), g["q4m_clip_dq"].view(np.uint16))


def test_q4_g64_and_marlin_rtn_identical_values():
    # test_phase0_research.py:56-95: MARLIN RTN == Q4_G64 value for value
    g = _load("quant.npz")
    p, s = O.pack_q4_g64(g["W"])
    assert np.array_equal(p, g["q4g_w"]) and np.array_equal(s.view(np.uint16), g["q4g_sb"].view(np.uint16))
    dq = O.dequant_q4_g64(p, s, 256)
    assert np.array_equal(dq.view(np.uint16), g["q4g_dq"].view(np.uint16))
    assert np.array_equal(dq.view(np.uint16), g["q4m_dq"].view(np.uint16))


def test_q8_pack_dequant_rows_bit_exact():
    g = _load("quant.npz")
    p, s = O.pack_q8_g64(g["W"])
    assert np.array_equal(p, g["q8_w"]) and np.array_equal(s.view(np.uint16), g["q8_sb"].view(np.uint16))
    assert np.array_equal(O.dequant_q8_g64(p, s, 256).view(np.uint16), g["q8_dq"].view(np.uint16))
    rows = O.dequant_q8_rows(g["q8_rows_idx"], p, s)
    assert np.array_equal(rows.view(np.uint16), g["q8_rows"].view(np.uint16))


def test_ternary_bit_exact():
    g = _load("quant.npz")
    p, s = O.pack_ternary(g["Wt"])
    assert np.array_equal(p, g["ter_w"]) and np.array_equal(s.view(np.uint16), g["ter_s"].view(np.uint16))
    assert np.array_equal(O.dequant_ternary(p, s, 256).view(np.uint16), g["ter_dq"].view(np.uint16))


def test_ternary_all_256_bytes():
    # test_phase3_task33_bitnet_q2k.py:62-80: every byte decodes into {-1,0,1}
    b = np.arange(256, dtype=np.uint8)
    q = O.axb_oracle._ternary_codes(b)
    assert set(np.unique(q)) <= {-1, 0, 1}
    assert q[0b10011001].tolist() == [1, -1, 1, -1]


def test_q2_bit_exact():
    g = _load("quant.npz")
    p, s = O.pack_q2(g["Wt"])
    assert np.array_equal(p, g["q2_w"]) and np.array_equal(s.view(np.uint16), g["q2_sb"].view(np.uint16))
    assert np.array_equal(O.dequant_q2(p, s, 256).view(np.uint16), g["q2_dq"].view(np.uint16))


def test_fp8_encode_matches_torch_on_every_fp16():
    x = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    ours = O.fp8_e4m3fn_encode(x)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, ref)
    # decode is the exact inverse on all non-NaN codes
    codes = np.arange(256, dtype=np.uint8)
    dec = O.fp8_e4m3fn_decode(codes)
    ref_dec = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(dec), np.isnan(ref_dec))
    fin = ~np.isnan(dec)
    assert np.array_equal(dec[fin], ref_dec[fin])


@pytest.mark.parametrize("hd", [64, 128])
def test_kv_fp8_bit_exact(hd):
    g = _load("kv.npz")
    x = g[f"x{hd}"]
    q, s = O.quant_kv_fp8(x)
    assert np.array_equal(q, g[f"fp8_q{hd}"])
    assert np.array_equal(s.view(np.uint16), g[f"fp8_s{hd}"].view(np.uint16))
    vq, vs = O.quant_kv_fp8(x[..., ::-1])
    assert np.array_equal(vq, g[f"fp8_vq{hd}"]) and np.array_equal(vs.view(np.uint16), g[f"fp8_vs{hd}"].view(np.uint16))
    dq = O.dequant_kv_fp8(q, s)
    assert np.array_equal(dq.view(np.uint16), g[f"fp8_dq{hd}"].view(np.uint16))


@pytest.mark.parametrize("hd", [64, 128])
def test_kv_quant_fp32_inputs_bit_exact(hd):
    g = _load("kv.npz")
    x = g[f"x32_{hd}"]
    q, s = O.quant_kv_fp8(x)
    assert np.array_equal(q, g[f"fp8_q32_{hd}"]) and np.array_equal(s.view(np.uint16), g[f"fp8_s32_{hd}"].view(np.uint16))
    q, s = O.quant_kv_int4(x)
    assert np.array_equal(q, g[f"i4_q32_{hd}"]) and np.array_equal(s.view(np.uint16), g[f"i4_s32_{hd}"].view(np.uint16))


@pytest.mark.parametrize("hd", [64, 128])
def test_kv_int4_bit_exact(hd):
    g = _load("kv.npz")
    q, s = O.quant_kv_int4(g[f"x{hd}"])
    assert np.array_equal(q, g[f"i4_q{hd}"])
    assert np.array_equal(s.view(np.uint16), g[f"i4_s{hd}"].view(np.uint16))
    assert np.array_equal(O.dequant_kv_int4(q, s).view(np.uint16), g[f"i4_dq{hd}"].view(np.uint16))


def test_kv_fp8_all_zero_group_is_nan_in_reference_rule():
    # quant.py:713-716: the fp16 clamp at 1e-8 is a no-op, so an all-zero group
    # has scale 0 and 0/0 -> NaN codes (the reference's own test_08 fails on
    # this; the CUDA path writes finite zeros instead, as the Metal kernel does)
    q, s = O.quant_kv_fp8(np.zeros((1, 64), np.float16))
    assert s[0, 0] == 0 and np.all((q & 0x7F) == 0x7F)


def test_rope_tables_bit_exact():
    g = _load("rope.npz")
    for hd in (64, 128):
        f = torch.view_as_real(O.rope_freqs(hd, 64, 10000.0)).numpy()
        assert np.array_equal(f, g[f"f{hd}"])
    sc = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}
    f = torch.view_as_real(O.rope_freqs(128, 64, 500000.0, sc)).numpy()
    assert np.array_equal(f, g["f128_llama3"])


def test_attention_decode_and_tree_match_reference():
    g = _load("attn.npz")
    q, k, v = (torch.from_numpy(g[n]) for n in ("q", "k", "v"))
    out = O.attention_decode(q, k, v, 33)
    assert torch.equal(out, torch.from_numpy(g["dec_fp16"]))
    kd = torch.from_numpy(O.dequant_kv_fp8(g["kq8"], g["ks8"]))
    vd = torch.from_numpy(O.dequant_kv_fp8(g["vq8"], g["vs8"]))
    assert torch.equal(O.attention_decode(q, kd, vd, 33), torch.from_numpy(g["dec_fp8"]))
    kd = torch.from_numpy(O.dequant_kv_int4(g["kq4"], g["ks4"]))
    vd = torch.from_numpy(O.dequant_kv_int4(g["vq4"], g["vs4"]))
    assert torch.equal(O.attention_decode(q, kd, vd, 33), torch.from_numpy(g["dec_int4"]))
    tq = torch.from_numpy(g["tq"])
    t = O.attention_tree(tq, k, v, [int(m) for m in g["tmask"]], 30, 30)
    assert torch.equal(t.transpose(1, 2).reshape(5, -1), torch.from_numpy(g["tree_fp16"]))


def test_medusa_tree_compile_matches_reference():
    with open(os.path.join(GOLDEN, "trees.json")) as f:
        ref = json.load(f)
    from axiomlm_tree_choices import DEFAULT_MEDUSA_TREE_CHOICES

    assert O.compile_medusa_tree(DEFAULT_MEDUSA_TREE_CHOICES, 4) == ref["default4"]
    assert O.compile_medusa_tree(DEFAULT_MEDUSA_TREE_CHOICES, 3) == ref["default3"]
    wide = O.compile_medusa_tree([(a, b) for a in range(6) for b in range(6)], 2)
    assert wide == ref["wide"]  # truncated at 31 paths, as the reference does


def _small_model(fx, cfg):
    from model_weights import make_weights

    W = make_weights(cfg, int(fx["seed"]), ln_random=bool(fx["ln_random"]), tied=bool(fx["tied"]))
    return O.OracleModel(cfg, W, rope_len=cfg["block_size"])


@pytest.mark.parametrize("name", ["small_fp16", "small_fp8", "small_int4", "small_fp8_ring", "small_tied"])
def test_oracle_model_greedy_matches_reference(name):
    from model_weights import SMALL

    fx = _load(f"{name}.npz")
    m = _small_model(fx, SMALL)
    hd = SMALL["d_model"] // SMALL["n_head"]
    kv = "fp16" if "fp16" in name or "tied" in name else ("fp8" if "fp8" in name else "int4")
    cache = O.OracleCache(SMALL["n_layer"], 1, SMALL["n_kv_head"], int(fx["max_seq"]), hd, kv, bool(fx["ring"]))
    prompt = fx["prompt"]
    logits, _ = m.forward(prompt, cache)
    steps = [logits[0, -1]]
    toks = [int(torch.argmax(logits[0, -1]))]
    for _ in range(len(fx["tokens"]) - 1):
        logits, _ = m.forward(np.array([[toks[-1]]]), cache)
        steps.append(logits[0, -1])
        toks.append(int(torch.argmax(logits[0, -1])))
    assert toks == fx["tokens"].tolist()
    # the oracle is the reference's own op sequence: logits are bit-identical
    assert np.array_equal(torch.stack(steps).to(torch.float16).numpy().view(np.uint16), fx["logits"].view(np.uint16))
    if "tree_logits" in fx.files:
        tl, _ = m.forward_tree(fx["tree_tokens"], cache, fx["tree_depths"].tolist(), fx["tree_mask"].tolist())
        assert np.array_equal(tl[0].float().numpy(), fx["tree_logits"].astype(np.float32))


@pytest.mark.parametrize("name", ["small_q8", "small_q4km", "small_q4"])
def test_oracle_model_q8_modes_match_reference(name):
    """The oracle in the reference's "q8" and "q4_k_m" modes against the
    reference's own greedy decode of the same model (tests/golden/make_golden.py
    --modes-only): tokens and logits bit-identical."""
    from model_weights import SMALL, make_weights

    fx = _load(f"{name}.npz")
    mode = str(fx["mode"])
    W = make_weights(SMALL, int(fx["seed"]), ln_random=bool(fx["ln_random"]))
    packs = None
    if mode in ("q4_k_m", "q4"):
        packs = {k: [(fx[f"pk_{k}_p_{i}"], fx[f"pk_{k}_s_{i}"]) for i in range(SMALL["n_layer"])]
                 for k in ("c_attn", "c_proj", "gu") + (("wd",) if mode == "q4" else ())}
        if mode == "q4":
            packs["lmh"] = (fx["pk_lmh_p"], fx["pk_lmh_sb"])
    m = O.OracleModel(SMALL, W, rope_len=SMALL["block_size"], weight_format=mode, packs=packs)
    hd = SMALL["d_model"] // SMALL["n_head"]
    cache = O.OracleCache(SMALL["n_layer"], 1, SMALL["n_kv_head"], int(fx["max_seq"]), hd, "fp16", False)
    logits, _ = m.forward(fx["prompt"], cache)
    steps = [logits[0, -1]]
    toks = [int(torch.argmax(logits[0, -1]))]
    for _ in range(len(fx["tokens"]) - 1):
        logits, _ = m.forward(np.array([[toks[-1]]]), cache)
        steps.append(logits[0, -1])
        toks.append(int(torch.argmax(logits[0, -1])))
    assert toks == fx["tokens"].tolist()
    assert np.array_equal(torch.stack(steps).to(torch.float16).numpy().view(np.uint16), fx["logits"].view(np.uint16))
