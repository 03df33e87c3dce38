"""Generate the golden fixtures by running the reference's own CPU path.

Run in a container where the reference checkout is available (it is NOT
available on GPU boxes; the fixtures it writes are committed instead):

    python tests/golden/make_golden.py --reference /path/to/AxiomLM [--skip-tiny]

Every fixture stores seeded inputs together with the reference's outputs for
them.  The oracle (``oracle/axb_oracle.py``) is checked against these in
``tests/test_oracle_golden.py``; the CUDA path is then checked against the
oracle and, for the model-level cases, against these same reference outputs.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from model_weights import SMALL, TINY, make_hf_checkpoint, make_prompt, make_weights  # noqa: E402


def _np(t):
    return t.detach().cpu().numpy()


def gen_quant(q):
    g = torch.Generator().manual_seed(1234)
    out = {}
    # ragged N (not a multiple of 8 or 16) exercises tile padding
    W = torch.randn(40, 256, generator=g) * 0.02
    W[3, 17] = 0.5  # outlier
    W[7, :64] = 0.0  # constant group
    out["W"] = _np(W)
    wm, sb = q.pack_linear_q4_marlin(W, clip_search=False)
    out["q4m_w"], out["q4m_sb"] = _np(wm), _np(sb)
    out["q4m_dq"] = _np(q.dequantize_q4_marlin(wm, sb, 256, out_features=40))
    wm2, sb2 = q.pack_linear_q4_marlin(W, clip_search=True)
    out["q4m_clip_w"], out["q4m_clip_sb"] = _np(wm2), _np(sb2)
    out["q4m_clip_dq"] = _np(q.dequantize_q4_marlin(wm2, sb2, 256, out_features=40))
    p, s = q.pack_linear_q4_g64(W)
    out["q4g_w"], out["q4g_sb"], out["q4g_dq"] = _np(p), _np(s), _np(q.dequantize_q4_g64(p, s, 256))
    p, s = q.pack_linear_q8_g64(W)
    out["q8_w"], out["q8_sb"], out["q8_dq"] = _np(p), _np(s), _np(q.dequantize_q8_g64(p, s, 256))
    idx = torch.tensor([[0, 39, 5], [7, 7, 12]])
    out["q8_rows_idx"] = _np(idx)
    out["q8_rows"] = _np(q.dequant_q8_rows(idx, p, s))
    Wt = torch.randn(32, 256, generator=g) * 0.02
    out["Wt"] = _np(Wt)
    p, s = q.pack_linear_ternary(Wt)
    out["ter_w"], out["ter_s"], out["ter_dq"] = _np(p), _np(s), _np(q.dequantize_ternary(p, s, 256))
    p, s = q.pack_linear_q2_k(Wt)
    out["q2_w"], out["q2_sb"], out["q2_dq"] = _np(p), _np(s), _np(q.dequantize_q2_k(p, s, 256))
    # reference GEMV (dequant + F.linear in fp16) on a few activations
    x = torch.randn(3, 256, generator=g).to(torch.float16)
    out["x"] = _np(x)
    out["q4m_y"] = _np(q.qmv_q4_marlin(x, wm, sb, out_features=40))
    out["ter_y"] = _np(q.qmv_ternary(x, *q.pack_linear_ternary(Wt)))
    out["q2_y"] = _np(q.qmv_q2_k(x, *q.pack_linear_q2_k(Wt)))
    return out


def gen_kv(q):
    g = torch.Generator().manual_seed(99)
    out = {}
    for hd in (64, 128):
        x = torch.randn(2, 3, 5, hd, generator=g).to(torch.float16)
        x[0, 0, 0, 3] = 60000.0  # near fp16 max
        x[0, 1, 1, :] = x[0, 1, 1, :] * 1e-3
        x[1, 2, 4, 10] = -300.0
        kq, ks, vq, vs = q.quantize_kv_fp8(x, x.flip(-1))
        out[f"x{hd}"] = _np(x)
        out[f"fp8_q{hd}"], out[f"fp8_s{hd}"] = _np(kq), _np(ks)
        out[f"fp8_vq{hd}"], out[f"fp8_vs{hd}"] = _np(vq), _np(vs)
        out[f"fp8_dq{hd}"] = _np(q.dequantize_kv_fp8(kq, ks, hd))
        kq, ks, vq, vs = q.quantize_kv_int4(x, x.flip(-1))
        out[f"i4_q{hd}"], out[f"i4_s{hd}"] = _np(kq), _np(ks)
        out[f"i4_dq{hd}"] = _np(q.dequantize_kv_int4(kq, ks, hd))
        # fp32 inputs (the model path: K after RoPE is fp32) round differently
        x32 = torch.randn(2, 3, 5, hd, generator=g) * 0.7
        x32[0, 0, 1, :] = x32[0, 0, 1, :] * 1e-4
        out[f"x32_{hd}"] = _np(x32)
        kq, ks, _, _ = q.quantize_kv_fp8(x32, x32)
        out[f"fp8_q32_{hd}"], out[f"fp8_s32_{hd}"] = _np(kq), _np(ks)
        kq, ks, _, _ = q.quantize_kv_int4(x32, x32)
        out[f"i4_q32_{hd}"], out[f"i4_s32_{hd}"] = _np(kq), _np(ks)
    return out


def gen_rope(modules):
    out = {}
    for hd in (64, 128):
        out[f"f{hd}"] = _np(torch.view_as_real(modules.precompute_rope_frequencies(hd, 64, 10000.0)))
    sc = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}
    out["f128_llama3"] = _np(torch.view_as_real(modules.precompute_rope_frequencies(128, 64, 500000.0, sc)))
    return out


def gen_attn(q, ops):
    g = torch.Generator().manual_seed(7)
    out = {}
    B, Hkv, S, hd, Hq = 1, 2, 40, 64, 8
    qv = torch.randn(1, Hq, 1, hd, generator=g).to(torch.float16)
    k = torch.randn(B, Hkv, S, hd, generator=g).to(torch.float16)
    v = torch.randn(B, Hkv, S, hd, generator=g).to(torch.float16)
    out["q"], out["k"], out["v"] = _np(qv), _np(k), _np(v)
    out["dec_fp16"] = _np(ops.gqa_flash_decode_mps(qv, k, v, 33))
    kq, ks, vq, vs = q.quantize_kv_fp8(k, v)
    out["kq8"], out["ks8"], out["vq8"], out["vs8"] = _np(kq), _np(ks), _np(vq), _np(vs)
    out["dec_fp8"] = _np(ops.gqa_flash_decode_mps(qv, kq, vq, 33, 0, ks, vs, "fp8"))
    kq, ks, vq, vs = q.quantize_kv_int4(k, v)
    out["kq4"], out["ks4"], out["vq4"], out["vs4"] = _np(kq), _np(ks), _np(vq), _np(vs)
    out["dec_int4"] = _np(ops.gqa_flash_decode_mps(qv, kq, vq, 33, 0, ks, vs, "int4"))
    # tree verify: T=5 nodes at write_pos 30 over prefix 30
    T = 5
    masks = [1, 3, 5, 11, 17]
    # (1, Hq, T, hd): the fallback at ops.py:740 re-reads head_dim from q's last
    # dimension, so only the 4-D form is well defined on the CPU path.
    qt = torch.randn(1, Hq, T, hd, generator=g).to(torch.float16)
    out["tq"] = _np(qt)
    out["tmask"] = np.array(masks, np.int64)
    y = ops.gqa_tree_verify_mps(qt, k, v, masks, 30, 30, Hq)
    out["tree_fp16"] = _np(y.reshape(T, Hq * hd))
    return out


def _ref_model(cfg, W, tied, mode="q4_rtn"):
    from axiomlm.models.transformer import ModelConfig, Transformer

    mc = ModelConfig(block_size=cfg["block_size"], vocab_size=cfg["vocab"], n_layer=cfg["n_layer"],
                     n_head=cfg["n_head"], n_embd=cfg["d_model"], n_kv_head=cfg["n_kv_head"],
                     intermediate_size=cfg["ffn"], rms_norm_eps=cfg["eps"], rope_theta=cfg["theta"],
                     tie_word_embeddings=tied)
    m = Transformer(mc, init_weights=False)
    with torch.no_grad():
        m.transformer.wte.weight.copy_(W["wte"])
        if not tied:
            m.lm_head.weight.copy_(W["lm_head"])
        for b, lw in zip(m.transformer.h, W["layers"]):
            b.attn.c_attn.weight.copy_(lw["c_attn"])
            b.attn.c_proj.weight.copy_(lw["c_proj"])
            b.mlp.w_gate.weight.copy_(lw["w_gate"])
            b.mlp.w_up.weight.copy_(lw["w_up"])
            b.mlp.w_down.weight.copy_(lw["w_down"])
            b.ln_1.weight.copy_(lw["ln_1"])
            b.ln_2.weight.copy_(lw["ln_2"])
        m.transformer.ln_f.weight.copy_(W["ln_f"])
    m.eval()
    m.quantize(mode)
    return m


# The reference's MSE-clipped MARLIN packs of a q4_k_m model
# (_ensure_quant_weights, quant.py:495-571), per layer.  No packer here
# repeats the clip search, so the GPU test serves these tensors as packed; the
# model's Q8_G64 tensors (w_down, lm_head, embeddings) are plain RTN and are
# packed again on the GPU.
_PACKED_Q4 = ("c_attn_p", "c_attn_s", "c_proj_p", "c_proj_s", "gu_p", "gu_s")


def _packed_arrays(m, keys=_PACKED_Q4, single=()):
    qw = m._ensure_quant_weights(torch.device("cpu"))
    out = {}
    for k in keys:
        for i, t in enumerate(qw[k]):
            out[f"pk_{k}_{i}"] = _np(t)
    for k in single:
        out[f"pk_{k}"] = _np(qw[k])
    return out


def gen_model(cfg, seed, prompt_len, n_new, kv, ln_random, tied=False, with_tree=False, ring=None, mode="q4_rtn"):
    from axiomlm.engine.medusa import DEFAULT_MEDUSA_TREE_CHOICES, compile_medusa_tree
    from axiomlm.engine.paged_cache import StaticKVCache

    W = make_weights(cfg, seed, ln_random=ln_random, tied=tied)
    m = _ref_model(cfg, W, tied, mode)
    hd = cfg["d_model"] // cfg["n_head"]
    max_seq = ring if ring else cfg["block_size"]
    prompt = make_prompt(prompt_len, cfg["vocab"], seed + 1)
    out = {"prompt": _np(prompt), "seed": np.array(seed), "ln_random": np.array(int(ln_random)),
           "tied": np.array(int(tied)), "max_seq": np.array(max_seq), "ring": np.array(int(bool(ring))),
           "mode": np.array(mode)}
    if mode == "q4_k_m":
        out.update(_packed_arrays(m))
    elif mode == "q4":  # every projection and the lm_head clip-searched: the packer under test
        out.update(_packed_arrays(m, _PACKED_Q4 + ("wd_p", "wd_s"), ("lmh_p", "lmh_sb")))
    with torch.no_grad():
        cache = StaticKVCache(1, max_seq, cfg["n_layer"], cfg["n_kv_head"], hd, dtype=torch.float16,
                              device="cpu", ring_buffer=bool(ring), cache_dtype=kv)
        logits, _, _ = m(prompt, kv_caches=cache)
        steps = [logits[0, -1].clone()]
        toks = [int(torch.argmax(logits[0, -1]))]
        for _ in range(n_new - 1):
            logits, _, _ = m(torch.tensor([[toks[-1]]]), kv_caches=cache)
            steps.append(logits[0, -1].clone())
            toks.append(int(torch.argmax(logits[0, -1])))
        out["tokens"] = np.array(toks, np.int64)
        L = torch.stack(steps).float()
        out["logits"] = _np(L.to(torch.float16))
        top2 = torch.topk(L, 2, dim=-1).values
        out["margin"] = _np((top2[:, 0] - top2[:, 1]) / top2[:, 0].abs().clamp(min=1e-6))
        if with_tree:
            tree = compile_medusa_tree(DEFAULT_MEDUSA_TREE_CHOICES, 4)
            T = tree["num_nodes"]
            g = torch.Generator().manual_seed(seed + 2)
            verif = torch.randint(0, cfg["vocab"], (1, T), generator=g)
            verif[0, 0] = toks[-1]
            seen0 = cache.total_seen_tokens[0]
            tl, _, _ = m.forward_tree_verify(verif, [cache] * cfg["n_layer"], tree["tree_depths"],
                                             tree["tree_mask"], return_medusa=False)
            out["tree_tokens"] = _np(verif)
            out["tree_logits"] = _np(tl[0])
            out["tree_seen"] = np.array(seen0)
            out["tree_depths"] = np.array(tree["tree_depths"])
            out["tree_mask"] = np.array(tree["tree_mask"], np.int64)
    return out


def _gen_small(q, ops, modules, compile_medusa_tree, DEFAULT_MEDUSA_TREE_CHOICES):
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **gen_quant(q))
    np.savez_compressed(os.path.join(HERE, "kv.npz"), **gen_kv(q))
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **gen_rope(modules))
    np.savez_compressed(os.path.join(HERE, "attn.npz"), **gen_attn(q, ops))
    trees = {
        "default4": compile_medusa_tree(DEFAULT_MEDUSA_TREE_CHOICES, 4),
        "default3": compile_medusa_tree(DEFAULT_MEDUSA_TREE_CHOICES, 3),
        "wide": compile_medusa_tree([(a, b) for a in range(6) for b in range(6)], 2),
    }
    with open(os.path.join(HERE, "trees.json"), "w") as f:
        json.dump(trees, f)
    for kv in ("fp16", "fp8", "int4"):
        t0 = time.time()
        # the reference's CPU tree-verify path casts K/V straight to the cache
        # dtype (transformer.py:728-733), which is only meaningful for fp16 KV
        o = gen_model(SMALL, 11, 12, 24, kv, ln_random=True, with_tree=(kv == "fp16"))
        np.savez_compressed(os.path.join(HERE, f"small_{kv}.npz"), **o)
        print(f"small {kv}: {time.time() - t0:.1f}s tokens={o['tokens'][:8]}")
    o = gen_model(SMALL, 21, 12, 40, "fp8", ln_random=True, ring=32)
    np.savez_compressed(os.path.join(HERE, "small_fp8_ring.npz"), **o)
    o = gen_model(SMALL, 31, 10, 16, "fp16", ln_random=True, tied=True)
    np.savez_compressed(os.path.join(HERE, "small_tied.npz"), **o)


def gen_mse(q):
    """pack_linear_q4_marlin's clip search (quant.py:495-571) with column
    importance, on fp32 and fp16 inputs (the model's parameters can be
    either): the packs the clip-search restatement must reproduce."""
    g = torch.Generator().manual_seed(4321)
    W = torch.randn(40, 256, generator=g) * 0.02
    W[5, 100] = 0.4  # outlier
    W[9, 64:128] = 0.01  # constant group
    imp_ln = (1.0 + 0.1 * torch.randn(256, generator=g)).abs()  # |ln weight| (c_attn, gate_up, lm_head)
    a = torch.randn(256, 256, generator=g) * 0.02
    b = torch.randn(256, 256, generator=g) * 0.02
    imp_sw = a.norm(dim=1) * b.norm(dim=1)  # |w_gate row| * |w_up row| (w_down)
    out = {"W": _np(W), "imp_ln": _np(imp_ln), "imp_sw": _np(imp_sw)}
    for tag, w, imp in (("f32_ln", W, imp_ln), ("f16_none", W.half(), None), ("f16_sw", W.half(), imp_sw)):
        wm, sb = q.pack_linear_q4_marlin(w, clip_search=True, col_importance=imp)
        out[f"{tag}_w"], out[f"{tag}_sb"] = _np(wm), _np(sb)
    np.savez_compressed(os.path.join(HERE, "quant_mse.npz"), **out)
    print("quant_mse:", len(out), "arrays")


def gen_hf():
    """The reference's load_hf_safetensors (hf_importer.py:199-305) on seeded
    tiny checkpoints: its fp16 parameters, which the importer here must
    reproduce from the same checkpoint files."""
    import tempfile

    from axiomlm.utils.hf_importer import load_hf_safetensors

    out = {}
    for tag, seed, bias, tied, shards in (("llama", 71, False, False, 1), ("qwen", 72, True, True, 2)):
        with tempfile.TemporaryDirectory() as d:
            make_hf_checkpoint(d, seed, bias=bias, tied=tied, shards=shards)
            m = load_hf_safetensors(d, device="cpu", dtype=torch.float16)
        out[f"{tag}_wte"] = _np(m.transformer.wte.weight)
        out[f"{tag}_ln_f"] = _np(m.transformer.ln_f.weight)
        out[f"{tag}_lm_head"] = _np(m.lm_head.weight)
        out[f"{tag}_block_size"] = np.array(m.config.block_size)
        out[f"{tag}_theta"] = np.array(m.config.rope_theta)
        for i, b in enumerate(m.transformer.h):
            out[f"{tag}_{i}_c_attn"] = _np(b.attn.c_attn.weight)
            if b.attn.c_attn.bias is not None:
                out[f"{tag}_{i}_c_attn_b"] = _np(b.attn.c_attn.bias)
            out[f"{tag}_{i}_c_proj"] = _np(b.attn.c_proj.weight)
            out[f"{tag}_{i}_w_gate"] = _np(b.mlp.w_gate.weight)
            out[f"{tag}_{i}_w_up"] = _np(b.mlp.w_up.weight)
            out[f"{tag}_{i}_w_down"] = _np(b.mlp.w_down.weight)
            out[f"{tag}_{i}_ln_1"] = _np(b.ln_1.weight)
            out[f"{tag}_{i}_ln_2"] = _np(b.ln_2.weight)
    np.savez_compressed(os.path.join(HERE, "hf_import.npz"), **out)
    print("hf_import:", len(out), "arrays")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AXIOMLM_REFERENCE", ""))
    ap.add_argument("--skip-tiny", action="store_true")
    ap.add_argument("--tiny-only", action="store_true", help="regenerate only the tiny-model fixtures")
    ap.add_argument("--mse-only", action="store_true",
                    help="regenerate only the clip-search packing fixture (quant_mse.npz)")
    ap.add_argument("--hf-only", action="store_true",
                    help="regenerate only the Hugging Face importer fixture (hf_import.npz)")
    ap.add_argument("--modes-only", action="store_true",
                    help="regenerate only the q8 / q4_k_m / q4 model fixtures (small_q8, small_q4km, small_q4)")
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        raise SystemExit("pass --reference <path to the AxiomLM checkout>")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(os.cpu_count() or 1)
    import axiomlm.kernels.ops as ops
    import axiomlm.kernels.quant as q
    import axiomlm.models.modules as modules
    from axiomlm.engine.medusa import DEFAULT_MEDUSA_TREE_CHOICES, compile_medusa_tree

    # with one of the --*-only flags, only that part; with none, everything
    only = [k for k in ("tiny", "mse", "hf", "modes") if getattr(args, f"{k}_only")]

    def part(name):
        return not only or name in only

    if part("mse"):
        gen_mse(q)
    if part("hf"):
        gen_hf()
    if part("modes"):
        # the reference's other quantized-forward modes (transformer.py:797-799):
        # Q8_G64 everywhere ("q8"), MSE-clipped Q4 with Q8 w_down and lm_head
        # ("q4_k_m"), MSE-clipped Q4 everywhere ("q4")
        for mode, name, seed in (("q8", "small_q8", 41), ("q4_k_m", "small_q4km", 55), ("q4", "small_q4", 84)):
            t0 = time.time()
            o = gen_model(SMALL, seed, 12, 16, "fp16", ln_random=True, mode=mode)
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **o)
            print(f"{name}: {time.time() - t0:.1f}s tokens={o['tokens'][:8]}")
    if not only:
        _gen_small(q, ops, modules, compile_medusa_tree, DEFAULT_MEDUSA_TREE_CHOICES)
    if part("tiny") and not args.skip_tiny:
        for kv in ("fp16", "fp8"):
            t0 = time.time()
            o = gen_model(TINY, 5, 128, 128, kv, ln_random=False)
            # the full (128, 32000) logits are too large for a fixture: keep,
            # per step, the top-32 entries, a fixed sample of 256 columns and
            # the largest |logit| (the scale of the per-step tolerance)
            lg = torch.from_numpy(o.pop("logits")).float()
            top = torch.topk(lg, 32, dim=-1)
            cols = torch.randperm(lg.shape[1], generator=torch.Generator().manual_seed(77))[:256].sort().values
            o["logit_top_idx"] = _np(top.indices.to(torch.int32))
            o["logit_top_val"] = _np(top.values.to(torch.float16))
            o["logit_cols"] = _np(cols.to(torch.int32))
            o["logit_col_val"] = _np(lg[:, cols].to(torch.float16))
            o["logit_absmax"] = _np(lg.abs().amax(-1))
            np.savez_compressed(os.path.join(HERE, f"tiny_{kv}.npz"), **o)
            print(f"tiny {kv}: {time.time() - t0:.1f}s min-margin={o['margin'].min():.2e}")


if __name__ == "__main__":
    main()
