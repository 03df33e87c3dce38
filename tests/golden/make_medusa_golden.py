"""Generate the Medusa / speculative-decoding golden fixtures from the reference.

Run in a container that has the AxiomLM checkout (CPU only):

    python tests/golden/make_medusa_golden.py --reference <path to AxiomLM>

Writes ``medusa_small.npz`` and ``sequoia.npz`` next to this file:

* medusa_small.npz -- the SMALL parity model (seed 11, as small_fp16) with 4
  residual Medusa heads trained by the reference's ``train_medusa_heads`` on
  the model's own greedy continuation, then packed by ``quantize("q4_rtn")``
  (the MARLIN head packs are stored, so the GPU side serves the very same
  codes).  Reference outputs: ``eval_medusa_heads`` logits on seeded rows,
  and ``MedusaSpeculativeDecoder.generate`` at temperature 0 with the default
  tree and with the linear chain: the tokens, the cache length before every
  verification pass and every accepted node list.
* sequoia.npz -- seeded tree logits with ``SequoiaTreeVerifier.verify_tree_step``
  and ``sample_without_replacement`` results at several temperatures and
  generator seeds (JSON in the ``results`` entry).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from model_weights import SMALL, make_prompt, make_weights  # noqa: E402

SEED = 11
PROMPT_LEN = 12
N_HEADS = 4
N_NEW = 40


def _np(t):
    return t.detach().cpu().numpy()


def _model(cfg, W):
    from axiomlm.models.transformer import ModelConfig, Transformer

    mc = ModelConfig(block_size=cfg["block_size"], vocab_size=cfg["vocab"], n_layer=cfg["n_layer"],
                     n_head=cfg["n_head"], n_embd=cfg["d_model"], n_kv_head=cfg["n_kv_head"],
                     intermediate_size=cfg["ffn"], rms_norm_eps=cfg["eps"], rope_theta=cfg["theta"],
                     tie_word_embeddings=False)
    m = Transformer(mc, init_weights=False)
    with torch.no_grad():
        m.transformer.wte.weight.copy_(W["wte"])
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
    return m


def _cache(cfg):
    from axiomlm.engine.paged_cache import StaticKVCache

    hd = cfg["d_model"] // cfg["n_head"]
    return StaticKVCache(1, cfg["block_size"], cfg["n_layer"], cfg["n_kv_head"], hd, dtype=torch.float16,
                         device="cpu", cache_dtype="fp16")


def _traced_generate(m, cfg, prompt, tree_choices):
    """generate() with the cache length at every verification pass and every
    compact_tree_path accepted list recorded."""
    from axiomlm.engine.medusa import MedusaSpeculativeDecoder

    cache = _cache(cfg)
    seen_at_verify, accepted_lists = [], []
    orig_tree, orig_med = m.forward_tree_verify, m.forward_with_medusa
    orig_compact = cache.compact_tree_path

    def tree_verify(*a, **k):
        seen_at_verify.append(int(cache.total_seen_tokens[0]))
        return orig_tree(*a, **k)

    def with_medusa(idx, *a, **k):
        if cache.total_seen_tokens[0] > 0:  # not the prefill
            seen_at_verify.append(int(cache.total_seen_tokens[0]))
        return orig_med(idx, *a, **k)

    def compact(write_pos, accepted_indices, new_total_seen=None):
        accepted_lists.append([int(a) for a in accepted_indices])
        return orig_compact(write_pos, accepted_indices, new_total_seen)

    m.forward_tree_verify, m.forward_with_medusa = tree_verify, with_medusa
    cache.compact_tree_path = compact
    try:
        dec = MedusaSpeculativeDecoder(num_heads=N_HEADS, temperature=0.0, tree_choices=tree_choices)
        toks, stats = dec.generate(m, prompt, max_new_tokens=N_NEW, cache=cache, device=torch.device("cpu"))
    finally:
        m.forward_tree_verify, m.forward_with_medusa = orig_tree, orig_med
    return toks, stats, seen_at_verify, accepted_lists


def gen_medusa(args):
    from axiomlm.engine.medusa import DEFAULT_MEDUSA_TREE_CHOICES, train_medusa_heads

    cfg = SMALL
    W = make_weights(cfg, SEED, ln_random=True)
    m = _model(cfg, W)
    prompt = make_prompt(PROMPT_LEN, cfg["vocab"], SEED + 1)
    # the fp32 model's own greedy continuation is the heads' training text
    seq = prompt.clone()
    with torch.no_grad():
        for _ in range(96):
            logits = m(seq)[0]
            seq = torch.cat([seq, logits[:, -1:].argmax(-1)], 1)
    torch.manual_seed(SEED + 3)
    m.add_medusa_heads(num_heads=N_HEADS, use_residual=True)
    losses = train_medusa_heads(m, seq, epochs=args.epochs, lr=3e-3)
    print(f"medusa heads trained: loss {losses[0]:.3f} -> {losses[-1]:.3f}")
    for p in m.parameters():
        p.requires_grad = False
    m.quantize("q4_rtn")
    qw = m._ensure_quant_weights(torch.device("cpu"))
    out = {"seed": np.array(SEED), "prompt": _np(prompt[0]), "n_new": np.array(N_NEW), "n_heads": np.array(N_HEADS)}
    for k, hp in enumerate(qw["medusa_packs"]):
        out[f"head{k}_p"] = _np(hp["head_p"])
        out[f"head{k}_s"] = _np(hp["head_s"])
        out[f"res{k}_p"] = _np(hp["res_p"])
        out[f"res{k}_s"] = _np(hp["res_s"])
    # eval_medusa_heads on seeded final-norm rows
    g = torch.Generator().manual_seed(SEED + 4)
    xn = torch.randn(1, 3, cfg["d_model"], generator=g)
    with torch.no_grad():
        ml = m.eval_medusa_heads(xn)
    out["eval_x"] = _np(xn[0])
    out["eval_logits"] = _np(torch.stack([t[0] for t in ml]).to(torch.float16))  # (K, 3, V)
    with torch.no_grad():
        for name, choices in (("tree", DEFAULT_MEDUSA_TREE_CHOICES), ("chain", None)):
            toks, stats, seen, acc = _traced_generate(m, cfg, prompt[0].tolist(), choices)
            out[f"{name}_tokens"] = np.array(toks, np.int64)
            out[f"{name}_seen"] = np.array(seen, np.int64)
            flat = [a for lst in acc for a in lst]
            out[f"{name}_acc_flat"] = np.array(flat, np.int64)
            out[f"{name}_acc_len"] = np.array([len(lst) for lst in acc], np.int64)
            out[f"{name}_stats"] = np.array([stats["forward_calls"], stats["drafted_tokens"],
                                             stats["accepted_draft_tokens"], stats["new_tokens"]], np.int64)
            steps = np.diff(np.array(seen + [len(toks) - 1]))
            print(f"{name}: {stats['new_tokens']} tokens in {stats['forward_calls']} forward calls, "
                  f"accepted {stats['accepted_draft_tokens']} of {stats['drafted_tokens']}; per-pass advance {steps}")
    np.savez_compressed(os.path.join(HERE, "medusa_small.npz"), **out)


def gen_sequoia():
    from axiomlm.engine.medusa import DEFAULT_MEDUSA_TREE_CHOICES, compile_medusa_tree
    from axiomlm.speculative.sampling import SequoiaTreeVerifier, sample_without_replacement

    tree = compile_medusa_tree(DEFAULT_MEDUSA_TREE_CHOICES, 4)
    T, V = tree["num_nodes"], 64
    g = torch.Generator().manual_seed(7)
    logits = (torch.randn(T, V, generator=g) * 3.0).to(torch.float16).float()
    # drafts: each node's token is one of its parent's likelier tokens
    order = logits.argsort(dim=-1, descending=True)
    verif = [int(order[0, 0])]
    for u in range(1, T):
        verif.append(int(order[tree["parent"][u], tree["topk_rank"][u]]))
    results = []
    for temp in (0.0, 0.7, 1.3):
        for seed in range(6):
            v = SequoiaTreeVerifier(temperature=temp, generator=torch.Generator().manual_seed(100 + seed))
            for max_accept in (None, 2):
                acc, em, st = v.verify_tree_step(logits, tree, verif, temperature=temp, max_accept=max_accept)
                results.append(dict(kind="tree", temp=temp, seed=100 + seed, max_accept=max_accept, accepted=acc,
                                    emitted=em, stats=st))
        for seed in range(3):
            gen = torch.Generator().manual_seed(200 + seed)
            idx = sample_without_replacement(logits[:4], 5, temperature=temp, generator=gen)
            results.append(dict(kind="swr", temp=temp, seed=200 + seed, k=5, rows=4, indices=idx.tolist()))
    np.savez_compressed(os.path.join(HERE, "sequoia.npz"), logits=_np(logits.to(torch.float16)),
                        verif=np.array(verif, np.int64), results=np.array(json.dumps(results)))
    print(f"sequoia: {len(results)} cases")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AXIOMLM_REFERENCE", ""))
    ap.add_argument("--epochs", type=int, default=300)
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        raise SystemExit("pass --reference <path to the AxiomLM checkout>")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(os.cpu_count() or 1)
    gen_sequoia()
    gen_medusa(args)


if __name__ == "__main__":
    main()
