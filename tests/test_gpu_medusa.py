"""Medusa speculative decoding on the GPU against the oracle and the
reference's own outputs (tests/golden/medusa_small.npz, made by
make_medusa_golden.py):

* the device greedy walk (axb_tree_accept) vs the oracle's walk
  (engine/medusa.py:312-330), bit-exact;
* the per-row top-k vs a stable (value desc, index asc) sort;
* the device-counted KV compaction vs the host-list compaction;
* the quantized Medusa heads vs the reference's eval_medusa_heads (rel 2e-3);
* whole speculative generations vs the reference's
  MedusaSpeculativeDecoder.generate: identical tokens, identical accepted
  node lists (accept lengths) at every verification pass, identical stats.
"""

import os
import random

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from model_weights import SMALL, make_weights
from oracle import axb_oracle as O

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


@pytest.fixture(scope="module")
def md():
    from axiomlm_b200 import medusa

    return medusa


def _fx():
    return np.load(os.path.join(GOLDEN, "medusa_small.npz"))


def _packs(fx):
    K = int(fx["n_heads"])
    return [{"head_p": torch.from_numpy(fx[f"head{k}_p"]), "head_s": torch.from_numpy(fx[f"head{k}_s"]),
             "res_p": torch.from_numpy(fx[f"res{k}_p"]), "res_s": torch.from_numpy(fx[f"res{k}_s"])}
            for k in range(K)]


def _decoder(fx, md, max_seq=None, kv="fp16"):
    from axiomlm_b200.model import QuantizedDecoder

    W = make_weights(SMALL, int(fx["seed"]), ln_random=True)
    dec = QuantizedDecoder.from_weights(SMALL, W, "q4_rtn", kv_dtype=kv, max_seq=max_seq or SMALL["block_size"],
                                        max_tokens=64, rope_len=SMALL["block_size"])
    dec.add_medusa_heads(md.MedusaHeads.from_packs(_packs(fx), SMALL["d_model"], SMALL["vocab"]))
    return dec


def _rel(a, b):
    a = torch.as_tensor(a).float().cpu()
    b = torch.as_tensor(b).float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-6))


# ------------------------------------------------------------ device walk
def _random_tree(md, rng, heads, nodes):
    choices = set()
    for _ in range(4 * nodes):
        d = rng.randint(1, heads)
        choices.add(tuple(rng.randint(0, 7) for _ in range(d)))
    return md.compile_medusa_tree(sorted(choices), heads, max_nodes=64)


def test_tree_accept_matches_oracle(md):
    import axiomlm_b200._lib as L

    rng = random.Random(1)
    cases = 0
    for trial in range(200):
        tree = _random_tree(md, rng, rng.randint(1, 6), rng.randint(1, 80))
        T = tree["num_nodes"]
        verif = [rng.randint(0, 5) for _ in range(T)]
        preds = [rng.randint(0, 5) for _ in range(T)]
        # plant a deep path half of the time: follow random children
        if trial % 2 == 0:
            cur = 0
            while tree["children"][cur]:
                c = rng.choice(tree["children"][cur])
                preds[cur] = verif[c]
                cur = c
        budget = rng.choice([1, 2, 3, 5, 64, 1000])
        dt = md.DeviceTree(tree, "cuda")
        res = md.tree_accept(dt, torch.tensor(verif, dtype=torch.int32, device="cuda"),
                             torch.tensor(preds, dtype=torch.int32, device="cuda"), budget).cpu().tolist()
        acc, em = O.greedy_tree_accept(preds, verif, tree["children"], budget)
        n = res[0]
        H = L.TREE_RESULT_HDR
        assert n == len(acc) and res[2] == len(em) and res[1] == acc[-1] and res[3] == em[-1], (trial, res[:4])
        assert res[H:H + n] == acc
        assert res[H + L.TREE_MAX_NODES:H + L.TREE_MAX_NODES + n] == em
        cases += n > 2
    assert cases > 30  # deep paths were exercised


def test_tree_accept_rejects_bad_args(md):
    from axiomlm_b200._lib import AxbError

    tree = md.compile_medusa_tree(md.DEFAULT_MEDUSA_TREE_CHOICES, 4)
    dt = md.DeviceTree(tree, "cuda")
    v = torch.zeros(dt.T, dtype=torch.int32, device="cuda")
    with pytest.raises(AxbError):
        md.tree_accept(dt, v, v, 0)


# ------------------------------------------------------------------ top-k
def _stable_topk(x: np.ndarray, k: int) -> np.ndarray:
    order = np.lexsort((np.arange(x.shape[-1])[None, :].repeat(x.shape[0], 0), -x.astype(np.float32)), axis=-1)
    return order[:, :k]


@pytest.mark.parametrize("n", [1000, 1001, 32000, 128256])
@pytest.mark.parametrize("k", [1, 4, 10, 64])
def test_topk_rows(md, n, k):
    g = torch.Generator(device="cuda").manual_seed(n * 7 + k)
    x = (torch.randn(5, n, device="cuda", generator=g) * 4).half()
    x[1] = torch.round(x[1])  # few distinct values: ties everywhere
    x[2] = -x[2].abs()  # all negative
    x[3] = 0.0
    x[3, n // 3] = 1.0
    got = md.topk_rows(x, k).cpu().numpy()
    ref = _stable_topk(x.cpu().numpy(), k)
    np.testing.assert_array_equal(got, ref)


def test_topk_strided_rows(md):
    x = (torch.randn(3, 4100, device="cuda") * 2).half()
    import axiomlm_b200._lib as L
    from axiomlm_b200 import ops

    out = torch.empty(3, 7, dtype=torch.int32, device="cuda")
    # rows of 4000 inside a 4100-wide buffer, offset by one element (no 16-byte alignment)
    L.call("axb_topk_rows", ops._p(x[:, 1:]), 3, 4000, 4100, 7, ops._p(out), ops._stream())
    ref = _stable_topk(x[:, 1:4001].cpu().numpy(), 7)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


# --------------------------------------------------------------- compaction
@pytest.mark.parametrize("kv", ["fp16", "fp8", "int4"])
def test_compact_kv_dev_matches_host_list(md, kv):
    import axiomlm_b200._lib as L
    from axiomlm_b200 import ops
    from axiomlm_b200.cache import StaticKVCache
    from axiomlm_b200.model import QuantizedDecoder

    def cache():
        c = StaticKVCache(1, 96, 2, 2, 64, cache_dtype=kv)
        g = torch.Generator(device="cuda").manual_seed(3)
        if c.cache.dtype == torch.uint8:
            c.cache.copy_(torch.randint(0, 256, c.cache.shape, generator=g, device="cuda", dtype=torch.int32))
            c.scales.copy_(torch.rand(c.scales.shape, generator=g, device="cuda"))
        else:
            c.cache.copy_(torch.randn(c.cache.shape, generator=g, device="cuda"))
        return c

    for acc in ([0, 2, 8, 15], [0, 1, 2], [0, 4], [0]):
        a, b = cache(), cache()
        before = b.cache.clone()
        ops.compact_tree_kv(a.cache, a.scales, 30, acc, kv)
        result = torch.zeros(L.TREE_RESULT_WORDS, dtype=torch.int32, device="cuda")
        result[0] = len(acc)
        result[L.TREE_RESULT_HDR:L.TREE_RESULT_HDR + len(acc)] = torch.tensor(acc, dtype=torch.int32)
        fake = type("D", (), {})()
        fake.cache = b
        QuantizedDecoder.compact_device(fake, 30, result)
        torch.cuda.synchronize()
        assert torch.equal(a.cache, b.cache), acc
        if a.scales is not None:
            assert torch.equal(a.scales, b.scales), acc
        if acc == sorted(acc) and acc == list(range(len(acc))):
            assert torch.equal(b.cache, before)


# ------------------------------------------------------------------ heads
def test_medusa_heads_match_reference(md):
    fx = _fx()
    heads = md.MedusaHeads.from_packs(_packs(fx), SMALL["d_model"], SMALL["vocab"])
    x = torch.from_numpy(fx["eval_x"]).cuda()
    out = heads(x.view(1, 3, -1))
    ref = fx["eval_logits"]  # (K, 3, V)
    for k in range(int(fx["n_heads"])):
        assert out[k].shape == (1, 3, SMALL["vocab"])
        assert _rel(out[k][0], ref[k]) < REL_TOL, k
        assert torch.equal(out[k][0].float().cpu().argmax(-1), torch.from_numpy(ref[k]).float().argmax(-1))
    # the device draft path (leaf row staging + top-k) agrees with eval
    norm = x.float().contiguous()
    for row in range(3):
        topk = heads.draft(norm, 3, leaf=row).cpu().numpy()
        lg = torch.stack([o[0, row] for o in out]).cpu().numpy()
        np.testing.assert_array_equal(topk, _stable_topk(lg, 3))


def test_medusa_heads_without_residual_stack(md):
    """Heads without residual blocks run as one stacked GEMV; the result
    matches head-by-head GEMVs (the two may split K differently, so the
    comparison is at the GEMV tolerance, not bitwise)."""
    from axiomlm_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(5)
    ws = [torch.randn(1024, 256, device="cuda", generator=g) * 0.05 for _ in range(3)]
    heads = md.MedusaHeads([(None, ops.pack_q4t(w, 128, True)) for w in ws])
    assert heads.head_stack is not None
    x = torch.randn(2, 256, device="cuda", generator=g)
    out = heads(x)
    for k, w in enumerate(heads.head):
        ref = x.half().float() @ w.dequant().float().t()
        per_head = ops.qgemm(x.half(), w)
        assert _rel(per_head, ref) < REL_TOL, ("per-head GEMV", k, _rel(per_head, ref))
        assert _rel(out[k], ref) < REL_TOL, ("stacked GEMV", k, _rel(out[k], ref))


# -------------------------------------------------------- whole generation
@pytest.mark.parametrize("mode", ["tree", "chain"])
def test_generate_matches_reference(md, mode):
    fx = _fx()
    dec = _decoder(fx, md)
    choices = md.DEFAULT_MEDUSA_TREE_CHOICES if mode == "tree" else None
    sd = md.MedusaSpeculativeDecoder(num_heads=int(fx["n_heads"]), tree_choices=choices)
    toks, stats = sd.generate(dec, fx["prompt"].tolist(), max_new_tokens=int(fx["n_new"]))
    assert toks == fx[f"{mode}_tokens"].tolist()
    # accept lengths: the cache length before every verification pass
    seen = [len(fx["prompt"])]
    for nodes in stats["accepted_nodes"][:-1]:
        seen.append(seen[-1] + len(nodes))
    assert seen == fx[f"{mode}_seen"].tolist()
    if mode == "tree":  # every accepted node list handed to compact_tree_path
        lens = fx["tree_acc_len"].tolist()
        flat = fx["tree_acc_flat"].tolist()
        ref_lists = [flat[sum(lens[:i]):sum(lens[:i + 1])] for i in range(len(lens))]
        assert stats["accepted_nodes"] == ref_lists
    calls, drafted, accepted, new = fx[f"{mode}_stats"].tolist()
    assert (stats["forward_calls"], stats["drafted_tokens"], stats["accepted_draft_tokens"],
            stats["new_tokens"]) == (calls, drafted, accepted, new)
    assert dec.status() == 0
    dec.close()


def test_generate_64_node_tree_is_lossless(md):
    """A 64-node tree (uint64 masks; beyond the reference's 32) emits exactly
    the greedy tokens."""
    fx = _fx()
    dec = _decoder(fx, md)
    choices = [(a, b, c) for a in range(4) for b in range(4) for c in range(4)]
    sd = md.MedusaSpeculativeDecoder(num_heads=4, tree_choices=choices, max_nodes=64)
    toks, stats = sd.generate(dec, fx["prompt"].tolist(), max_new_tokens=int(fx["n_new"]))
    assert stats["tree_nodes_per_step"] == 64
    assert toks == fx["tree_tokens"].tolist()
    assert stats["forward_calls"] < int(fx["n_new"])
    dec.close()


def test_generate_tree_falls_back_to_chain_near_cache_end(md):
    """engine/medusa.py:292-296: once the tree does not fit the cache the
    chain verification takes over; the output is still the greedy text."""
    fx = _fx()
    dec = _decoder(fx, md, max_seq=60)
    sd = md.MedusaSpeculativeDecoder(num_heads=4, tree_choices=md.DEFAULT_MEDUSA_TREE_CHOICES)
    toks, stats = sd.generate(dec, fx["prompt"].tolist(), max_new_tokens=int(fx["n_new"]))
    assert toks == fx["tree_tokens"].tolist()
    seen = [len(fx["prompt"])]
    for nodes in stats["accepted_nodes"][:-1]:
        seen.append(seen[-1] + len(nodes))
    assert any(s + 17 > 60 for s in seen)  # some passes ran as the chain
    dec.close()


def test_generate_sampled_regime(md):
    fx = _fx()
    dec = _decoder(fx, md)
    sd = md.MedusaSpeculativeDecoder(num_heads=4, temperature=0.8, tree_choices=md.DEFAULT_MEDUSA_TREE_CHOICES)
    runs = []
    for _ in range(2):
        toks, stats = sd.generate(dec, fx["prompt"].tolist(), max_new_tokens=24,
                                  generator=torch.Generator().manual_seed(4))
        assert len(toks) == len(fx["prompt"]) + 24 and all(0 <= t < SMALL["vocab"] for t in toks)
        assert stats["forward_calls"] <= 24
        runs.append(toks)
    assert runs[0] == runs[1]
    dec.close()
