"""Medusa host logic on the CPU: tree compilation, the greedy walk, the
Sequoia verifier and sampling, pinned to the reference's outputs
(tests/golden/trees.json from make_golden.py, tests/golden/sequoia.npz from
make_medusa_golden.py)."""

import json
import os
import random

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from axiomlm_b200 import medusa
from oracle import axb_oracle as O


def test_compile_tree_matches_reference():
    ref = json.load(open(os.path.join(GOLDEN, "trees.json")))
    cases = {"default4": (medusa.DEFAULT_MEDUSA_TREE_CHOICES, 4), "default3": (medusa.DEFAULT_MEDUSA_TREE_CHOICES, 3),
             "wide": ([(a, b) for a in range(6) for b in range(6)], 2)}
    for name, (choices, heads) in cases.items():
        mine = medusa.compile_medusa_tree(choices, heads)
        for key, val in ref[name].items():
            assert mine[key] == val, (name, key)


def test_compile_tree_64_nodes():
    choices = [(a, b) for a in range(8) for b in range(8)]
    t32 = medusa.compile_medusa_tree(choices, 2)
    t64 = medusa.compile_medusa_tree(choices, 2, max_nodes=64)
    assert t32["num_nodes"] == 32 and t64["num_nodes"] == 64
    # the first 32 nodes are the same tree; masks reach bit 63
    for key in ("tree_depths", "tree_mask", "parent", "head_idx", "topk_rank"):
        assert t64[key][:32] == t32[key]
    assert t64["tree_mask"][63] >> 63 == 1
    for u in range(1, 64):
        p = t64["parent"][u]
        assert t64["tree_mask"][u] == t64["tree_mask"][p] | (1 << u)
    with pytest.raises(ValueError):
        medusa.compile_medusa_tree(choices, 2, max_nodes=65)


def test_chain_tree():
    t = medusa.chain_tree(4)
    assert t["num_nodes"] == 5 and t["parent"] == [-1, 0, 1, 2, 3] and t["tree_mask"] == [1, 3, 7, 15, 31]
    assert t["head_idx"] == [-1, 0, 1, 2, 3] and t["topk_rank"] == [-1, 0, 0, 0, 0]


def random_tree(rng, heads, nodes):
    choices = set()
    for _ in range(4 * nodes):  # bounded: small head counts have few distinct paths
        d = rng.randint(1, heads)
        choices.add(tuple(rng.randint(0, 5) for _ in range(d)))
    return medusa.compile_medusa_tree(sorted(choices), heads, max_nodes=64)


def test_greedy_walk_matches_oracle():
    rng = random.Random(5)
    for _ in range(300):
        tree = random_tree(rng, rng.randint(1, 5), rng.randint(1, 40))
        T = tree["num_nodes"]
        verif = [rng.randint(0, 7) for _ in range(T)]
        preds = [rng.randint(0, 7) for _ in range(T)]
        budget = rng.randint(1, 8)
        assert medusa.greedy_tree_walk(preds, verif, tree["children"], budget) == \
            O.greedy_tree_accept(preds, verif, tree["children"], budget)


def test_linear_chain_is_the_walk_on_the_chain_tree():
    """engine/medusa.py:383-418 (linear verification, bonus token when every
    candidate matched) equals the greedy walk over the first k + 1 nodes of
    the chain tree, which the device pipeline relies on."""
    rng = random.Random(9)
    for _ in range(500):
        K = rng.randint(1, 5)
        cand = [rng.randint(0, 3) for _ in range(K)]
        remaining = rng.randint(1, 8)
        k = min(K, remaining)
        preds = [rng.randint(0, 3) for _ in range(k + 1)]
        out, all_matched = [], True  # the reference's loop
        for j in range(k):
            out.append(preds[j])
            if preds[j] != cand[j] or len(out) >= remaining:
                all_matched = False
                break
        if all_matched and len(out) < remaining:
            out.append(preds[k])
        kids = [c if i < k else [] for i, c in enumerate(medusa.chain_tree(K)["children"][: k + 1])]
        nodes, emitted = medusa.greedy_tree_walk(preds, [0] + cand[:k], kids, remaining)
        assert emitted == out and nodes == list(range(len(out))), (preds, cand, remaining)


def _sequoia():
    f = np.load(os.path.join(GOLDEN, "sequoia.npz"))
    return torch.from_numpy(f["logits"].astype(np.float32)), f["verif"].tolist(), json.loads(str(f["results"]))


def test_sequoia_tree_verifier_matches_reference():
    logits, verif, results = _sequoia()
    tree = medusa.compile_medusa_tree(medusa.DEFAULT_MEDUSA_TREE_CHOICES, 4)
    n = 0
    v = None
    for r in results:
        if r["kind"] != "tree":
            continue
        if r["max_accept"] is None:  # the generator script reuses one verifier for max_accept None, then 2
            v = medusa.SequoiaTreeVerifier(temperature=r["temp"], generator=torch.Generator().manual_seed(r["seed"]))
        acc, em, st = v.verify_tree_step(logits, tree, verif, temperature=r["temp"], max_accept=r["max_accept"])
        assert acc == r["accepted"] and em == r["emitted"], r
        assert st["tested_candidates"] == r["stats"]["tested_candidates"]
        assert st["accepted_draft_tokens"] == r["stats"]["accepted_draft_tokens"]
        assert np.allclose(st["rejection_rates_per_rank"], r["stats"]["rejection_rates_per_rank"])
        n += 1
    assert n == 36


def test_sample_without_replacement_matches_reference():
    logits, _, results = _sequoia()
    n = 0
    for r in results:
        if r["kind"] != "swr":
            continue
        gen = torch.Generator().manual_seed(r["seed"])
        got = medusa.sample_without_replacement(logits[: r["rows"]], r["k"], temperature=r["temp"],
                                                generator=gen).tolist()
        if r["temp"] <= 1e-6:  # torch.topk leaves the order of equal values open: compare values
            vals = logits[: r["rows"]]
            for row, (a, b) in enumerate(zip(got, r["indices"])):
                assert vals[row, a].tolist() == vals[row, b].tolist()
        else:
            assert got == r["indices"], r
        n += 1
    assert n == 9


def test_power_law_fit():
    rates = [0.5 * k ** -0.7 for k in range(1, 6)]
    fit = medusa.fit_power_law_rejection_bound(rates)
    assert fit["valid"] and abs(fit["exponent_b"] - 0.7) < 1e-9 and abs(fit["scale_a"] - 0.5) < 1e-9
    assert abs(fit["r_squared"] - 1.0) < 1e-9
    assert not medusa.fit_power_law_rejection_bound([0.0, 1.0, 0.3])["valid"]


def test_device_tree_rejects_bad_tables():
    tree = medusa.compile_medusa_tree(medusa.DEFAULT_MEDUSA_TREE_CHOICES, 4)
    bad = dict(tree, parent=[-1, 0, 3] + tree["parent"][3:])
    with pytest.raises(ValueError):
        medusa.DeviceTree(bad, "cpu")
    medusa.DeviceTree(tree, "cpu")  # tables only; nothing launched
