"""The clip-search Q4 packing (``ops.q4_mse_codes``; the reference's
pack_linear_q4_marlin with clip_search=True, quant.py:495-571) against the
reference's own packs (tests/golden/make_golden.py --mse-only ->
quant_mse.npz): codes, scales and biases bit-identical, with and without
column importance, from fp32 and fp16 weights.  Runs on the host: the search
is device-agnostic torch code (on the GPU it runs where the weights are).
"""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import axb_oracle as O


@pytest.mark.parametrize("tag,half,imp", [("f32_ln", False, "imp_ln"), ("f16_none", True, None),
                                          ("f16_sw", True, "imp_sw")])
def test_clip_search_matches_reference_packs(tag, half, imp):
    from axiomlm_b200.ops import q4_mse_codes

    fx = np.load(os.path.join(GOLDEN, "quant_mse.npz"))
    W = torch.from_numpy(fx["W"])
    if half:
        W = W.half()
    q, sc, bi = q4_mse_codes(W, None if imp is None else torch.from_numpy(fx[imp]))
    N, K = W.shape
    ref_q = O._marlin_unlayout(fx[f"{tag}_w"]).reshape(-1, K)[:N]
    sb = fx[f"{tag}_sb"]  # (tiles, K/64, 8, 2): back to (rows, K/64, 2)
    sb = sb.transpose(0, 2, 1, 3).reshape(-1, K // 64, 2)[:N]
    assert np.array_equal(q.numpy(), ref_q)
    assert np.array_equal(sc.numpy().view(np.uint16), sb[..., 0].view(np.uint16))
    assert np.array_equal(bi.numpy().view(np.uint16), sb[..., 1].view(np.uint16))


def test_clip_search_never_worse_than_round_to_nearest():
    """The search starts from the full range (factor 1), so its weighted
    error is at most that of plain min/max rounding, group by group."""
    from axiomlm_b200.ops import q4_mse_codes

    g = torch.Generator().manual_seed(3)
    W = torch.randn(16, 512, generator=g) * 0.02
    W[2, 7] = 0.3
    q, sc, bi = q4_mse_codes(W)
    wg = W.view(16, 8, 64)
    deq = q.view(16, 8, 64).float() * sc.float()[..., None] + bi.float()[..., None]
    mn, mx = wg.amin(-1, keepdim=True), wg.amax(-1, keepdim=True)
    s0 = ((mx - mn).clamp(min=1e-8) / 15.0).half().float()
    b0 = mn.half().float()
    q0 = ((wg - b0) / s0).round().clamp(0, 15)
    e_rtn = ((wg - (q0 * s0 + b0)) ** 2).sum(-1)
    e_mse = ((wg - deq) ** 2).sum(-1)
    assert bool((e_mse <= e_rtn + 1e-12).all())
    assert bool((e_mse < e_rtn).any())


def test_q4_model_packs_match_reference_quantize():
    """Every projection of a model in the reference's "q4" mode (its own
    quantize("q4") packs in small_q4.npz) from ``q4_mse_codes`` with the
    importance ``clip_importance`` picks per projection: the packing rule of
    from_weights(..., "q4"), bit-identical on the host."""
    from model_weights import SMALL, make_weights

    from axiomlm_b200.model import clip_importance
    from axiomlm_b200.ops import q4_mse_codes

    fx = np.load(os.path.join(GOLDEN, "small_q4.npz"))
    W = make_weights(SMALL, int(fx["seed"]), ln_random=bool(fx["ln_random"]))

    def check(w, imp, p, s):
        q, sc, bi = q4_mse_codes(w, imp)
        N, K = w.shape
        assert np.array_equal(q.numpy(), O._marlin_unlayout(p).reshape(-1, K)[:N])
        sb = s.transpose(0, 2, 1, 3).reshape(-1, K // 64, 2)[:N]
        assert np.array_equal(sc.numpy().view(np.uint16), sb[..., 0].view(np.uint16))
        assert np.array_equal(bi.numpy().view(np.uint16), sb[..., 1].view(np.uint16))

    for i, lw in enumerate(W["layers"]):
        gu = torch.cat([lw["w_gate"], lw["w_up"]], 0)
        for key, w, which in (("c_attn", lw["c_attn"], "qkv"), ("c_proj", lw["c_proj"], "o"), ("gu", gu, "gu"),
                              ("wd", lw["w_down"], "down")):
            check(w, clip_importance(lw, which), fx[f"pk_{key}_p_{i}"], fx[f"pk_{key}_s_{i}"])
    check(W["lm_head"], clip_importance(None, "lm", W["ln_f"]), fx["pk_lmh_p"], fx["pk_lmh_sb"])
