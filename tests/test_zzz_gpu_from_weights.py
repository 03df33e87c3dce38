"""Models packed on the GPU by ``from_weights``, against references that
pin them.  First, the reference's default "q4" mode
(``from_weights(..., "q4")``: the clip search of ``ops.q4_mse_codes`` with the
per-projection importance of ``clip_importance``, then the q4t relayout)
against the reference's own greedy decode of the same model
(tests/golden/make_golden.py --modes-only -> small_q4.npz).

The host tests pin the packer bit-exactly to the reference's packs; here it
runs on the GPU, where the same torch code sums in another order, so a group
whose best two clip candidates tie to the last fp32 bit may pick the other
one.  The check is therefore the model-level one: teacher-forced greedy
tokens and logits within rel 2e-3.  Then 2-bit models packed from fp32
weights against the oracle's forward.  (This file sorts last so that, under
``-x``, it runs after every other GPU suite.)
"""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from model_weights import SMALL, make_weights

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a = torch.as_tensor(a).float().cpu()
    b = torch.as_tensor(b).float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-6))


def test_q4_clip_search_model_matches_reference():
    from axiomlm_b200.model import QuantizedDecoder

    fx = np.load(os.path.join(GOLDEN, "small_q4.npz"))
    W = make_weights(SMALL, int(fx["seed"]), ln_random=bool(fx["ln_random"]))
    dec = QuantizedDecoder.from_weights(SMALL, W, "q4", kv_dtype="fp16", max_seq=int(fx["max_seq"]),
                                        rope_len=SMALL["block_size"])
    lg = dec.prefill(torch.as_tensor(fx["prompt"]).cuda())
    steps = [lg[0, -1].float().cpu()]
    forced = fx["tokens"]
    for i in range(len(forced) - 1):
        lg = dec.decode_step(torch.tensor([[int(forced[i])]], device="cuda"))
        steps.append(lg[0, -1].float().cpu())
    for i, s in enumerate(steps):
        assert _rel(s, fx["logits"][i]) < 2e-3, (i, _rel(s, fx["logits"][i]))
        ours, ref = int(torch.argmax(s)), int(forced[i])
        assert ours == ref or fx["margin"][i] < 2e-3, i
    dec.close()


@pytest.mark.parametrize("fmt,oracle_fmt", [("ternary", "ternary_g64"), ("q2k", "q2k")])
def test_lowbit_from_weights_matches_oracle(fmt, oracle_fmt):
    """2-bit models packed on the GPU by ``from_weights`` (the packers the
    host tests pin to the reference's packs and to the oracle's statement)
    against the oracle's forward over its own packs of the same weights."""
    from oracle import axb_oracle as O

    from axiomlm_b200.model import QuantizedDecoder

    W = make_weights(SMALL, 63, ln_random=True)
    m = O.OracleModel(SMALL, W, rope_len=SMALL["block_size"], weight_format=oracle_fmt)
    hd = SMALL["d_model"] // SMALL["n_head"]
    prompt = np.random.default_rng(64).integers(0, SMALL["vocab"], (1, 12))
    cache = O.OracleCache(SMALL["n_layer"], 1, SMALL["n_kv_head"], 128, hd, "fp16", False)
    lg, _ = m.forward(prompt, cache)
    ref = [lg[0, -1].float()]
    toks = [int(torch.argmax(ref[-1]))]
    for _ in range(7):
        lg, _ = m.forward(np.array([[toks[-1]]]), cache)
        ref.append(lg[0, -1].float())
        toks.append(int(torch.argmax(ref[-1])))
    dec = QuantizedDecoder.from_weights(SMALL, W, fmt, kv_dtype="fp16", max_seq=128, rope_len=SMALL["block_size"])
    ours = [dec.prefill(torch.as_tensor(prompt).cuda())[0, -1].float().cpu()]
    for i in range(7):
        ours.append(dec.decode_step(torch.tensor([[toks[i]]], device="cuda"))[0, -1].float().cpu())
    for i, (a, b) in enumerate(zip(ours, ref)):
        assert _rel(a, b) < 2e-3, (i, _rel(a, b))
    dec.close()
