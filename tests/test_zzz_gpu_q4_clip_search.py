"""A model packed on the GPU in the reference's default "q4" mode
(``from_weights(..., "q4")``: the clip search of ``ops.q4_mse_codes`` with the
per-projection importance of ``clip_importance``, then the q4t relayout)
against the reference's own greedy decode of the same model
(tests/golden/make_golden.py --modes-only -> small_q4.npz).

The host tests pin the packer bit-exactly to the reference's packs; here it
runs on the GPU, where the same torch code sums in another order, so a group
whose best two clip candidates tie to the last fp32 bit may pick the other
one.  The check is therefore the model-level one: teacher-forced greedy
tokens and logits within rel 2e-3.  (This file sorts last so that, under
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
