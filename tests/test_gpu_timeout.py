"""A device-side wait that runs out.

Every wait of the persistent step kernel is bounded (polls of a flagged
activation word, of a split-tile piece's flags, of a copy's mbarrier).
``axb_runner_set_debug`` lowers those limits to a single poll, so waits give
up long before what they wait for can arrive: the host-side stand-in for a
word that never arrives (nothing is made to fault or hang).  The step must
then wind down by itself, waiting for its own copies in flight, report
AXB_ETIMEOUT in the error word, and leave the context usable: the same
decoder runs clean steps once the limits are restored, and a fresh decoder
on the same weights still gives the logits of a decoder that never timed out.
"""

import pytest
import torch

from model_weights import make_weights

pytestmark = pytest.mark.gpu

MID = dict(n_layer=2, d_model=1024, n_head=8, n_kv_head=2, ffn=2048, vocab=4096, eps=1e-5, theta=10000.0,
           block_size=512)


def _decoder(W):
    from axiomlm_b200.model import QuantizedDecoder

    return QuantizedDecoder.from_weights(MID, W, "q4_g128_sym", kv_dtype="fp8", kv_group=128, max_seq=256,
                                         rope_len=256)


def test_step_wait_timeout_reports_and_recovers():
    from axiomlm_b200 import _lib as L

    W = make_weights(MID, 11, ln_random=True)
    g = torch.Generator().manual_seed(12)
    prompt = torch.randint(0, MID["vocab"], (1, 24), generator=g).cuda()
    toks = torch.randint(0, MID["vocab"], (4, 1), generator=g).cuda()

    clean = _decoder(W)
    assert clean.uses_step_kernel
    clean.prefill(prompt)
    ref = [clean.decode_step(toks[i].view(1, 1)).float().clone() for i in range(2)]
    assert clean.status() == 0
    clean.close()

    dec = _decoder(W)
    dec.prefill(prompt)
    L.call("axb_runner_set_debug", dec._h, 0, 1, 1)  # one poll per wait
    dec.decode_step(toks[0].view(1, 1))
    assert dec.status() == L.AXB_ETIMEOUT
    dec.error_buf.zero_()
    L.call("axb_runner_set_debug", dec._h, 0, 0, 0)  # default limits
    for i in range(2):
        dec.decode_step(toks[2 + i].view(1, 1))
        assert dec.status() == 0, f"clean step {i} after the timeout: status {dec.status()}"
    dec.close()

    again = _decoder(W)
    again.prefill(prompt)
    out = [again.decode_step(toks[i].view(1, 1)).float() for i in range(2)]
    assert again.status() == 0
    again.close()
    for a, b in zip(out, ref):
        assert torch.equal(a, b), "a decoder built after the timeout computes different logits"
