"""Prompt-lookup speculative decoding on the GPU decoder against plain greedy
decoding of the same model: the tokens must be identical up to the first
step where greedy decoding itself is a near-tie (top-2 margin below 2e-3 of
the largest |logit|: there the chain verification and the single-token step
may round differently), and drafts must actually be accepted."""

import pytest
import torch

from model_weights import SMALL, make_weights

pytestmark = pytest.mark.gpu
TIE = 2e-3


def _decoder(W):
    from axiomlm_b200.model import QuantizedDecoder

    return QuantizedDecoder.from_weights(SMALL, W, "q4_rtn", kv_dtype="fp16", max_seq=256, rope_len=256)


@pytest.mark.parametrize("ngram,k", [(3, 4), (2, 7)])
def test_prompt_lookup_matches_greedy(ngram, k):
    from axiomlm_b200.speculative import SpeculativePromptLookupDecoder

    W = make_weights(SMALL, 41, ln_random=True)
    g = torch.Generator().manual_seed(42)
    motif = torch.randint(0, SMALL["vocab"], (12,), generator=g).tolist()
    prompt = motif * 3 + motif[:5]  # repeated text: the drafts find matches
    n_new = 48

    dec = _decoder(W)
    logits = dec.prefill(torch.tensor([prompt], device="cuda"))
    ref, margins = [], []
    for _ in range(n_new):
        row = logits[0, -1].float()
        top = row.topk(2).values
        margins.append(float(top[0] - top[1]) / float(row.abs().max()))
        ref.append(int(row.argmax()))
        logits = dec.decode_step(torch.tensor([[ref[-1]]], device="cuda"))
    dec.close()

    dec = _decoder(W)
    out, stats = SpeculativePromptLookupDecoder(ngram, k).generate(dec, prompt, n_new)
    dec.close()
    ours = out[len(prompt):]
    assert len(ours) == n_new and stats["new_tokens"] == n_new
    first_tie = next((i for i, m in enumerate(margins) if m < TIE), n_new)
    assert ours[:first_tie] == ref[:first_tie], (ours, ref, first_tie)
    assert stats["drafted_tokens"] > 0 and stats["forward_calls"] < n_new
    print(f"prompt lookup n={ngram} k={k}: identical for {first_tie} of {n_new} tokens; "
          f"{stats['forward_calls']} forward calls, {stats['accepted_draft_tokens']} of "
          f"{stats['drafted_tokens']} drafts accepted")
