"""Prompt-lookup speculative decoding on the CUDA decoder (drop-in for
``axiomlm/engine/speculative.py:18-241``).

Draft tokens come from the sequence itself: the most recent earlier
occurrence of the last ``ngram_size`` tokens proposes the tokens that followed
it (``find_candidate_ngram``, speculative.py:18-45).  The last generated token
and the drafts are verified in one forward pass of ``1 + K`` tokens on the
GPU, as a chain (each node attends to the nodes before it: a causal block,
run by the tree-verification kernels with a chain mask).  Greedy acceptance
follows the reference (speculative.py:168-205): drafts are accepted while they
equal the model's argmax; the first mismatch contributes the model's own token
instead, and a fully matched chain adds the bonus token of its last position.
The accepted nodes are the chain's prefix, so committing them only moves the
cache's position counters (no row moves), as the reference's rollback does.
"""

from __future__ import annotations

import time
from typing import Any

import torch


def find_candidate_ngram(input_ids: list[int], ngram_size: int = 3, max_spec_tokens: int = 4) -> list[int]:
    """speculative.py:18-45: the tokens that followed the most recent earlier
    occurrence of the last ``ngram_size`` tokens (at most ``max_spec_tokens``,
    never reaching into the matched tail itself); [] when there is none."""
    n = len(input_ids)
    if n < ngram_size + 1:
        return []
    tail = input_ids[n - ngram_size:]
    limit = n - ngram_size  # drafts end before the tail being matched
    for i in range(limit - 1, -1, -1):  # newest occurrence first
        if input_ids[i:i + ngram_size] == tail:
            start = i + ngram_size
            end = min(start + max_spec_tokens, limit)
            if start < end:
                return input_ids[start:end]
    return []


def _chain(T: int) -> tuple[list[int], list[int]]:
    """Depths and ancestor masks of a T-node chain: node i sees nodes 0..i."""
    return list(range(T)), [(1 << (i + 1)) - 1 for i in range(T)]


class SpeculativePromptLookupDecoder:
    """speculative.py:48-241 on an ``axiomlm_b200.model.QuantizedDecoder``."""

    def __init__(self, ngram_size: int = 3, max_spec_tokens: int = 4):
        if max_spec_tokens + 1 > 64:
            raise ValueError("at most 63 draft tokens per verification (64-node chains)")
        self.ngram_size = ngram_size
        self.max_spec_tokens = max_spec_tokens

    @torch.no_grad()
    def generate(self, decoder, prompt_tokens: list[int], max_new_tokens: int = 64) -> tuple[list[int], dict[str, Any]]:
        """Greedy generation of ``max_new_tokens`` tokens after ``prompt_tokens``
        on a fresh decoder (batch 1).  Returns (prompt + generated tokens,
        stats) with the reference's stats keys."""
        dev = decoder.device
        cache = decoder.cache
        logits = decoder.prefill(torch.tensor([prompt_tokens], device=dev, dtype=torch.long))
        generated = list(prompt_tokens) + [int(torch.argmax(logits[0, -1]))]
        target = len(prompt_tokens) + max_new_tokens
        drafted = accepted_drafts = calls = 0
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        while len(generated) < target:
            cand = find_candidate_ngram(generated, self.ngram_size, self.max_spec_tokens)
            if not cand:
                lg = decoder.decode_step(torch.tensor([[generated[-1]]], device=dev))
                generated.append(int(torch.argmax(lg[0, -1])))
                calls += 1
                continue
            k = len(cand)
            seen0 = cache.total_seen_tokens[0]
            depths, masks = _chain(k + 1)
            lg = decoder.forward_tree_verify(torch.tensor([[generated[-1]] + cand], device=dev), depths, masks)
            calls += 1
            drafted += k
            preds = lg[0].float().argmax(-1).tolist()
            accepted = 0
            for j in range(k):
                generated.append(preds[j])
                accepted += 1
                if preds[j] != cand[j] or len(generated) >= target:
                    break
            else:
                if len(generated) < target:  # every draft matched: the bonus token
                    generated.append(preds[k])
                    accepted += 1
            accepted_drafts += max(0, accepted - 1)
            # the verified chain's first `accepted` nodes are the committed prefix
            cache.advance(seen0 + accepted)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        new = len(generated) - len(prompt_tokens)
        stats = {
            "new_tokens": new,
            "elapsed_seconds": elapsed,
            "tokens_per_second": new / elapsed if elapsed > 0 else 0.0,
            "ms_per_token": elapsed / new * 1000.0 if new > 0 else 0.0,
            "forward_calls": calls,
            "tokens_per_forward_call": new / calls if calls > 0 else 0.0,
            "drafted_tokens": drafted,
            "accepted_draft_tokens": accepted_drafts,
            "acceptance_rate_pct": accepted_drafts / drafted * 100.0 if drafted > 0 else 0.0,
        }
        return generated, stats
