"""Prompt-lookup drafting (speculative.py:18-45), host logic: the newest
earlier occurrence of the tail n-gram proposes the tokens after it, never
reaching into the tail itself."""

from axiomlm_b200.speculative import _chain, find_candidate_ngram


def test_find_candidate_ngram_cases():
    assert find_candidate_ngram([1, 2, 3, 4, 1, 2, 3], 3, 4) == [4]
    assert find_candidate_ngram([5, 6, 7, 8, 9, 5, 6, 7], 3, 4) == [8, 9]
    assert find_candidate_ngram([1, 2, 9, 1, 2, 8, 1, 2], 2, 4) == [8]  # the newest occurrence wins
    assert find_candidate_ngram([1, 2, 3, 4, 5, 6, 7, 8, 9, 1, 2, 3], 3, 4) == [4, 5, 6, 7]
    assert find_candidate_ngram([1, 2, 3, 4, 5, 6, 7, 8, 9, 1, 2, 3], 3, 2) == [4, 5]
    assert find_candidate_ngram([1, 2, 3], 3, 4) == []  # too short
    assert find_candidate_ngram([1, 2, 3, 4, 5, 6], 2, 4) == []  # no earlier occurrence
    assert find_candidate_ngram([7, 7, 7, 7], 2, 4) == []  # drafts may not reach into the matched tail


def test_chain_masks():
    depths, masks = _chain(4)
    assert depths == [0, 1, 2, 3]
    assert masks == [0b1, 0b11, 0b111, 0b1111]
