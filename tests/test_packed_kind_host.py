"""``packed_kind`` (the rule ``QuantizedDecoder.from_packed`` uses to tell
the reference's packings apart) on the reference's own packs
(tests/golden/quant.npz: MARLIN, legacy Q4_G64, Q8_G64, ternary, Q2 G64)."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN


@pytest.mark.parametrize("w,s,kind", [("q4m_w", "q4m_sb", "marlin"), ("q4m_clip_w", "q4m_clip_sb", "marlin"),
                                      ("q4g_w", "q4g_sb", "q4_g64"), ("q8_w", "q8_sb", "q8_g64"),
                                      ("ter_w", "ter_s", "ternary_g64"), ("q2_w", "q2_sb", "q2_g64")])
def test_packed_kind_of_reference_packs(w, s, kind):
    from axiomlm_b200.model import packed_kind

    fx = np.load(os.path.join(GOLDEN, "quant.npz"))
    assert packed_kind(torch.from_numpy(fx[w]), torch.from_numpy(fx[s])) == kind


def test_packed_kind_rejects_unknown_shapes():
    from axiomlm_b200.model import packed_kind

    with pytest.raises(NotImplementedError):
        packed_kind(torch.zeros(4, 3, dtype=torch.int32), torch.zeros(4, 1, 2, dtype=torch.float16))
