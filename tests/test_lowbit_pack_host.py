"""2-bit packers of the product (``ops.ternary_g64_codes`` and friends; they
run where the weights are) on the host: the reference formats against the
reference's own packs (tests/golden/quant.npz: pack_linear_ternary,
pack_linear_q2_k), the benchmark-only layouts against the oracle's
statement of them.  Codes and scales bit-identical."""

import os

import numpy as np
import torch

from conftest import GOLDEN
from oracle import axb_oracle as O


def _bits(t):
    return np.asarray(t).view(np.uint16) if np.asarray(t).dtype == np.float16 else np.asarray(t)


def test_ternary_and_q2_g64_match_reference_packs():
    from axiomlm_b200 import ops

    fx = np.load(os.path.join(GOLDEN, "quant.npz"))
    W = torch.from_numpy(fx["Wt"])  # the input of both reference packs
    c, s = ops.ternary_g64_codes(W)
    assert np.array_equal(c.numpy(), fx["ter_w"]) and np.array_equal(_bits(s.numpy()), _bits(fx["ter_s"]))
    c, sb = ops.q2_g64_codes(W)
    assert np.array_equal(c.numpy(), fx["q2_w"]) and np.array_equal(_bits(sb.numpy()), _bits(fx["q2_sb"]))


def test_benchmark_layouts_match_oracle():
    from axiomlm_b200 import ops

    g = torch.Generator().manual_seed(17)
    W = torch.randn(24, 512, generator=g) * 0.02
    W[3, 300] = 0.5
    W[7, :256] = -0.01
    c, s = ops.ternary_pt_codes(W)
    oc, os_ = O.ternary_pt_pack(W.numpy())
    assert np.array_equal(c.numpy(), oc) and np.array_equal(_bits(s.numpy()), _bits(os_))
    c, sub, dm = ops.q2k_sb256_codes(W)
    oc, osub, odm = O.q2k_pack(W.numpy())
    assert np.array_equal(c.numpy(), oc) and np.array_equal(sub.numpy(), osub)
    assert np.array_equal(_bits(dm.numpy()), _bits(odm))
