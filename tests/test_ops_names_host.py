"""The reference's hot-path Metal entry points (the _METAL_MOD names its
quantized decode calls) are importable from ``axiomlm_b200.ops`` under the
same names.  Training-only entry points (backward passes, cross entropy,
flash-attention training forward) and the ones fused into the runner here
(SwiGLU, add + RMSNorm, RoPE) are not standalone ops."""

import pytest

HOT_PATH = [
    "qmv_q4_marlin_mps", "qmm_q4_marlin_mps", "qmv_q4_g64_mps", "qmm_q4_g64_mps", "qmv_q8_g64_mps",
    "qmm_q8_g64_mps", "qmv_ternary_mps", "qmv_q2_k_mps", "gqa_flash_decode_mps", "gqa_flash_decode_fp8_mps",
    "gqa_flash_decode_int4_mps", "gqa_tree_verify_mps", "gqa_tree_verify_fp8_mps", "gqa_tree_verify_int4_mps",
    "rmsnorm_infer_mps", "compact_tree_kv_mps",
]


@pytest.mark.parametrize("name", HOT_PATH)
def test_ops_exports_metal_entry_point(name):
    from axiomlm_b200 import ops

    assert callable(getattr(ops, name))
