"""ctypes binding of ``libaxb.so`` (the C ABI declared in ``include/axb.h``).

The library is loaded from this package directory only; there is no fallback
implementation.  Every call checks the returned status and raises
``AxbError`` (a ``RuntimeError``, like the reference's ``TORCH_CHECK``
failures) with the library's message.
"""

from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libaxb.so")

AXB_OK = 0
AXB_EINVAL = -1
AXB_ECUDA = -2
AXB_EUNSUPPORTED = -3
AXB_ETIMEOUT = -4
DEBUG_HDUMP = 1  # AXB_DEBUG_HDUMP: per-layer hidden states into runner buffer 6
DEBUG_TRACE = 2  # AXB_DEBUG_TRACE: step-kernel phase timeline into runner buffer 5

W_Q4T_SYM = 1
W_Q4T_AFFINE = 2
W_Q8_G64 = 3
W_TERNARY_G64 = 4
W_TERNARY_PT = 5
W_Q2_G64 = 6
W_Q2K_SB256 = 7

KV_F16 = 0
KV_FP8 = 1
KV_INT4 = 2
KV_TYPES = {"fp16": KV_F16, "fp8": KV_FP8, "int4": KV_INT4}

EPI_STORE = 0
EPI_RESIDUAL = 1
EPI_SWIGLU = 2
EPI_F32 = 3
EPI_F32_ACC = 4
TREE_MAX_NODES = 64
TREE_RESULT_HDR = 4
TREE_RESULT_WORDS = TREE_RESULT_HDR + 2 * TREE_MAX_NODES
TOPK_MAX = 64

TP_SUM_F32 = 0
TP_SUM_F16 = 1
TP_MAX_U64 = 2


class AxbError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"axb status {status}: {msg}")
        self.status = status


vp = C.c_void_p
i32 = C.c_int
f32 = C.c_float
sz = C.c_size_t


class QGemmDesc(C.Structure):
    _fields_ = [
        ("fmt", i32), ("group", i32), ("words", vp), ("scales", vp),
        ("N", i32), ("K", i32), ("M", i32), ("x", vp), ("ldx", i32), ("y", vp), ("ldy", i32),
        ("bias", vp), ("norm_w", vp), ("eps", f32), ("epilogue", i32), ("gate_up_interleave", i32),
        ("workspace", vp), ("workspace_bytes", sz), ("pdl", i32),
    ]


class KvWriteDesc(C.Structure):
    _fields_ = [
        ("kv_type", i32), ("kv_group", i32), ("B", i32), ("T", i32),
        ("n_head", i32), ("n_kv_head", i32), ("head_dim", i32), ("max_seq", i32), ("max_batch", i32),
        ("qkv", vp), ("bias", vp), ("rope", vp), ("rope_len", i32), ("rope_pos", i32), ("depths", vp),
        ("write_pos", i32), ("q_out", vp), ("dev_params", vp), ("k_cache", vp), ("v_cache", vp),
        ("k_scale", vp), ("v_scale", vp), ("k_is_fp32", i32),
    ]


class Q2TMeta(C.Structure):
    """axb_q2t_meta: a 2-bit projection's metadata, passed to the runner in
    place of a scale pointer."""
    _fields_ = [("meta", vp), ("meta2", vp), ("pt_scale", vp)]


class LbGemvDesc(C.Structure):
    _fields_ = [
        ("fmt", i32), ("words", vp), ("meta", vp), ("meta2", vp), ("pt_scale", vp),
        ("N", i32), ("K", i32), ("M", i32), ("x", vp), ("ldx", i32), ("y", vp), ("ldy", i32),
        ("bias", vp), ("workspace", vp), ("workspace_bytes", sz),
    ]


class AttnDesc(C.Structure):
    _fields_ = [
        ("kv_type", i32), ("kv_group", i32), ("B", i32), ("n_head", i32), ("n_kv_head", i32),
        ("head_dim", i32), ("max_seq", i32), ("max_batch", i32), ("q", vp), ("q_is_fp32", i32),
        ("k_cache", vp), ("v_cache", vp), ("k_scale", vp), ("v_scale", vp), ("out", vp),
        ("active_len", i32), ("num_splits", i32), ("T", i32), ("prefix_len", i32), ("write_pos", i32),
        ("masks", vp), ("dev_params", vp), ("workspace", vp), ("workspace_bytes", sz), ("pdl", i32),
    ]


class ModelCfg(C.Structure):
    _fields_ = [
        ("n_layer", i32), ("d_model", i32), ("n_head", i32), ("n_kv_head", i32), ("head_dim", i32),
        ("ffn", i32), ("vocab", i32), ("eps", f32), ("wfmt", i32), ("group", i32), ("lm_fmt", i32),
        ("lm_group", i32), ("kv_type", i32), ("kv_group", i32), ("max_batch", i32), ("max_seq", i32),
        ("max_tokens", i32), ("rope_len", i32), ("has_qkv_bias", i32), ("tp_world", i32), ("tp_rank", i32),
        ("dn_fmt", i32), ("dn_group", i32),
    ]


class ModelPtrs(C.Structure):
    _fields_ = [
        ("emb_w", vp), ("emb_s", vp), ("lm_w", vp), ("lm_s", vp), ("ln_f", vp), ("rope", vp),
        ("qkv_w", C.POINTER(vp)), ("qkv_s", C.POINTER(vp)), ("qkv_b", C.POINTER(vp)),
        ("o_w", C.POINTER(vp)), ("o_s", C.POINTER(vp)), ("gu_w", C.POINTER(vp)), ("gu_s", C.POINTER(vp)),
        ("dn_w", C.POINTER(vp)), ("dn_s", C.POINTER(vp)), ("ln1", C.POINTER(vp)), ("ln2", C.POINTER(vp)),
        ("k_cache", C.POINTER(vp)), ("v_cache", C.POINTER(vp)), ("k_scale", C.POINTER(vp)),
        ("v_scale", C.POINTER(vp)), ("tp_comm", vp),
    ]


# name -> (restype, argtypes); every entry point of include/axb.h
_SIGS = {
    "axb_last_error": (C.c_char_p, []),
    "axb_version": (i32, []),
    "axb_check_device": (i32, []),
    "axb_q4t_words_bytes": (sz, [i32, i32]),
    "axb_q4t_scales_bytes": (sz, [i32, i32, i32, i32]),
    "axb_q4t_pack": (i32, [vp, i32, i32, i32, i32, i32, vp, vp, vp]),
    "axb_q4t_from_marlin": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, vp]),
    "axb_q4t_dequant": (i32, [vp, vp, i32, i32, i32, i32, i32, vp, vp]),
    "axb_q4_marlin_dequant": (i32, [vp, vp, i32, i32, i32, vp, vp]),
    "axb_q8_pack": (i32, [vp, i32, i32, vp, vp, vp]),
    "axb_q8_rows": (i32, [vp, vp, vp, i32, i32, vp, vp]),
    "axb_ternary_dequant": (i32, [vp, vp, i32, i32, i32, vp, vp]),
    "axb_q2_dequant": (i32, [vp, vp, i32, i32, vp, vp]),
    "axb_q2t_words_bytes": (sz, [i32, i32]),
    "axb_q2t_meta_bytes": (sz, [i32, i32, i32]),
    "axb_q2t_meta2_bytes": (sz, [i32, i32, i32]),
    "axb_q2t_from_ref": (i32, [i32, vp, vp, vp, i32, i32, vp, vp, vp, vp]),
    "axb_q2t_dequant": (i32, [i32, vp, vp, vp, vp, i32, i32, vp, vp]),
    "axb_lbgemv_workspace_bytes": (sz, [i32, i32, i32, i32]),
    "axb_lbgemv": (i32, [C.POINTER(LbGemvDesc), vp]),
    "axb_qgemm_tc_workspace_bytes": (sz, [i32, i32, i32]),
    "axb_qgemm_tc": (i32, [C.POINTER(QGemmDesc), vp]),
    "axb_qgemm_tc_status": (i32, [vp, vp]),
    "axb_qgemm_workspace_bytes": (sz, [i32, i32, i32, i32]),
    "axb_qgemm": (i32, [C.POINTER(QGemmDesc), vp]),
    "axb_qgemm_status": (i32, [vp, vp]),
    "axb_qgemm_noalloc": (i32, [C.POINTER(QGemmDesc), vp]),
    "axb_qgemm_noalloc_scratch_bytes": (sz, []),
    "axb_qgemm_noalloc_status": (i32, [vp]),
    "axb_q8g64_gemv": (i32, [vp, i32, i32, i32, vp, vp, i32, vp, i32, vp]),
    "axb_q4t_from_q4g64": (i32, [vp, vp, i32, i32, i32, vp, vp, vp]),
    "axb_rmsnorm": (i32, [vp, vp, i32, i32, f32, vp, vp]),
    "axb_rope_kv_write": (i32, [C.POINTER(KvWriteDesc), vp]),
    "axb_kv_quantize": (i32, [vp, i32, i32, i32, i32, i32, vp, vp, vp]),
    "axb_kv_dequantize": (i32, [vp, vp, i32, i32, i32, i32, vp, vp]),
    "axb_attn_workspace_bytes": (sz, [i32, i32, i32, i32, i32, i32, i32]),
    "axb_attention": (i32, [C.POINTER(AttnDesc), vp]),
    "axb_compact_kv": (i32, [vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, i32, vp]),
    "axb_argmax": (i32, [vp, i32, i32, i32, vp, vp]),
    "axb_compact_kv_dev": (i32, [vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, vp, i32, vp]),
    "axb_tree_accept": (i32, [i32, vp, vp, vp, i32, vp, vp]),
    "axb_medusa_leaf": (i32, [vp, i32, vp, i32, vp, vp, vp]),
    "axb_medusa_silu_add": (i32, [i32, i32, vp, vp, vp, vp]),
    "axb_topk_rows": (i32, [vp, i32, i32, i32, i32, vp, vp]),
    "axb_draft_tokens": (i32, [i32, vp, vp, vp, i32, vp, vp, vp]),
    "axb_runner_workspace_bytes": (sz, [C.POINTER(ModelCfg)]),
    "axb_runner_create": (i32, [C.POINTER(ModelCfg), C.POINTER(ModelPtrs), vp, sz, C.POINTER(vp)]),
    "axb_runner_destroy": (i32, [vp]),
    "axb_runner_buffer": (i32, [vp, i32, C.POINTER(sz), C.POINTER(sz)]),
    "axb_runner_step": (i32, [vp, i32, i32, i32, i32, i32, i32, vp, vp, i32, vp]),
    "axb_runner_uses_step_kernel": (i32, [vp]),
    "axb_runner_step_launches": (i32, [vp, i32, i32, i32]),
    "axb_runner_set_debug": (i32, [vp, i32, C.c_uint32, C.c_uint32]),
    "axb_tp_unique_id": (i32, [vp]),
    "axb_tp_comm_create": (i32, [vp, i32, i32, C.POINTER(vp)]),
    "axb_tp_comm_destroy": (i32, [vp]),
    "axb_tp_comm_abort": (i32, [vp]),
    "axb_tp_allreduce": (i32, [vp, vp, sz, i32, vp]),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load libaxb.so once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python -m axiomlm_b200.build` (there is no CPU fallback)"
        )
    lib = C.CDLL(path)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(status: int, what: str = ""):
    if status != AXB_OK:
        msg = load().axb_last_error().decode(errors="replace")
        raise AxbError(status, f"{what}: {msg}" if what else msg)


def call(name: str, *args):
    fn = getattr(load(), name)
    rc = fn(*args)
    if fn.restype is i32 and name not in ("axb_version",):
        check(rc, name)
    return rc
