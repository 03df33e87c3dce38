"""CPU restatement of AxiomLM's quantized decode path -- TEST INFRASTRUCTURE.

This module is the parity oracle.  It restates, in numpy (integer / byte work)
and torch-on-CPU (the floating-point forward, whose rounding points must match
the reference's own torch CPU path), every function on the hot path:

* weight packers / dequantizers (MARLIN-ladder Q4, Q4_G64, Q8_G64, ternary,
  affine 2-bit), ``axiomlm/kernels/quant.py``;
* FP8-e4m3fn and INT4 KV-cache quantization, ``axiomlm/kernels/quant.py``;
* RoPE tables, RMSNorm, GQA attention, ``axiomlm/models/modules.py`` and
  ``axiomlm/kernels/ops.py``;
* the quantized whole-model forward and the tree-verify forward,
  ``axiomlm/models/transformer.py``;
* the ``StaticKVCache`` write / compaction rules,
  ``axiomlm/engine/paged_cache.py``;
* Medusa tree compilation and the greedy accept walk,
  ``axiomlm/engine/medusa.py``.

It also states the layout variants the B200 build adds on top of the
reference formats (group-128 symmetric Q4 in the mma-fragment tile layout,
per-tensor ternary, K-quant-style 2-bit super-blocks, per-head FP8 KV and
group-32 INT4 KV).  Those have no reference implementation, so their parity
is *unpinned*: the oracle is the only statement of them, self-checked at the
reference granularity where one exists.

The oracle is pinned against fixtures under ``tests/golden/`` that were made
by running the reference itself (see ``tests/golden/make_golden.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import this module.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F

__all__ = [
    "marlin_lane_maps",
    "pack_q4_marlin_rtn",
    "dequant_q4_marlin",
    "dequant_q4_marlin_torch",
    "pack_q4_g64",
    "dequant_q4_g64",
    "pack_q8_g64",
    "dequant_q8_g64",
    "dequant_q8_rows",
    "pack_ternary",
    "dequant_ternary",
    "pack_q2",
    "dequant_q2",
    "fp8_e4m3fn_encode",
    "fp8_e4m3fn_decode",
    "quant_kv_fp8",
    "dequant_kv_fp8",
    "quant_kv_int4",
    "dequant_kv_int4",
    "q4t_pack",
    "q4t_dequant",
    "q4t_from_marlin",
    "ternary_pt_pack",
    "ternary_pt_dequant",
    "q2k_pack",
    "q2k_dequant",
    "quant_kv_fp8_head",
    "dequant_kv_fp8_head",
    "quant_kv_int4_g32",
    "dequant_kv_int4_g32",
    "rope_freqs",
    "rmsnorm",
    "OracleCache",
    "OracleModel",
    "compile_medusa_tree",
    "greedy_tree_accept",
    "attention_decode",
    "attention_tree",
]


def _f32(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32)


def _to_np(a) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        return a.detach().cpu().numpy()
    return np.asarray(a)


# ---------------------------------------------------------------------------
# MARLIN-ladder Q4, group 64, affine (scale, bias)
# reference: axiomlm/kernels/quant.py:447-594 (pack), :597-634 (dequant)
# ---------------------------------------------------------------------------


def marlin_lane_maps() -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Lane -> (r, c0, c1) maps of the ladder layout (quant.py:573-576)."""
    lanes = np.arange(32)
    r = ((lanes & 16) >> 2) | ((lanes & 6) >> 1)
    c0 = ((lanes & 8) >> 1) | ((lanes & 1) << 1)
    return r, c0, c0 + 1


def _rtn_affine(wg: np.ndarray, levels: float):
    """min/max round-to-nearest affine quantization of (..., G) groups.

    Matches quant.py:475-486 (Q4 MARLIN RTN), :31-43 (Q4_G64), :97-109 (Q8),
    :362-374 (2-bit) when ``wg`` is float32: ``scale = fp16((max-min)/L)``,
    ``bias = fp16(min)``, ``q = clip(rint((w - bias) / scale), 0, L)``.
    """
    wg = wg.astype(np.float32)
    w_min = wg.min(axis=-1, keepdims=True)
    w_max = wg.max(axis=-1, keepdims=True)
    denom = np.maximum(w_max - w_min, np.float32(1e-8))
    scale = (denom / np.float32(levels)).astype(np.float16)
    bias = w_min.astype(np.float16)
    q = np.clip(
        np.rint((wg - bias.astype(np.float32)) / np.maximum(scale.astype(np.float32), np.float32(1e-8))),
        0,
        levels,
    ).astype(np.int32)
    return q, scale[..., 0], bias[..., 0]


def pack_q4_marlin_rtn(w) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:447-594 with ``clip_search=False``: RTN Q4 in the ladder layout.

    Returns ``w_marlin`` int32 (ceil(N/8), K/64, 32, 2) and ``sb_marlin`` fp16
    (ceil(N/8), K/64, 8, 2).
    """
    w = _f32(_to_np(w))
    N, K = w.shape
    assert K % 64 == 0
    nt = (N + 7) // 8
    kg = K // 64
    wp = np.zeros((nt * 8, K), np.float32)
    wp[:N] = w
    q, scale, bias = _rtn_affine(wp.reshape(nt * 8, kg, 64), 15.0)
    return _marlin_layout(q, scale, bias, nt, kg)


def _marlin_layout(q, scale, bias, nt, kg):
    r, c0, c1 = marlin_lane_maps()
    # (nt, c=8, kg, word=2, s=4, r=8) -> (nt, kg, c, r, word, s)   (quant.py:578-579)
    qcr = q.reshape(nt, 8, kg, 2, 4, 8).transpose(0, 2, 1, 5, 3, 4)
    q0 = qcr[:, :, c0, r, :, :].astype(np.uint32)  # (nt, kg, 32, 2, 4)
    q1 = qcr[:, :, c1, r, :, :].astype(np.uint32)
    shifts = np.array([0, 4, 8, 12], np.uint32)
    lo = ((q0 & 0xF) << shifts).sum(-1, dtype=np.uint32)
    hi = ((q1 & 0xF) << shifts).sum(-1, dtype=np.uint32) << np.uint32(16)
    w_marlin = (lo | hi).view(np.int32)
    sb = np.stack([scale, bias], -1).reshape(nt, 8, kg, 2).transpose(0, 2, 1, 3)
    return np.ascontiguousarray(w_marlin), np.ascontiguousarray(sb.astype(np.float16))


def _marlin_unlayout(w_marlin: np.ndarray):
    """Inverse permutation of the ladder layout -> q (nt*8, kg, 64) int32."""
    w_marlin = _to_np(w_marlin)
    nt, kg = w_marlin.shape[:2]
    r, c0, c1 = marlin_lane_maps()
    wu = w_marlin.view(np.uint32)[..., None]  # (nt, kg, 32, 2, 1)
    q0 = (wu >> np.array([0, 4, 8, 12], np.uint32)) & 0xF
    q1 = (wu >> np.array([16, 20, 24, 28], np.uint32)) & 0xF
    qcr = np.empty((nt, kg, 8, 8, 2, 4), np.int32)
    qcr[:, :, c0, r] = q0
    qcr[:, :, c1, r] = q1
    # (nt, kg, c, r, word, s) -> (nt, c, kg, word, s, r)   (quant.py:623)
    return qcr.transpose(0, 2, 1, 4, 5, 3).reshape(nt * 8, kg, 64)


def dequant_q4_marlin(w_marlin, sb_marlin, K: int, out_features: int | None = None) -> np.ndarray:
    """quant.py:597-634: ``fp16(fp32(q) * fp32(scale) + fp32(bias))``."""
    q = _marlin_unlayout(w_marlin).astype(np.float32)
    sb = _to_np(sb_marlin)
    nt, kg = sb.shape[:2]
    assert kg * 64 == K
    sb = sb.transpose(0, 2, 1, 3).reshape(nt * 8, kg, 2).astype(np.float32)
    w = (q * sb[:, :, 0:1] + sb[:, :, 1:2]).reshape(nt * 8, K).astype(np.float16)
    if out_features is not None and out_features < w.shape[0]:
        w = w[:out_features]
    return w


def dequant_q4_marlin_torch(w_marlin: torch.Tensor, sb_marlin: torch.Tensor, K: int, out_features: int | None = None):
    """quant.py:597-634 with the reference's own torch ops (multi-threaded on
    the CPU); used to time the reference's per-call dequant fairly.  Equal to
    ``dequant_q4_marlin`` value for value."""
    nt, kg = w_marlin.shape[:2]
    lanes = torch.arange(32)
    r_idx = ((lanes & 16) >> 2) | ((lanes & 6) >> 1)
    c0 = ((lanes & 8) >> 1) | ((lanes & 1) << 1)
    c1 = c0 + 1
    w = w_marlin.unsqueeze(-1)
    q0 = ((w >> torch.tensor([0, 4, 8, 12], dtype=torch.int32)) & 0xF).float()
    q1 = ((w >> torch.tensor([16, 20, 24, 28], dtype=torch.int32)) & 0xF).float()
    q = torch.empty((nt, kg, 8, 8, 2, 4), dtype=torch.float32)
    q[:, :, c0, r_idx, :, :] = q0
    q[:, :, c1, r_idx, :, :] = q1
    q = q.permute(0, 2, 1, 4, 5, 3).reshape(nt * 8, kg, 64)
    sb = sb_marlin.permute(0, 2, 1, 3).reshape(nt * 8, kg, 2)
    out = (q * sb[:, :, 0:1].float() + sb[:, :, 1:2].float()).reshape(nt * 8, K).to(torch.float16)
    return out[:out_features] if out_features is not None and out_features < out.shape[0] else out


# ---------------------------------------------------------------------------
# Legacy Q4_G64 and Q8_G64 (row-major, sequential nibbles / bytes)
# reference: quant.py:17-69 (Q4_G64), :72-163 (Q8_G64, dequant_q8_rows)
# ---------------------------------------------------------------------------


def pack_q4_g64(w):
    w = _f32(_to_np(w))
    N, K = w.shape
    q, scale, bias = _rtn_affine(w.reshape(N, K // 64, 64), 15.0)
    qs = q.reshape(N, K // 8, 8).astype(np.uint32)
    packed = np.zeros((N, K // 8), np.uint32)
    for i in range(8):
        packed |= (qs[:, :, i] & 0xF) << np.uint32(4 * i)
    return packed.view(np.int32), np.stack([scale, bias], -1).astype(np.float16)


def dequant_q4_g64(w_packed, sb, K: int) -> np.ndarray:
    p = _to_np(w_packed).view(np.uint32)
    N = p.shape[0]
    q = np.stack([(p >> np.uint32(4 * i)) & 0xF for i in range(8)], -1).astype(np.float32)
    q = q.reshape(N, K // 64, 64)
    sb = _to_np(sb).astype(np.float32)
    return (q * sb[:, :, 0:1] + sb[:, :, 1:2]).reshape(N, K).astype(np.float16)


def pack_q8_g64(w):
    w = _f32(_to_np(w))
    N, K = w.shape
    q, scale, bias = _rtn_affine(w.reshape(N, K // 64, 64), 255.0)
    qs = q.reshape(N, K // 4, 4).astype(np.uint32)
    packed = np.zeros((N, K // 4), np.uint32)
    for i in range(4):
        packed |= (qs[:, :, i] & 0xFF) << np.uint32(8 * i)
    return packed.view(np.int32), np.stack([scale, bias], -1).astype(np.float16)


def dequant_q8_g64(w_packed, sb, K: int) -> np.ndarray:
    p = _to_np(w_packed).view(np.uint32)
    N = p.shape[0]
    q = np.stack([(p >> np.uint32(8 * i)) & 0xFF for i in range(4)], -1).astype(np.float32)
    q = q.reshape(N, K // 64, 64)
    sb = _to_np(sb).astype(np.float32)
    return (q * sb[:, :, 0:1] + sb[:, :, 1:2]).reshape(N, K).astype(np.float16)


def dequant_q8_rows(idx, w_packed, sb) -> np.ndarray:
    """quant.py:132-163: embedding-row gather + Q8_G64 dequant."""
    idx = _to_np(idx)
    p = _to_np(w_packed)[idx.reshape(-1)]
    s = _to_np(sb)[idx.reshape(-1)]
    K = p.shape[1] * 4
    return dequant_q8_g64(p, s, K).reshape(*idx.shape, K)


# ---------------------------------------------------------------------------
# BitNet ternary (group-64 absmean scale) and affine 2-bit ("Q2_K")
# reference: quant.py:236-295 (ternary), :339-403 (2-bit)
# ---------------------------------------------------------------------------


def pack_ternary(w):
    """quant.py:236-274.  The group absmean is a float reduction; it is taken
    with torch (the reference's own arithmetic) so the fp16 scale matches."""
    wt = torch.as_tensor(_to_np(w))
    N, K = wt.shape
    wg = wt.view(N, K // 64, 64)
    scale = wg.abs().mean(dim=-1, keepdim=True).clamp(min=1e-5).to(torch.float16)
    q = torch.clamp(torch.round(wg.float() / scale.float().clamp(min=1e-5)), -1.0, 1.0)
    q = q.numpy().astype(np.int8)
    code = np.where(q == 1, 1, np.where(q == -1, 2, 0)).astype(np.uint8).reshape(N, K // 4, 4)
    packed = code[..., 0] | (code[..., 1] << 2) | (code[..., 2] << 4) | (code[..., 3] << 6)
    return packed.astype(np.uint8), scale.squeeze(-1).numpy()


def _ternary_codes(packed: np.ndarray) -> np.ndarray:
    """quant.py:285-291: 2-bit field b -> (b & 1) - ((b >> 1) & 1)."""
    b = packed.astype(np.int32)[..., None]
    sh = np.array([0, 2, 4, 6])
    return ((b >> sh) & 1) - ((b >> (sh + 1)) & 1)


def dequant_ternary(packed, scales, K: int | None = None) -> np.ndarray:
    """quant.py:277-295: ``fp16(q * scale)`` (exact: q in {-1, 0, 1})."""
    p = _to_np(packed)
    N = p.shape[0]
    K = K or p.shape[1] * 4
    q = _ternary_codes(p).reshape(N, K // 64, 64).astype(np.float16)
    return (q * _to_np(scales)[..., None]).reshape(N, K).astype(np.float16)


def pack_q2(w):
    w = _f32(_to_np(w))
    N, K = w.shape
    q, scale, bias = _rtn_affine(w.reshape(N, K // 64, 64), 3.0)
    qs = q.reshape(N, K // 4, 4).astype(np.uint8)
    packed = (qs[..., 0] & 3) | ((qs[..., 1] & 3) << 2) | ((qs[..., 2] & 3) << 4) | ((qs[..., 3] & 3) << 6)
    return packed.astype(np.uint8), np.stack([scale, bias], -1).astype(np.float16)


def dequant_q2(packed, sb, K: int | None = None) -> np.ndarray:
    """quant.py:383-403.  The reference multiplies and adds in fp16 tensors, so
    there are two fp16 roundings: ``fp16(fp16(q * scale) + bias)``."""
    p = _to_np(packed).astype(np.int32)
    N = p.shape[0]
    K = K or p.shape[1] * 4
    q = np.stack([(p >> s) & 3 for s in (0, 2, 4, 6)], -1).reshape(N, K // 64, 64).astype(np.float16)
    sb = _to_np(sb)
    t = (q.astype(np.float32) * sb[..., 0:1].astype(np.float32)).astype(np.float16)
    return (t.astype(np.float32) + sb[..., 1:2].astype(np.float32)).astype(np.float16).reshape(N, K)


# ---------------------------------------------------------------------------
# FP8 e4m3fn bit conversion (torch's c10 Float8_e4m3fn rules, restated)
# ---------------------------------------------------------------------------


def fp8_e4m3fn_encode(x) -> np.ndarray:
    """float32 -> e4m3fn byte, round-half-even, |x| >= 480 or NaN -> NaN (0x7F|sign).

    This is the conversion ``Tensor.to(torch.float8_e4m3fn)`` performs (used at
    quant.py:720); the tests pin it against torch on every fp16 value.
    """
    x = _f32(x)
    bits = x.view(np.uint32)
    sign = ((bits >> 24) & 0x80).astype(np.uint8)
    a = np.abs(x).astype(np.float64)
    out = np.zeros(x.shape, np.uint8)
    nan = ~np.isfinite(x) | (a >= 480.0)
    # normal range of e4m3: exponent e in [-6, 8], 3 mantissa bits
    with np.errstate(divide="ignore", invalid="ignore"):
        e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.clip(e, -6, 8)
    step = np.exp2(e - 3)  # quantum at this exponent (subnormals use 2^-9)
    m = a / step
    r = np.rint(m)  # half-even
    val = r * step  # rounded magnitude
    # re-derive exponent after rounding (may carry into the next binade)
    code = np.zeros(x.shape, np.int64)
    sub = val < 2.0 ** -6
    code_sub = np.rint(val / 2.0 ** -9).astype(np.int64)  # 0..8 (8 == min normal)
    with np.errstate(divide="ignore", invalid="ignore"):
        en = np.floor(np.log2(np.where(val > 0, val, 1.0)))
    mant = np.rint(val / np.exp2(en - 3)).astype(np.int64) - 8
    code_norm = ((en.astype(np.int64) + 7) << 3) | mant
    code = np.where(sub, code_sub, code_norm)
    code = np.where(nan, 0x7F, code)
    out = (code.astype(np.uint8) & 0x7F) | sign
    return out


_E4M3_TABLE = None


def fp8_e4m3fn_decode(b) -> np.ndarray:
    """e4m3fn byte -> float32 (exact)."""
    global _E4M3_TABLE
    if _E4M3_TABLE is None:
        t = np.zeros(256, np.float32)
        for c in range(256):
            s = -1.0 if c & 0x80 else 1.0
            e = (c >> 3) & 0xF
            m = c & 7
            if e == 15 and m == 7:
                t[c] = np.nan
            elif e == 0:
                t[c] = s * m * 2.0 ** -9
            else:
                t[c] = s * (1 + m / 8.0) * 2.0 ** (e - 7)
        _E4M3_TABLE = t
    return _E4M3_TABLE[_to_np(b).astype(np.uint8)]


# ---------------------------------------------------------------------------
# KV-cache quantization, reference granularity (64-element groups)
# reference: quant.py:692-724 (fp8 quant), :727-768 (fp8 dequant),
#            :771-807 (int4 quant), :810-852 (int4 dequant)
# ---------------------------------------------------------------------------


def _group_amax(x16: np.ndarray, G: int) -> np.ndarray:
    xg = x16.reshape(*x16.shape[:-1], -1, G)
    return np.abs(xg).max(-1), xg


def _kv_scale_and_ratio(xg: np.ndarray, qmax: float):
    """Shared rule of quant.py:709-719 / :788-797 for one dtype.

    fp16 input: ``amax`` is fp16, ``amax / qmax`` is rounded to fp16 (the
    clamp at 1e-8 then is a no-op in fp16) and ``x / scale`` is an fp16
    division.  fp32 input (the model path: K after RoPE stays fp32):
    ``scale = fp16(max(amax / qmax, 1e-8))`` and ``x / scale`` is an fp32
    division with no fp16 rounding.
    """
    if xg.dtype == np.float16:
        amax = np.abs(xg).max(-1)
        scale = (amax.astype(np.float32) / np.float32(qmax)).astype(np.float16)
        with np.errstate(divide="ignore", invalid="ignore"):
            r = (xg.astype(np.float32) / scale[..., None].astype(np.float32)).astype(np.float16).astype(np.float32)
    else:
        xg = xg.astype(np.float32)
        amax = np.abs(xg).max(-1)
        scale = np.maximum(amax / np.float32(qmax), np.float32(1e-8)).astype(np.float16)
        with np.errstate(divide="ignore", invalid="ignore"):
            r = xg / scale[..., None].astype(np.float32)
    return scale, r


def _as_kv_input(x) -> np.ndarray:
    a = _to_np(x)
    return a if a.dtype in (np.float16, np.float32) else a.astype(np.float32)


def quant_kv_fp8(x, group: int = 64) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:692-724: ``q = e4m3fn(x / scale)`` with ``scale = amax/448``
    (rounding points per ``_kv_scale_and_ratio``).  ``group`` = 64 is the
    reference; ``group`` = head_dim is the per-(token, head) benchmark variant."""
    a = _as_kv_input(x)
    xg = a.reshape(*a.shape[:-1], -1, group)
    scale, r = _kv_scale_and_ratio(xg, 448.0)
    q = fp8_e4m3fn_encode(r).reshape(a.shape)
    return q, scale


def dequant_kv_fp8(q, scales, group: int = 64) -> np.ndarray:
    """quant.py:727-768: ``fp16(e4m3 -> fp16) * fp16 scale`` rounded to fp16."""
    q = _to_np(q)
    s = _to_np(scales).astype(np.float32)
    v = fp8_e4m3fn_decode(q).astype(np.float16).astype(np.float32)
    vg = v.reshape(*q.shape[:-1], -1, group)
    return (vg * s[..., None]).astype(np.float16).reshape(q.shape)


def quant_kv_int4(x, group: int = 64) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:771-807: ``q = clip(rint(x / scale), -8, 7)``, ``scale =
    amax/7``, low nibble = even element.  A zero scale gives the reference's
    x/0 path: +inf -> 7, -inf -> -8, NaN -> 0.  ``group`` = 32 is the
    long-context benchmark's variant."""
    a = _as_kv_input(x)
    hd = a.shape[-1]
    xg = a.reshape(*a.shape[:-1], -1, group)
    scale, r = _kv_scale_and_ratio(xg, 7.0)
    q = np.clip(np.rint(r), -8, 7)
    q = np.where(np.isnan(q), 0, q).astype(np.int8)
    qp = q.reshape(*a.shape[:-1], hd // 2, 2).astype(np.uint8)
    packed = (qp[..., 0] & 0xF) | ((qp[..., 1] & 0xF) << 4)
    return packed.astype(np.uint8), scale


def dequant_kv_int4(q, scales, group: int = 64) -> np.ndarray:
    """quant.py:810-852: ``(((n ^ 8) - 8) as fp16) * fp16 scale`` rounded to fp16."""
    q = _to_np(q).astype(np.int32)
    s = _to_np(scales).astype(np.float32)
    lo = ((q & 0xF) ^ 8) - 8
    hi = (((q >> 4) & 0xF) ^ 8) - 8
    v = np.stack([lo, hi], -1).reshape(*q.shape[:-1], -1).astype(np.float32)
    vg = v.reshape(*q.shape[:-1], -1, group)
    return (vg * s[..., None]).astype(np.float16).reshape(*q.shape[:-1], q.shape[-1] * 2)


# ---------------------------------------------------------------------------
# B200 layout variants (no reference implementation: parity unpinned)
# ---------------------------------------------------------------------------
#
# Q4 tile layout ("q4t"): rows in 16-row tiles, K in 64-wide blocks.  Block
# (tile t, k-block b) is 512 bytes: 32 lanes x 4 words.  Lane l = 4*g + j4
# (g = l >> 2 is the mma groupID, j4 = l & 3 the thread-in-group) holds, in
# word j (j = 0..3), the eight weights of rows {g, g+8} at the four columns
# k = 64*b + 16*j4 + 4*j + {0,1,2,3}:
#     fragment register a0 = (row g,   k+0, k+1)   a1 = (row g+8, k+0, k+1)
#                       a2 = (row g,   k+2, k+3)   a3 = (row g+8, k+2, k+3)
# Nibble i (i = 0..3) holds the low half of register a_i and nibble i+4 its
# high half; listing a register's halves high-first this is the 64207531
# interleave (high 16 bits: elements 6,4,2,0; low 16 bits: 7,5,3,1), so one
# lop3 with mask 0x000F000F per 4-bit shift yields an mma A-fragment half2.
# Scales: fp16, (tiles, K/G, 16) for the symmetric form ``w = (q - 8) * s``,
# (tiles, K/G, 16, 2) = (scale, bias) pairs for the affine form.


def _q4t_word_coords():
    """(lane, word, nibble) -> (row-in-tile, k-in-block)."""
    rows = np.zeros((32, 4, 8), np.int32)
    ks = np.zeros((32, 4, 8), np.int32)
    for lane in range(32):
        g, j4 = lane >> 2, lane & 3
        for j in range(4):
            kb = 16 * j4 + 4 * j
            # register index i: (row, k offset)
            regs = [(g, 0), (g + 8, 0), (g, 2), (g + 8, 2)]
            for i, (rr, ko) in enumerate(regs):
                rows[lane, j, i] = rr
                ks[lane, j, i] = kb + ko  # low half = even k
                rows[lane, j, i + 4] = rr
                ks[lane, j, i + 4] = kb + ko + 1  # high half = odd k
    return rows, ks


_Q4T_ROWS, _Q4T_KS = _q4t_word_coords()


_Q4T_FLAT = (_Q4T_ROWS * 64 + _Q4T_KS).reshape(-1)  # (32*4*8,) offsets into a 16 x 64 block


def _q4t_pack_codes(q: np.ndarray) -> np.ndarray:
    """q (Npad, K) int codes 0..15 -> words uint32 (tiles, K/64, 32, 4).
    Processed in tile chunks: (tile, k-block) blocks made contiguous, the
    fragment positions gathered by one flat index, 8 nibbles per word."""
    npad, K = q.shape
    nt, kb = npad // 16, K // 64
    out = np.empty((nt, kb, 32, 4), np.uint32)
    step = max(1, (1 << 22) // (16 * K))  # about 4M codes per chunk
    sh = (np.arange(8, dtype=np.uint32) * 4)
    for t0 in range(0, nt, step):
        t1 = min(nt, t0 + step)
        qb = np.ascontiguousarray(q[t0 * 16:t1 * 16].astype(np.uint8).reshape(t1 - t0, 16, kb, 64)
                                  .transpose(0, 2, 1, 3)).reshape(t1 - t0, kb, 1024)
        vals = np.take(qb, _Q4T_FLAT, axis=2).reshape(t1 - t0, kb, 32, 4, 8).astype(np.uint32)
        out[t0:t1] = ((vals & 0xF) << sh).sum(-1, dtype=np.uint32)
    return out


def _q4t_unpack_codes(words: np.ndarray) -> np.ndarray:
    words = _to_np(words).view(np.uint32)
    nt, kb = words.shape[:2]
    vals = (words[..., None] >> (np.arange(8, dtype=np.uint32) * 4)) & 0xF  # (nt,kb,32,4,8)
    qb = np.zeros((nt, kb, 16, 64), np.int32)
    qb[:, :, _Q4T_ROWS, _Q4T_KS] = vals
    return qb.transpose(0, 2, 1, 3).reshape(nt * 16, kb * 64)


def _gu_rows(npad: int, N: int, gu: bool) -> np.ndarray:
    """packed row -> source row (N = padding) for the gate/up interleave:
    tile t holds gate rows 8t..8t+7 then up rows F+8t..F+8t+7."""
    p = np.arange(npad)
    if not gu:
        return np.where(p < N, p, N)
    F = N // 2
    j = (p >> 4) * 8 + (p & 7)
    src = np.where((p >> 3) & 1, F + j, j)
    return np.where(j < F, src, N)


def q4t_pack(w, group: int = 128, symmetric: bool = True, gate_up: bool = False):
    """Quantize (N, K) fp32 weights into the q4t layout (RTN).

    symmetric: ``s = fp16(max(absmax, 1e-8) / 7)``, ``q = clip(rint(w / s),
    -8, 7) + 8`` (q = 8 where s rounds to 0); dequant ``fp16((q - 8) * s)``.
    affine: the reference's RTN min/max rule (quant.py:475-486) at ``group``.
    Scales: symmetric (tiles, K/G, 8, 2) = (s[g], s[g+8]); affine
    (tiles, K/G, 8, 4) = (s[g], b[g], s[g+8], b[g+8]).
    """
    w = _f32(_to_np(w))
    N, K = w.shape
    assert K % 64 == 0 and K % group == 0
    nt = (N + 15) // 16
    src = _gu_rows(nt * 16, N, gate_up)
    words = np.empty((nt, K // 64, 32, 4), np.uint32)
    sc = np.empty((nt, K // group, 8, 2 if symmetric else 4), np.float16)
    step = max(1, (1 << 22) // (16 * K))  # tiles per chunk: about 4M weights (rows are independent)
    zero = np.zeros((1, K), np.float32)
    for t0 in range(0, nt, step):
        t1 = min(nt, t0 + step)
        rows = src[t0 * 16:t1 * 16]
        wp = np.where((rows < N)[:, None], w[np.minimum(rows, N - 1)], zero)
        wg = wp.reshape((t1 - t0) * 16, K // group, group)
        if symmetric:
            amax = np.abs(wg).max(-1)
            s16 = (np.maximum(amax, np.float32(1e-8)) / np.float32(7.0)).astype(np.float16)
            sf = s16[..., None].astype(np.float32)
            with np.errstate(divide="ignore", invalid="ignore"):
                q = np.clip(np.rint(wg / sf), -8, 7)
            q = np.where(sf == 0, 0, q).astype(np.int32) + 8
            sc[t0:t1] = s16.reshape(t1 - t0, 2, 8, K // group).transpose(0, 3, 2, 1)  # (nt, grp, 8, [g, g+8])
        else:
            q, s16, b16 = _rtn_affine(wg, 15.0)
            sb = np.stack([s16, b16], -1).reshape(t1 - t0, 2, 8, K // group, 2)  # (nt, h, g, grp, 2)
            sc[t0:t1] = sb.transpose(0, 3, 2, 1, 4).reshape(t1 - t0, K // group, 8, 4)
        words[t0:t1] = _q4t_pack_codes(q.reshape((t1 - t0) * 16, K))
    return words.view(np.int32), sc


def q4t_dequant(words, scales, K: int, group: int, symmetric: bool, out_features: int | None = None,
                gate_up: bool = False):
    """Inverse of ``q4t_pack``: fp16 (N, K) in the source row order."""
    q = _q4t_unpack_codes(words).astype(np.float32)
    npad = q.shape[0]
    nt = npad // 16
    s = _to_np(scales).astype(np.float32)
    qg = q.reshape(npad, K // group, group)
    if symmetric:
        sc = s.transpose(0, 3, 2, 1).reshape(npad, K // group)  # (nt, h, g, grp)
        w = ((qg - 8.0) * sc[..., None]).astype(np.float16).reshape(npad, K)
    else:
        sb = s.reshape(nt, K // group, 8, 2, 2).transpose(0, 3, 2, 1, 4).reshape(npad, K // group, 2)
        w = (qg * sb[..., 0:1] + sb[..., 1:2]).astype(np.float16).reshape(npad, K)
    N = out_features if out_features is not None else npad
    src = _gu_rows(npad, N, gate_up)
    out = np.zeros((N, K), np.float16)
    ok = src < N
    out[src[ok]] = w[ok]
    return out


def q4t_from_marlin(w_marlin, sb_marlin, n_out: int | None = None, gate_up: bool = False):
    """Relayout reference ladder Q4 (G64 affine) into q4t affine G64.

    Bit-exact on values: the same codes, scales and biases, only moved."""
    q = _marlin_unlayout(w_marlin)  # (nt8*8, kg, 64)
    sb = _to_np(sb_marlin)
    nt8, kg = sb.shape[:2]
    n8 = nt8 * 8
    sbr = sb.transpose(0, 2, 1, 3).reshape(n8, kg, 2)
    N = n_out if n_out is not None else n8
    nt = (N + 15) // 16
    src = _gu_rows(nt * 16, N, gate_up)
    qz = np.concatenate([q.reshape(n8, kg * 64)[:N], np.zeros((1, kg * 64), np.int32)], 0)
    sz = np.concatenate([sbr[:N], np.zeros((1, kg, 2), np.float16)], 0)
    qq = qz[np.minimum(src, N)]
    ss = sz[np.minimum(src, N)]
    words = _q4t_pack_codes(qq)
    sc = ss.reshape(nt, 2, 8, kg, 2).transpose(0, 3, 2, 1, 4).reshape(nt, kg, 8, 4)
    return words.view(np.int32), np.ascontiguousarray(sc)


def ternary_pt_pack(w):
    """BitNet b1.58 with one per-tensor absmean fp16 scale (the format of the GEMV sweep's ternary case).

    Same 2-bit codes and byte order as the reference (quant.py:264-274);
    ``scale = fp16(max(mean|w|, 1e-5))`` over the whole matrix (float64 sum).
    """
    w = _f32(_to_np(w))
    N, K = w.shape
    s = np.float16(max(float(np.abs(w.astype(np.float64)).mean()), 1e-5))
    q = np.clip(np.rint(w / np.float32(s)), -1, 1).astype(np.int8)
    code = np.where(q == 1, 1, np.where(q == -1, 2, 0)).astype(np.uint8).reshape(N, K // 4, 4)
    packed = code[..., 0] | (code[..., 1] << 2) | (code[..., 2] << 4) | (code[..., 3] << 6)
    return packed.astype(np.uint8), np.array([s], np.float16)


def ternary_pt_dequant(packed, scale) -> np.ndarray:
    p = _to_np(packed)
    N = p.shape[0]
    q = _ternary_codes(p).reshape(N, -1).astype(np.float32)
    return (q * np.float32(_to_np(scale).reshape(-1)[0])).astype(np.float16)


def q2k_pack(w):
    """K-quant-style 2-bit super-blocks (the long-context low-bit format; no reference implementation).

    Per 256-element super-block: fp16 ``d`` (scale of sub-scales) and fp16
    ``dmin`` (scale of sub-mins); per 16-element sub-block a 4-bit sub-scale
    ``sc`` and 4-bit sub-min ``mn``; weight ``w = d*sc*q - dmin*mn`` with
    ``q`` in 0..3.  Bytes per super-block: 64 (codes, 4 per byte, element i
    of the block at byte i//4, bits 2*(i%4)) + 16 (sub-scale | sub-min << 4)
    + 4 (d, dmin) = 84 -> 2.625 bits/weight.
    Layout: codes (N, K/4) uint8, sub (N, K/16) uint8, dm (N, K/256, 2) fp16.
    """
    w = _f32(_to_np(w))
    N, K = w.shape
    assert K % 256 == 0
    sb = w.reshape(N, K // 256, 16, 16)
    mn = np.minimum(sb.min(-1), 0.0)  # (N, SB, 16) <= 0
    mx = sb.max(-1)
    sub_scale = np.maximum(mx - mn, 1e-8) / 3.0
    sub_min = -mn
    d = (sub_scale.max(-1) / 15.0).astype(np.float16)
    dmin = (sub_min.max(-1) / 15.0).astype(np.float16)
    df = np.maximum(d.astype(np.float32), 1e-8)[..., None]
    mf = np.maximum(dmin.astype(np.float32), 1e-8)[..., None]
    sc = np.clip(np.rint(sub_scale / df), 0, 15).astype(np.int32)
    mi = np.clip(np.rint(sub_min / mf), 0, 15).astype(np.int32)
    eff_s = d.astype(np.float32)[..., None] * sc
    eff_m = dmin.astype(np.float32)[..., None] * mi
    q = np.clip(np.rint((sb + eff_m[..., None]) / np.maximum(eff_s, 1e-12)[..., None]), 0, 3).astype(np.uint8)
    q = q.reshape(N, K // 4, 4)
    codes = q[..., 0] | (q[..., 1] << 2) | (q[..., 2] << 4) | (q[..., 3] << 6)
    sub = (sc | (mi << 4)).astype(np.uint8).reshape(N, K // 16)
    dm = np.stack([d, dmin], -1).astype(np.float16)
    return codes.astype(np.uint8), sub, dm


def q2k_dequant(codes, sub, dm) -> np.ndarray:
    """``fp16(fp32(d)*sc*q - fp32(dmin)*mn)`` evaluated in fp32."""
    c = _to_np(codes).astype(np.int32)
    N = c.shape[0]
    K = c.shape[1] * 4
    q = np.stack([(c >> s) & 3 for s in (0, 2, 4, 6)], -1).reshape(N, K // 16, 16).astype(np.float32)
    sb = _to_np(sub).astype(np.int32)
    sc = (sb & 15).astype(np.float32)
    mi = (sb >> 4).astype(np.float32)
    dmv = _to_np(dm).astype(np.float32)
    d = np.repeat(dmv[..., 0], 16, axis=-1)
    dmin = np.repeat(dmv[..., 1], 16, axis=-1)
    a = d * sc
    b = dmin * mi
    return (q * a[..., None] - b[..., None]).astype(np.float16).reshape(N, K)


def quant_kv_fp8_head(x):
    """FP8 KV with one fp16 scale per (token, head) (the 8B decode benchmark's cache format): the
    reference rule at group size = head_dim."""
    a = _as_kv_input(x)
    q, s = quant_kv_fp8(a, group=a.shape[-1])
    return q, s[..., 0]


def dequant_kv_fp8_head(q, scale):
    q = _to_np(q)
    return dequant_kv_fp8(q, _to_np(scale)[..., None], group=q.shape[-1])


def quant_kv_int4_g32(x):
    """INT4 KV with 32-element groups (the long-context low-bit configuration's format)."""
    return quant_kv_int4(x, group=32)


def dequant_kv_int4_g32(q, scales):
    return dequant_kv_int4(q, scales, group=32)


# ---------------------------------------------------------------------------
# RoPE table and RMSNorm (modules.py:30-92); same torch ops, same order
# ---------------------------------------------------------------------------


def rope_freqs(head_dim: int, max_seq_len: int, theta: float = 10000.0, rope_scaling: dict | None = None) -> torch.Tensor:
    """modules.py:46-92: complex64 (max_seq_len, head_dim/2)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    if rope_scaling is not None:
        rtype = rope_scaling.get("rope_type", rope_scaling.get("type", "default"))
        if rtype == "llama3":
            factor = float(rope_scaling["factor"])
            lo_f = float(rope_scaling.get("low_freq_factor", 1.0))
            hi_f = float(rope_scaling.get("high_freq_factor", 4.0))
            old = float(rope_scaling.get("original_max_position_embeddings", 8192))
            lo_wl = old / lo_f
            hi_wl = old / hi_f
            wavelen = 2.0 * math.pi / inv_freq
            inv_l = torch.where(wavelen > lo_wl, inv_freq / factor, inv_freq)
            smooth = (old / wavelen - lo_f) / (hi_f - lo_f)
            smoothed = (1.0 - smooth) * inv_l / factor + smooth * inv_l
            medium = ~(wavelen < hi_wl) & ~(wavelen > lo_wl)
            inv_freq = torch.where(medium, smoothed, inv_l)
        elif rtype == "linear" and "factor" in rope_scaling:
            inv_freq = inv_freq / float(rope_scaling["factor"])
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return torch.polar(torch.ones_like(freqs), freqs)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """modules.py:41-43 evaluated in the dtype of ``w`` (x is cast first,
    transformer.py:1102)."""
    x = x.to(w.dtype)
    rms = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return x * rms * w


def _rope_apply(x: torch.Tensor, f: torch.Tensor) -> torch.Tensor:
    """transformer.py:1112-1127: complex multiply in fp32, cast back."""
    B, H, T, hd = x.shape
    xc = torch.view_as_complex(x.float().reshape(B, H, T, -1, 2))
    return torch.view_as_real(xc * f).reshape(B, H, T, hd).to(x.dtype)


# ---------------------------------------------------------------------------
# Attention (ops.py:552-654 decode, :657-797 tree) on dequantized K/V
# ---------------------------------------------------------------------------


def _repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1:
        return x
    B, H, T, D = x.shape
    return x[:, :, None].expand(B, H, n_rep, T, D).reshape(B, H * n_rep, T, D)


def attention_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, active_len: int) -> torch.Tensor:
    """q (B, Hq, 1, hd) fp16; k/v (B, Hkv, S, hd) fp16 (dequantized) -> (B, Hq, 1, hd)."""
    n_rep = q.size(1) // k.size(1)
    ka = _repeat_kv(k[:, :, :active_len], n_rep).to(q.dtype)
    va = _repeat_kv(v[:, :, :active_len], n_rep).to(q.dtype)
    return F.scaled_dot_product_attention(q, ka, va)


def attention_tree(q, k, v, masks: list[int], prefix_len: int, write_pos: int) -> torch.Tensor:
    """q (B, Hq, T, hd); node u sees slots [0, prefix_len) and tree slot
    write_pos + j iff bit j of masks[u] is set (ops.py:770-794)."""
    T = len(masks)
    n_rep = q.size(1) // k.size(1)
    ka = torch.cat([k[:, :, :prefix_len], k[:, :, write_pos:write_pos + T]], 2)
    va = torch.cat([v[:, :, :prefix_len], v[:, :, write_pos:write_pos + T]], 2)
    mask = torch.zeros((1, 1, T, prefix_len + T), dtype=torch.bool)
    mask[..., :prefix_len] = True
    for u in range(T):
        for j in range(T):
            if (int(masks[u]) >> j) & 1:
                mask[0, 0, u, prefix_len + j] = True
    ka, va = ka.to(q.dtype), va.to(q.dtype)  # transformer.py:734-735
    return F.scaled_dot_product_attention(q, _repeat_kv(ka, n_rep), _repeat_kv(va, n_rep), attn_mask=mask)


# ---------------------------------------------------------------------------
# StaticKVCache rules (paged_cache.py:122-462)
# ---------------------------------------------------------------------------


@dataclass
class OracleCache:
    """numpy stand-in for ``StaticKVCache`` (paged_cache.py:122-215)."""

    n_layer: int
    max_batch: int
    n_kv_head: int
    max_seq: int
    head_dim: int
    cache_dtype: str = "fp16"  # fp16 | fp8 | int4
    ring_buffer: bool = False
    kv_group: int = 64  # 64: the reference; head_dim: one FP8 scale per (token, head); 32: INT4 G32
    seen: int = 0
    k: list = field(default_factory=list)
    v: list = field(default_factory=list)
    ks: list = field(default_factory=list)
    vs: list = field(default_factory=list)
    # Test hook for quantized caches: {layer: (k codes, v codes, k scales,
    # v scales)}, each (B, H, T, .), stored by write() in place of what it
    # computed; what it computed goes to ``written`` for comparison.
    pinned: dict | None = None
    written: dict = field(default_factory=dict)

    def __post_init__(self):
        L, B, H, S, D = self.n_layer, self.max_batch, self.n_kv_head, self.max_seq, self.head_dim
        G = max(1, D // self.kv_group)
        for _ in range(L):
            if self.cache_dtype == "fp16":
                self.k.append(np.zeros((B, H, S, D), np.float16))
                self.v.append(np.zeros((B, H, S, D), np.float16))
            else:
                w = D if self.cache_dtype == "fp8" else D // 2
                self.k.append(np.zeros((B, H, S, w), np.uint8))
                self.v.append(np.zeros((B, H, S, w), np.uint8))
                self.ks.append(np.zeros((B, H, S, G), np.float16))
                self.vs.append(np.zeros((B, H, S, G), np.float16))

    def slots(self, T: int) -> list[int]:
        """Slots the next T tokens go to (paged_cache.py:250-331)."""
        s, S = self.seen, self.max_seq
        if not self.ring_buffer and s + T <= S:
            return list(range(s, s + T))
        return [(s + i) % S for i in range(T)][-S:] if T < S else list(range(S))

    def write(self, layer: int, k16: np.ndarray, v16: np.ndarray, slots: list[int]):
        """k16/v16: (B, H, T, D) fp16."""
        B = k16.shape[0]
        if k16.shape[2] > len(slots):  # T >= max_seq: keep the last S tokens (paged_cache.py:291-296)
            k16, v16 = k16[:, :, -len(slots):], v16[:, :, -len(slots):]
        if self.cache_dtype == "fp16":
            self.k[layer][:B, :, slots] = k16
            self.v[layer][:B, :, slots] = v16
            return
        qf = quant_kv_fp8 if self.cache_dtype == "fp8" else quant_kv_int4
        kq, ks = qf(k16, self.kv_group)
        vq, vs = qf(v16, self.kv_group)
        if self.pinned is not None and layer in self.pinned:
            self.written[layer] = (kq, vq, ks, vs)
            kq, vq, ks, vs = self.pinned[layer]
        self.k[layer][:B, :, slots] = kq
        self.v[layer][:B, :, slots] = vq
        self.ks[layer][:B, :, slots] = ks
        self.vs[layer][:B, :, slots] = vs

    def dequant(self, layer: int, B: int, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Dequantized K/V for slots [0, n) (paged_cache.py:266-288)."""
        if self.cache_dtype == "fp16":
            k, v = self.k[layer][:B, :, :n], self.v[layer][:B, :, :n]
        elif self.cache_dtype == "fp8":
            k = dequant_kv_fp8(self.k[layer][:B, :, :n], self.ks[layer][:B, :, :n], self.kv_group)
            v = dequant_kv_fp8(self.v[layer][:B, :, :n], self.vs[layer][:B, :, :n], self.kv_group)
        else:
            k = dequant_kv_int4(self.k[layer][:B, :, :n], self.ks[layer][:B, :, :n], self.kv_group)
            v = dequant_kv_int4(self.v[layer][:B, :, :n], self.vs[layer][:B, :, :n], self.kv_group)
        return torch.from_numpy(np.ascontiguousarray(k)), torch.from_numpy(np.ascontiguousarray(v))

    def compact(self, write_pos: int, accepted: list[int], new_seen: int):
        """paged_cache.py:376-462: move accepted tree slots to a contiguous run."""
        S = self.max_seq
        src = [(write_pos + int(a)) % S for a in accepted]
        dst = [(write_pos + m) % S for m in range(len(accepted))]
        for arrs in (self.k, self.v, self.ks, self.vs):
            for a in arrs:
                staged = a[:, :, src].copy()
                a[:, :, dst] = staged
        self.seen = new_seen


# ---------------------------------------------------------------------------
# Quantized model forward (transformer.py:1036-1200) and tree verify
# (transformer.py:639-784), over weights packed by the oracle packers
# ---------------------------------------------------------------------------


class OracleModel:
    """The reference's quantized forward, over fp32 master weights.

    ``weights``: dict with ``wte`` (V, d), ``lm_head`` (V, d) or None (tied),
    ``ln_f`` (d,), and ``layers``: list of dicts ``c_attn`` (q+2kv, d),
    ``c_proj`` (d, q), ``w_gate``/``w_up`` (F, d), ``w_down`` (d, F),
    ``ln_1``/``ln_2`` (d,).  Packing follows ``_ensure_quant_weights``
    (transformer.py:822-1008) in ``q4_rtn`` mode: MARLIN Q4 RTN for the
    projections and lm_head (Q8_G64 when tied), Q8_G64 token embeddings.
    RMSNorm weights stay fp32 (the reference model's parameter dtype), so the
    norms are evaluated in fp32 and cast to fp16 by ``_qlin``.

    ``weight_format="q4_g128_sym"`` is the benchmark variant (parity
    unpinned): the projections and an untied lm_head are quantized by
    ``q4t_pack`` (symmetric, group 128, fp16 scales) and dequantized by
    ``q4t_dequant``; everything else -- embeddings, norms, the forward -- is the
    reference's ``q4_rtn`` path unchanged.

    2-bit models: ``"ternary_g64"`` and ``"q2_g64"`` pack projections and an
    untied lm_head with the reference's ``pack_linear_ternary`` /
    ``pack_linear_q2_k`` (its ``quantize("ternary" | "q2_k")``,
    transformer.py:857-862); ``"ternary_pt"`` and ``"q2k"`` use the
    benchmark-only layouts (parity unpinned, as above).

    The reference's other quantized-forward modes (transformer.py:840-858):
    ``"q8"`` packs every projection and the lm_head Q8_G64; ``"q4_k_m"`` takes
    the MSE-clipped MARLIN packs of c_attn, c_proj and gate_up as the
    reference made them (``packs``: {"c_attn"|"c_proj"|"gu": [(p, s) per
    layer]}, no clip search is restated here) with Q8_G64 w_down and lm_head;
    ``"q4"`` takes every projection's and the lm_head's clip-searched packs
    (also "wd" per layer and "lmh").
    """

    def __init__(self, cfg: dict, weights: dict, rope_len: int, weight_format: str = "q4_rtn",
                 packs: dict | None = None):
        self.cfg = cfg
        d, H, Hkv = cfg["d_model"], cfg["n_head"], cfg["n_kv_head"]
        self.hd = d // H
        self.q_dim, self.kv_dim = H * self.hd, Hkv * self.hd
        self.eps = cfg["eps"]
        self.V = cfg["vocab"]
        self.F = cfg["ffn"]
        lowbit = {"ternary_g64": lambda w: ("tern",) + pack_ternary(w),
                  "q2_g64": lambda w: ("q2",) + pack_q2(w),
                  "ternary_pt": lambda w: ("tpt",) + ternary_pt_pack(w),
                  "q2k": lambda w: ("q2k",) + q2k_pack(w)}
        if weight_format not in ("q4_rtn", "q4_g128_sym", "q8", "q4_k_m", "q4", *lowbit):
            raise ValueError(f"unknown weight format {weight_format}")
        self.sym = weight_format == "q4_g128_sym"
        # every packed tensor carries its format: "marlin" (MARLIN Q4), "q4t"
        # (symmetric G128), "q8" (Q8_G64)
        q8 = lambda w: ("q8",) + pack_q8_g64(w)  # noqa: E731
        if weight_format == "q8":  # transformer.py:852-854: every projection Q8_G64
            pack = q8
        elif weight_format in lowbit:  # 2-bit projections and lm_head (transformer.py:857-862)
            pack = lowbit[weight_format]
        elif self.sym:
            pack = lambda w: ("q4t",) + q4t_pack(w, 128, True)  # noqa: E731
        else:
            pack = lambda w: ("marlin",) + pack_q4_marlin_rtn(w)  # noqa: E731
        tied = weights.get("lm_head") is None
        self.wte = pack_q8_g64(weights["wte"])
        if tied:
            self.lmh = ("q8",) + self.wte
        elif weight_format == "q4":  # the reference's clip-searched lm_head, from ``packs``
            self.lmh = ("marlin",) + tuple(packs["lmh"])
        else:  # q8 / q4_k_m: a Q8_G64 lm_head (transformer.py:842-846)
            self.lmh = q8(weights["lm_head"]) if weight_format in ("q8", "q4_k_m") else pack(weights["lm_head"])
        self.layers = []
        for i, lw in enumerate(weights["layers"]):
            gu = np.concatenate([_f32(_to_np(lw["w_gate"])), _f32(_to_np(lw["w_up"]))], 0)
            if weight_format in ("q4_k_m", "q4"):
                # MSE-clipped MARLIN packs (quant.py:495-571) as the reference
                # made them, passed in ``packs``; w_down Q8_G64 in q4_k_m
                # (transformer.py:847), clip-searched too in q4
                ent = dict(c_attn=("marlin",) + tuple(packs["c_attn"][i]), c_proj=("marlin",) + tuple(packs["c_proj"][i]),
                           gu=("marlin",) + tuple(packs["gu"][i]),
                           wd=("marlin",) + tuple(packs["wd"][i]) if weight_format == "q4" else q8(lw["w_down"]))
            else:
                ent = dict(c_attn=pack(lw["c_attn"]), c_proj=pack(lw["c_proj"]), gu=pack(gu), wd=pack(lw["w_down"]))
            ent.update(ln_1=torch.as_tensor(_to_np(lw["ln_1"])).float(),
                       ln_2=torch.as_tensor(_to_np(lw["ln_2"])).float())
            self.layers.append(ent)
        self.ln_f = torch.as_tensor(_to_np(weights["ln_f"])).float()
        self.freqs = rope_freqs(self.hd, rope_len, cfg.get("theta", 10000.0), cfg.get("rope_scaling"))
        self._dq = {}

    def _w(self, key, packed, K, n):
        if key not in self._dq:
            tag, p, s = packed[:3]
            if tag == "q4t":
                w = q4t_dequant(p, s, K, 128, True, n)
            elif tag == "q8":  # quant.py:132-147
                w = dequant_q8_g64(p, s, K)
            elif tag == "tern":  # quant.py:277-295
                w = dequant_ternary(p, s, K)
            elif tag == "q2":  # quant.py:383-403
                w = dequant_q2(p, s, K)
            elif tag == "tpt":
                w = ternary_pt_dequant(p, s)
            elif tag == "q2k":
                w = q2k_dequant(p, s, packed[3])
            else:
                w = dequant_q4_marlin(p, s, K, n)
            self._dq[key] = torch.from_numpy(w)
        return self._dq[key]

    def qlin(self, x: torch.Tensor, key, packed, n_out: int) -> torch.Tensor:
        """transformer.py:1010-1034 -> quant.py:656-661 / 201-233: dequant +
        F.linear in fp16, result cast back to ``x``'s dtype (fp32 after an
        fp32 norm)."""
        x16 = x.to(torch.float16)
        return F.linear(x16, self._w(key, packed, x16.size(-1), n_out)).to(x.dtype)

    def embed(self, idx: np.ndarray) -> torch.Tensor:
        return torch.from_numpy(dequant_q8_rows(idx, self.wte[0], self.wte[1]))

    def lm_head(self, xn: torch.Tensor) -> torch.Tensor:
        return self.qlin(xn, "lmh", self.lmh, self.V)

    def forward(self, idx: np.ndarray, cache: OracleCache, return_all: bool = False, hidden: list | None = None):
        """One ``_forward_quantized_sequence`` call (transformer.py:1036-1200).
        idx (B, T) ints.  Returns (logits fp16, x_norm).  With ``hidden`` (a
        list) the residual stream after each layer, (B, T, d) fp16, is
        appended to it."""
        idx = np.asarray(idx)
        B, T = idx.shape
        H, Hkv, hd = self.cfg["n_head"], self.cfg["n_kv_head"], self.hd
        x = self.embed(idx).view(B, T, -1)
        start = cache.seen
        slots = cache.slots(T)
        new_seen = start + T
        active = min(new_seen, cache.max_seq)
        for i, L in enumerate(self.layers):
            h1 = rmsnorm(x, L["ln_1"], self.eps)
            qkv = self.qlin(h1, (i, "qkv"), L["c_attn"], self.q_dim + 2 * self.kv_dim)
            q = qkv[..., : self.q_dim].view(B, T, H, hd).transpose(1, 2)
            k = qkv[..., self.q_dim : self.q_dim + self.kv_dim].view(B, T, Hkv, hd).transpose(1, 2)
            v = qkv[..., self.q_dim + self.kv_dim :].view(B, T, Hkv, hd).transpose(1, 2)
            f = self.freqs[start : start + T].view(1, 1, T, -1)
            q = _rope_apply(q, f)
            k = _rope_apply(k, f)
            cache.write(i, k.contiguous().numpy(), v.contiguous().numpy(), slots)
            kd, vd = cache.dequant(i, B, active)
            mask = None
            is_causal = False
            if T > 1 and start > 0:
                qp = (start + torch.arange(T)).unsqueeze(1)
                kp = torch.arange(kd.size(2)).unsqueeze(0)
                mask = kp <= qp
            else:
                is_causal = T > 1 and start == 0
            n_rep = H // Hkv
            y = F.scaled_dot_product_attention(
                q, _repeat_kv(kd, n_rep).to(q.dtype), _repeat_kv(vd, n_rep).to(q.dtype), attn_mask=mask, is_causal=is_causal
            )
            y = y.transpose(1, 2).contiguous().view(B, T, self.q_dim)
            x = x + self.qlin(y, (i, "o"), L["c_proj"], self.q_dim).to(x.dtype)
            h2 = rmsnorm(x, L["ln_2"], self.eps)
            gu = self.qlin(h2, (i, "gu"), L["gu"], 2 * self.F)
            g, u = gu.chunk(2, dim=-1)
            sw = F.silu(g) * u
            x = x + self.qlin(sw, (i, "down"), L["wd"], self.q_dim).to(x.dtype)
            if hidden is not None:
                hidden.append(x.clone())
        cache.seen = new_seen
        xt = x if (return_all or T == 1) else x[:, -1:, :]
        xn = rmsnorm(xt, self.ln_f, self.eps)
        return self.lm_head(xn), xn

    def forward_tree(self, idx: np.ndarray, cache: OracleCache, depths: list[int], masks: list[int]):
        """transformer.py:639-784 (the eager tree-verify path), B = 1."""
        idx = np.asarray(idx)
        B, T = idx.shape
        H, Hkv, hd = self.cfg["n_head"], self.cfg["n_kv_head"], self.hd
        seen = cache.seen
        write_pos = seen % cache.max_seq if (cache.ring_buffer or seen >= cache.max_seq) else seen
        assert write_pos + T <= cache.max_seq and seen == write_pos
        x = self.embed(idx).view(B, T, -1)
        didx = torch.tensor([(seen + int(d)) % self.freqs.size(0) for d in depths])
        f = self.freqs.index_select(0, didx).view(1, 1, T, -1)
        slots = list(range(write_pos, write_pos + T))
        for i, L in enumerate(self.layers):
            h1 = rmsnorm(x, L["ln_1"], self.eps)
            qkv = self.qlin(h1, (i, "qkv"), L["c_attn"], self.q_dim + 2 * self.kv_dim)
            q = qkv[..., : self.q_dim].view(B, T, H, hd).transpose(1, 2)
            k = qkv[..., self.q_dim : self.q_dim + self.kv_dim].view(B, T, Hkv, hd).transpose(1, 2)
            v = qkv[..., self.q_dim + self.kv_dim :].view(B, T, Hkv, hd).transpose(1, 2)
            q = _rope_apply(q, f)
            k = _rope_apply(k, f)
            cache.write(i, k.contiguous().numpy(), v.contiguous().numpy(), slots)
            kd, vd = cache.dequant(i, B, seen + T)
            y = attention_tree(q, kd, vd, masks, seen, write_pos)
            y = y.transpose(1, 2).contiguous().view(B, T, self.q_dim)
            x = x + self.qlin(y, (i, "o"), L["c_proj"], self.q_dim).to(x.dtype)
            h2 = rmsnorm(x, L["ln_2"], self.eps)
            gu = self.qlin(h2, (i, "gu"), L["gu"], 2 * self.F)
            g, u = gu.chunk(2, dim=-1)
            x = x + self.qlin(F.silu(g) * u, (i, "down"), L["wd"], self.q_dim).to(x.dtype)
        xn = rmsnorm(x, self.ln_f, self.eps)
        return self.lm_head(xn), xn

    def greedy(self, prompt: np.ndarray, n_new: int, cache: OracleCache) -> list[int]:
        """Prefill then greedy decode (argmax = first max index)."""
        logits, _ = self.forward(np.asarray(prompt).reshape(1, -1), cache)
        out = []
        tok = int(torch.argmax(logits[0, -1]).item())
        out.append(tok)
        for _ in range(n_new - 1):
            logits, _ = self.forward(np.array([[tok]]), cache)
            tok = int(torch.argmax(logits[0, -1]).item())
            out.append(tok)
        return out


# ---------------------------------------------------------------------------
# Medusa tree compile and greedy accept (engine/medusa.py:48-116, :314-330)
# ---------------------------------------------------------------------------


def compile_medusa_tree(tree_choices, num_heads: int, max_nodes: int = 32) -> dict:
    """engine/medusa.py:48-116.  ``max_nodes`` = 32 reproduces the reference
    (31 paths + root, uint32 masks); 64 is the B200 build's uint64 extension."""
    closed = set()
    for ch in tree_choices:
        t = tuple(int(r) for r in ch)
        if len(t) == 0 or len(t) > num_heads:
            continue
        for p in range(1, len(t) + 1):
            closed.add(t[:p])
    paths = sorted(closed, key=lambda p: (len(p), p))[: max_nodes - 1]
    T = 1 + len(paths)
    ids = {(): 0}
    depths = [0] * T
    masks = [0] * T
    parent = [-1] * T
    children = [[] for _ in range(T)]
    head_idx = [-1] * T
    topk_rank = [-1] * T
    max_topk = [1] * num_heads
    masks[0] = 1
    max_depth = 0
    for i, p in enumerate(paths):
        u = i + 1
        ids[p] = u
        d = len(p)
        max_depth = max(max_depth, d)
        pu = ids[p[:-1]]
        depths[u] = d
        parent[u] = pu
        children[pu].append(u)
        head_idx[u] = d - 1
        topk_rank[u] = p[-1]
        masks[u] = masks[pu] | (1 << u)
        max_topk[d - 1] = max(max_topk[d - 1], p[-1] + 1)
    return dict(
        num_nodes=T,
        tree_depths=depths,
        tree_mask=masks,
        parent=parent,
        children=children,
        head_idx=head_idx,
        topk_rank=topk_rank,
        max_topk_per_head=max_topk,
        max_depth=max_depth,
    )


def greedy_tree_accept(preds: list[int], verif_seq: list[int], children: list[list[int]], budget: int):
    """engine/medusa.py:314-330: emit argmax at the current node, descend to
    the first child whose token equals it, stop when none does or the budget
    (tokens still to generate) is exhausted.  Returns (accepted_nodes, emitted)."""
    cur = 0
    accepted = [0]
    emitted = []
    while len(emitted) < budget:
        tok = preds[cur]
        nxt = None
        for c in children[cur]:
            if verif_seq[c] == tok:
                nxt = c
                break
        emitted.append(tok)
        if nxt is None or len(emitted) >= budget:
            break
        cur = nxt
        accepted.append(cur)
    return accepted, emitted
