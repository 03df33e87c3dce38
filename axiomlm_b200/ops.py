"""Op-level host API: the reference's ``_METAL_MOD`` function table on CUDA.

Each function keeps the name, argument order and meaning of the binding it
replaces (``axiomlm/kernels/mps_kernels.mm:4302-4640``, called from
``axiomlm/kernels/quant.py`` and ``axiomlm/kernels/ops.py``) and runs the
sm_100a kernels of ``libaxb.so`` through the C ABI.  Inputs must be CUDA
tensors; there is no CPU path (the reference's own CPU code is the oracle).

Besides the ``*_mps``-named table entries, this module exposes the B200
formats: ``Q4TWeight`` (16-row mma-fragment tiles, 64207531 interleave,
group 64 affine or group 128 symmetric) and ``qgemm``.
"""

from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import torch

from . import _lib as L

# ---------------------------------------------------------------- plumbing


def _p(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _cuda(t: torch.Tensor, name: str):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (axiomlm_b200 has no CPU path)")
    return t.contiguous()


class _Workspace:
    """Per-device zero-initialised scratch; kernels leave it zeroed again."""

    def __init__(self):
        self.bufs: dict[int, torch.Tensor] = {}

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        b = self.bufs.get(idx)
        if b is None or b.numel() < nbytes:
            b = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self.bufs[idx] = b
        return b


# One workspace per kernel family: each keeps its own fixed-offset layout (the
# Q4 GEMV's tile counters must stay zero between calls), so two families must
# never share one.
_WS = _Workspace()
_LB_WS = _Workspace()
_ATTN_WS = _Workspace()

# ---------------------------------------------------------------- formats


@dataclass
class Q4TWeight:
    """A projection in the q4t layout: 16-row tiles, each tile's K range stored
    contiguously as 64-wide k-blocks of 512 B of mma A-fragment words."""

    words: torch.Tensor  # int32, (tiles * K/64 * 128,)
    scales: torch.Tensor  # fp16
    N: int
    K: int
    group: int
    fmt: int  # L.W_Q4T_SYM | L.W_Q4T_AFFINE
    gate_up: bool = False

    @property
    def nbytes(self) -> int:
        return self.words.numel() * 4 + self.scales.numel() * 2

    def dequant(self) -> torch.Tensor:
        out = torch.empty((self.N, self.K), dtype=torch.float16, device=self.words.device)
        L.call("axb_q4t_dequant", _p(self.words), _p(self.scales), self.N, self.K, self.group, self.fmt,
               int(self.gate_up), _p(out), _stream())
        return out


def _alloc_q4t(N: int, K: int, group: int, fmt: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    lib = L.load()
    wb = lib.axb_q4t_words_bytes(N, K)
    sb = lib.axb_q4t_scales_bytes(N, K, group, fmt)
    return (torch.empty(wb // 4, dtype=torch.int32, device=device),
            torch.empty(sb // 2, dtype=torch.float16, device=device))


def pack_q4t(w: torch.Tensor, group: int = 128, symmetric: bool = True, gate_up: bool = False) -> Q4TWeight:
    """RTN-pack fp32 (N, K) CUDA weights.  ``symmetric=False`` gives the
    reference's min/max affine rule (pack_linear_q4_marlin(clip_search=False))."""
    w = _cuda(w, "w").float()
    N, K = w.shape
    fmt = L.W_Q4T_SYM if symmetric else L.W_Q4T_AFFINE
    words, scales = _alloc_q4t(N, K, group, fmt, w.device)
    L.call("axb_q4t_pack", _p(w), N, K, group, fmt, int(gate_up), _p(words), _p(scales), _stream())
    return Q4TWeight(words, scales, N, K, group, fmt, gate_up)


def q4t_from_marlin(w_marlin: torch.Tensor, sb_marlin: torch.Tensor, n_out: int | None = None,
                    gate_up: bool = False) -> Q4TWeight:
    """Relayout the reference's MARLIN-ladder Q4 (quant.py:447-594) into q4t
    (bit-identical codes, scales and biases)."""
    wm = _cuda(w_marlin, "w_marlin")
    sb = _cuda(sb_marlin, "sb_marlin")
    nt8, kg = wm.shape[0], wm.shape[1]
    K = kg * 64
    N = n_out if (n_out is not None and n_out > 0) else nt8 * 8
    words, scales = _alloc_q4t(N, K, 64, L.W_Q4T_AFFINE, wm.device)
    L.call("axb_q4t_from_marlin", _p(wm), _p(sb), nt8, K, N, int(gate_up), _p(words), _p(scales), _stream())
    return Q4TWeight(words, scales, N, K, 64, L.W_Q4T_AFFINE, gate_up)


def q4t_from_q4g64(w_packed: torch.Tensor, scales_biases: torch.Tensor, n_out: int | None = None,
                   gate_up: bool = False) -> Q4TWeight:
    """Relayout the reference's legacy Q4_G64 pack (pack_linear_q4_g64,
    quant.py:17-69) into q4t affine G64 (bit-identical codes, scales, biases)."""
    wp = _cuda(w_packed, "w_packed")
    sb = _cuda(scales_biases, "scales_biases")
    N, K = wp.shape[0], wp.shape[1] * 8
    if n_out is not None and n_out != N:
        raise ValueError(f"legacy pack has {N} rows, expected {n_out}")
    words, scales = _alloc_q4t(N, K, 64, L.W_Q4T_AFFINE, wp.device)
    L.call("axb_q4t_from_q4g64", _p(wp), _p(sb), N, K, int(gate_up), _p(words), _p(scales), _stream())
    return Q4TWeight(words, scales, N, K, 64, L.W_Q4T_AFFINE, gate_up)


def q4_mse_codes(w: torch.Tensor, importance: torch.Tensor | None = None, steps: int = 13,
                 min_shrink: float = 0.72) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The reference's clip search for affine Q4 G64 (pack_linear_q4_marlin
    with clip_search=True, quant.py:495-571), on ``w``'s device: per 64-wide
    group, shrink the low end towards the group's (importance-weighted) mean
    by each of ``steps`` factors from 1 to ``min_shrink`` and keep the one
    with the least importance-weighted squared error, then the high end the
    same way at that low end.  Scale and bias are evaluated as the fp16 values
    they are stored as.  ``importance`` (K,) is squared and normalized to a
    unit mean per group.  The steps and their fp32 / fp16 rounding points are
    the reference's, so the packs are identical.  Returns codes (N, K) int32
    in 0..15, scales and biases (N, K/64) fp16."""
    w = w.float()
    N, K = w.shape
    if K % 64:
        raise ValueError(f"K ({K}) must be a multiple of 64")
    wg = w.reshape(N, K // 64, 64)
    imp = None
    if importance is not None:
        if importance.numel() != K:
            raise ValueError(f"importance has {importance.numel()} entries, expected {K}")
        imp = importance.to(w.device, torch.float32).reshape(1, K // 64, 64)
        imp = imp * imp
        imp = imp / imp.mean(dim=-1, keepdim=True).clamp(min=1e-8)
    lo0 = wg.amin(dim=-1, keepdim=True)
    hi0 = wg.amax(dim=-1, keepdim=True)
    mu = (wg * imp).mean(dim=-1, keepdim=True) if imp is not None else wg.mean(dim=-1, keepdim=True)
    shrink = torch.linspace(1.0, min_shrink, steps=max(2, steps)).tolist()

    def err(scale_h, bias_h):
        sc, bi = scale_h.float(), bias_h.float()
        q = ((wg - bi) / sc.clamp(min=1e-8)).round().clamp(0.0, 15.0)
        d = wg - (q * sc + bi)
        return (imp * (d * d)).sum(dim=-1) if imp is not None else (d * d).sum(dim=-1)

    # the low end, with the group's maximum
    best = torch.full(wg.shape[:2], float("inf"), dtype=torch.float32, device=w.device)
    lo = lo0.clone()
    for a in shrink:
        cand = mu + a * (lo0 - mu)
        e = err(((hi0 - cand).clamp(min=1e-8) / 15.0).to(torch.float16), cand.to(torch.float16))
        better = e < best
        best = torch.where(better, e, best)
        lo = torch.where(better.unsqueeze(-1), cand, lo)
    # the high end, at that low end
    best.fill_(float("inf"))
    bias = lo.to(torch.float16)
    scale = ((hi0 - lo).clamp(min=1e-8) / 15.0).to(torch.float16)
    for a in shrink:
        cand = mu + a * (hi0 - mu)
        sc_h = ((cand - lo).clamp(min=1e-8) / 15.0).to(torch.float16)
        e = err(sc_h, bias)
        better = e < best
        best = torch.where(better, e, best)
        scale = torch.where(better.unsqueeze(-1), sc_h, scale)
    q = ((wg - bias.float()) / scale.float().clamp(min=1e-8)).round().clamp(0.0, 15.0).to(torch.int32)
    return q.reshape(N, K), scale.reshape(N, K // 64), bias.reshape(N, K // 64)


def pack_q4_mse(w: torch.Tensor, importance: torch.Tensor | None = None, gate_up: bool = False) -> Q4TWeight:
    """The reference's default Q4 packing ("q4" / "q4_k_m": the clip search
    of ``q4_mse_codes``) as q4t affine G64: the codes go through the legacy
    Q4_G64 word layout (8 sequential nibbles per int32, quant.py:42-46) into
    the q4t relayout."""
    q, sc, bi = q4_mse_codes(w, importance)
    N, K = q.shape
    qv = q.reshape(N, K // 8, 8)
    words = torch.zeros((N, K // 8), dtype=torch.int32, device=q.device)
    for j in range(8):  # nibble j of a word holds k = 8 * word + j
        words |= (qv[:, :, j] & 0xF) << (4 * j)
    return q4t_from_q4g64(words, torch.stack([sc, bi], dim=-1), N, gate_up=gate_up)


def qmv_q4_g64(x: torch.Tensor, w_packed: torch.Tensor, scales_biases: torch.Tensor) -> torch.Tensor:
    """qmv_q4_g64 / qmm_q4_g64 (quant.py:166-198) through the q4t GEMV (the
    relayout is cached per weight tensor)."""
    key = (w_packed.data_ptr(), w_packed._version, scales_biases.data_ptr(), scales_biases._version,
           tuple(w_packed.shape))
    W = _LEGACY_CACHE.get(key)
    if W is None:
        if len(_LEGACY_CACHE) > 256:
            _LEGACY_CACHE.clear()
        W = q4t_from_q4g64(w_packed, scales_biases)
        _LEGACY_CACHE[key] = W
    K = x.shape[-1]
    y = qgemm(x.reshape(-1, K).half(), W)
    return y.view(*x.shape[:-1], W.N)


_LEGACY_CACHE: dict = {}
qmm_q4_g64 = qmv_q4_g64
# the Metal entry points' names (quant.py:177-178, 194)
qmv_q4_g64_mps = qmm_q4_g64_mps = qmv_q4_g64


@dataclass
class Q8Weight:
    """A projection in the reference's own Q8_G64 layout (quant.py:72-129):
    ``words`` (N, K/4) int32, ``scales`` (N, K/64, 2) fp16 scale and bias."""

    words: torch.Tensor
    scales: torch.Tensor
    N: int
    K: int
    group: int = 64
    fmt: int = L.W_Q8_G64

    @property
    def nbytes(self) -> int:
        return self.words.numel() * 4 + self.scales.numel() * 2


def qmv_q8_g64(x: torch.Tensor, w_packed: torch.Tensor, scales_biases: torch.Tensor) -> torch.Tensor:
    """qmv_q8_g64 / qmm_q8_g64 (quant.py:201-233): y = x . dequant(W)^T, fp16,
    with the weights dequantized as dequantize_q8_g64 does."""
    x = _cuda(x, "x").half()
    w = _cuda(w_packed, "w_packed")
    sb = _cuda(scales_biases, "scales_biases").half()
    K = x.shape[-1]
    N = w.shape[0]
    M = x.numel() // K
    y = torch.empty((*x.shape[:-1], N), dtype=torch.float16, device=x.device)
    L.call("axb_q8g64_gemv", _p(x), K, M, K, _p(w), _p(sb), N, _p(y), N, _stream())
    return y


qmm_q8_g64 = qmv_q8_g64
# the Metal entry points' names (quant.py:212-213, 229)
qmv_q8_g64_mps = qmm_q8_g64_mps = qmv_q8_g64


def pack_q8_g64(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """pack_linear_q8_g64 (quant.py:72-129) on the GPU."""
    w = _cuda(w, "w").float()
    N, K = w.shape
    out = torch.empty((N, K // 4), dtype=torch.int32, device=w.device)
    sb = torch.empty((N, K // 64, 2), dtype=torch.float16, device=w.device)
    L.call("axb_q8_pack", _p(w), N, K, _p(out), _p(sb), _stream())
    return out, sb


def dequantize_q4_marlin(w_marlin, sb_marlin, K: int, out_features: int | None = None) -> torch.Tensor:
    """quant.py:597-634 on the GPU (bit-exact)."""
    wm = _cuda(w_marlin, "w_marlin")
    sb = _cuda(sb_marlin, "sb_marlin")
    nt8 = wm.shape[0]
    N = out_features if out_features is not None else nt8 * 8
    out = torch.empty((N, K), dtype=torch.float16, device=wm.device)
    L.call("axb_q4_marlin_dequant", _p(wm), _p(sb), nt8, K, N, _p(out), _stream())
    return out


def dequant_q8_rows(indices: torch.Tensor, w_packed: torch.Tensor, scales_biases: torch.Tensor) -> torch.Tensor:
    """quant.py:132-163."""
    idx = _cuda(indices, "indices").to(torch.int32)
    w = _cuda(w_packed, "w_packed")
    sb = _cuda(scales_biases, "scales_biases")
    K = w.shape[1] * 4
    out = torch.empty((*indices.shape, K), dtype=torch.float16, device=w.device)
    L.call("axb_q8_rows", _p(w), _p(sb), _p(idx), idx.numel(), K, _p(out), _stream())
    return out


def dequantize_ternary(w_packed, scales, K: int | None = None) -> torch.Tensor:
    """quant.py:277-295 (per-group scales) or the per-tensor benchmark form
    when ``scales`` has one element."""
    w = _cuda(w_packed, "w_packed")
    s = _cuda(scales, "scales")
    N = w.shape[0]
    K = K or w.shape[1] * 4
    out = torch.empty((N, K), dtype=torch.float16, device=w.device)
    L.call("axb_ternary_dequant", _p(w), _p(s), N, K, int(s.numel() == 1), _p(out), _stream())
    return out


def dequantize_q2_k(w_packed, scales_biases, K: int | None = None) -> torch.Tensor:
    """quant.py:383-403."""
    w = _cuda(w_packed, "w_packed")
    sb = _cuda(scales_biases, "scales_biases")
    N = w.shape[0]
    K = K or w.shape[1] * 4
    out = torch.empty((N, K), dtype=torch.float16, device=w.device)
    L.call("axb_q2_dequant", _p(w), _p(sb), N, K, _p(out), _stream())
    return out


# ---------------------------------------------------------------- 2-bit weights


@dataclass
class Q2TWeight:
    """A 2-bit projection in the q2t layout (16-row tiles of mma fragments,
    128-wide k-blocks), relaid out from a reference packing: BitNet ternary
    with group-64 or per-tensor scales, 2-bit affine group 64 ("Q2_K" in the
    reference) or K-quant-style 256-element super-blocks."""

    words: torch.Tensor  # uint8 q2t codes
    meta: torch.Tensor | None  # per-group metadata (None for per-tensor ternary)
    meta2: torch.Tensor | None  # K-quant (d, dmin) per super-block
    pt_scale: torch.Tensor | None  # per-tensor ternary fp16 scale (1,)
    N: int
    K: int
    fmt: int
    group: int = 0  # unused: the format fixes its grouping

    def runner_meta(self) -> "L.Q2TMeta":
        """The axb_q2t_meta the decode runner takes in place of a scale pointer."""
        return L.Q2TMeta(meta=None if self.meta is None else self.meta.data_ptr(),
                         meta2=None if self.meta2 is None else self.meta2.data_ptr(),
                         pt_scale=None if self.pt_scale is None else self.pt_scale.data_ptr())

    @property
    def nbytes(self) -> int:
        n = self.words.numel()
        for t in (self.meta, self.meta2, self.pt_scale):
            if t is not None:
                n += t.numel() * t.element_size()
        return n

    def dequant(self) -> torch.Tensor:
        out = torch.empty((self.N, self.K), dtype=torch.float16, device=self.words.device)
        L.call("axb_q2t_dequant", self.fmt, _p(self.words), _p(self.meta), _p(self.meta2), _p(self.pt_scale),
               self.N, self.K, _p(out), _stream())
        return out


def q2t_from_ref(fmt: int, codes: torch.Tensor, s1: torch.Tensor | None = None, s2: torch.Tensor | None = None,
                 K: int | None = None) -> Q2TWeight:
    """Relayout a reference 2-bit packing (``L.W_TERNARY_G64``: codes +
    group scales, quant.py:236-274; ``L.W_TERNARY_PT``: codes + one scale;
    ``L.W_Q2_G64``: codes + (scale, bias), quant.py:339-381;
    ``L.W_Q2K_SB256``: codes + sub bytes + (d, dmin)) into q2t."""
    c = _cuda(codes, "codes")
    if c.dtype != torch.uint8:
        raise RuntimeError("codes must be uint8 (4 codes per byte)")
    N = c.shape[0]
    K = K or c.shape[1] * 4
    lib = L.load()
    dev = c.device
    words = torch.empty(lib.axb_q2t_words_bytes(N, K), dtype=torch.uint8, device=dev)
    mb, m2b = lib.axb_q2t_meta_bytes(fmt, N, K), lib.axb_q2t_meta2_bytes(fmt, N, K)
    meta = torch.zeros(mb, dtype=torch.uint8, device=dev) if mb else None
    meta2 = torch.zeros(m2b, dtype=torch.uint8, device=dev) if m2b else None
    a = None if s1 is None else _cuda(s1, "s1")
    b = None if s2 is None else _cuda(s2, "s2")
    if words.numel() == 0:
        raise RuntimeError(f"q2t: K={K} must be a multiple of 128")
    L.call("axb_q2t_from_ref", fmt, _p(c), _p(a), _p(b), N, K, _p(words), _p(meta), _p(meta2), _stream())
    pt = a.to(torch.float16).reshape(1).contiguous() if fmt == L.W_TERNARY_PT else None
    return Q2TWeight(words, meta, meta2, pt, N, K, fmt)


def _pack4_2bit(c: torch.Tensor) -> torch.Tensor:
    """Four 2-bit codes per byte, element 4i + j at bits 2j (quant.py:266-273)."""
    N, K = c.shape
    c = c.to(torch.uint8).reshape(N, K // 4, 4)
    return (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).contiguous()


def ternary_g64_codes(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """pack_linear_ternary (quant.py:236-274) on ``w``'s device: per group of
    64 the absmean scale (in ``w``'s dtype, clamped to 1e-5, as fp16), codes
    round(w / scale) clamped to -1..1 as 0 -> 0, +1 -> 1, -1 -> 2.  Returns
    codes (N, K/4) uint8 and scales (N, K/64) fp16."""
    N, K = w.shape
    wg = w.reshape(N, K // 64, 64)
    scale = wg.abs().mean(dim=-1, keepdim=True).clamp(min=1e-5).to(torch.float16)
    q = torch.clamp(torch.round(wg.float() / scale.float().clamp(min=1e-5)), -1.0, 1.0)
    code = torch.where(q == 1, 1, torch.where(q == -1, 2, 0))
    return _pack4_2bit(code.reshape(N, K)), scale.reshape(N, K // 64)


def q2_g64_codes(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """pack_linear_q2_k (quant.py:339-381; 2-bit affine per group of 64) on
    ``w``'s device: scale fp16((max - min) / 3), bias fp16(min) (the range in
    ``w``'s dtype), codes round((w - bias) / scale) in 0..3.  Returns codes
    (N, K/4) uint8 and (scale, bias) pairs (N, K/64, 2) fp16."""
    N, K = w.shape
    wg = w.reshape(N, K // 64, 64)
    lo = wg.amin(dim=-1, keepdim=True)
    hi = wg.amax(dim=-1, keepdim=True)
    scale = (torch.clamp(hi - lo, min=1e-8) / 3.0).to(torch.float16)
    bias = lo.to(torch.float16)
    q = torch.clamp(torch.round((wg.float() - bias.float()) / torch.clamp(scale.float(), min=1e-8)), 0.0, 3.0)
    return _pack4_2bit(q.reshape(N, K)), torch.stack([scale.squeeze(-1), bias.squeeze(-1)], dim=-1).contiguous()


def ternary_pt_codes(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """BitNet b1.58 with one per-tensor absmean scale (the benchmark-only
    layout; the reference packs per group of 64): scale fp16(max(mean |w|,
    1e-5)) with the mean in float64, codes round(w / scale) clamped to -1..1
    in the reference's 2-bit code and byte order.  Returns codes (N, K/4)
    uint8 and the scale (1,) fp16."""
    N, K = w.shape
    s16 = torch.clamp(w.double().abs().mean(), min=1e-5).to(torch.float16)
    q = torch.clamp(torch.round(w.float() / s16.float()), -1.0, 1.0)
    code = torch.where(q == 1, 1, torch.where(q == -1, 2, 0))
    return _pack4_2bit(code), s16.reshape(1)


def q2k_sb256_codes(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """K-quant-style 2-bit super-blocks (the benchmark-only layout): per 256
    weights fp16 ``d`` and ``dmin`` (the largest 16-element sub-block scale
    and sub-min over 15), per 16 weights a 4-bit sub-scale and sub-min, codes
    round((w + dmin * mn) / (d * sc)) in 0..3, all in fp32.  Returns codes
    (N, K/4) uint8, sub-bytes (N, K/16) uint8 (scale | min << 4) and (d, dmin)
    (N, K/256, 2) fp16."""
    w = w.float()
    N, K = w.shape
    if K % 256:
        raise ValueError(f"K ({K}) must be a multiple of 256")
    sb = w.reshape(N, K // 256, 16, 16)
    mn = torch.clamp(sb.amin(dim=-1), max=0.0)
    sub_scale = torch.clamp(sb.amax(dim=-1) - mn, min=1e-8) / 3.0
    sub_min = -mn
    d = (sub_scale.amax(dim=-1) / 15.0).to(torch.float16)
    dmin = (sub_min.amax(dim=-1) / 15.0).to(torch.float16)
    df = torch.clamp(d.float(), min=1e-8)[..., None]
    mf = torch.clamp(dmin.float(), min=1e-8)[..., None]
    sc = torch.clamp(torch.round(sub_scale / df), 0, 15)
    mi = torch.clamp(torch.round(sub_min / mf), 0, 15)
    eff_s = d.float()[..., None] * sc
    eff_m = dmin.float()[..., None] * mi
    q = torch.clamp(torch.round((sb + eff_m[..., None]) / torch.clamp(eff_s, min=1e-12)[..., None]), 0, 3)
    sub = (sc.to(torch.uint8) | (mi.to(torch.uint8) << 4)).reshape(N, K // 16).contiguous()
    return _pack4_2bit(q.reshape(N, K)), sub, torch.stack([d, dmin], dim=-1).contiguous()


def pack_q2t(w: torch.Tensor, fmt: int) -> Q2TWeight:
    """fp32 / fp16 weights packed in a 2-bit format on their device, then
    relaid out into q2t: ``L.W_TERNARY_G64`` / ``L.W_Q2_G64`` (the reference's
    ternary / q2_k packings), ``L.W_TERNARY_PT`` / ``L.W_Q2K_SB256``."""
    N, K = w.shape
    if fmt == L.W_TERNARY_G64:
        c, s1 = ternary_g64_codes(w)
        return q2t_from_ref(fmt, c, s1, None, K)
    if fmt == L.W_Q2_G64:
        c, s1 = q2_g64_codes(w)
        return q2t_from_ref(fmt, c, s1, None, K)
    if fmt == L.W_TERNARY_PT:
        c, s1 = ternary_pt_codes(w)
        return q2t_from_ref(fmt, c, s1, None, K)
    if fmt == L.W_Q2K_SB256:
        c, s1, s2 = q2k_sb256_codes(w)
        return q2t_from_ref(fmt, c, s1, s2, K)
    raise ValueError(f"format {fmt} is not a 2-bit format")


def lbgemm(x: torch.Tensor, W: Q2TWeight, bias: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """y[M, N] = x[M, K] W^T (+ bias) on the 2-bit tensor-core kernel (M <= 8
    per launch; larger M is chunked)."""
    x = _cuda(x, "x")
    if x.dtype != torch.float16:
        x = x.to(torch.float16)
    lead = x.shape[:-1]
    K = x.shape[-1]
    if K != W.K:
        raise RuntimeError(f"x has K={K}, weight has K={W.K}")
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    if out is None:
        out = torch.empty((M, W.N), dtype=torch.float16, device=x.device)
    o2 = out.view(M, W.N)
    lib = L.load()
    ws = _LB_WS.get(lib.axb_lbgemv_workspace_bytes(W.fmt, W.N, K, 8), x.device)
    b = None if bias is None else _cuda(bias, "bias").to(torch.float16)
    for m0 in range(0, M, 8):
        m = min(8, M - m0)
        d = L.LbGemvDesc(fmt=W.fmt, words=W.words.data_ptr(),
                         meta=None if W.meta is None else W.meta.data_ptr(),
                         meta2=None if W.meta2 is None else W.meta2.data_ptr(),
                         pt_scale=None if W.pt_scale is None else W.pt_scale.data_ptr(),
                         N=W.N, K=K, M=m, x=x2.data_ptr() + m0 * K * 2, ldx=K, y=o2.data_ptr() + m0 * W.N * 2,
                         ldy=W.N, bias=None if b is None else b.data_ptr(), workspace=ws.data_ptr(),
                         workspace_bytes=ws.numel())
        L.call("axb_lbgemv", C.byref(d), _stream())
    return out.view(*lead, W.N)


_Q2T_CACHE: dict = {}


def _cached_q2t(fmt: int, codes: torch.Tensor, s1: torch.Tensor, s2: torch.Tensor | None = None) -> Q2TWeight:
    # relayout once per (tensor storage, version): weights are constant in decode
    key = (fmt, codes.data_ptr(), codes._version, s1.data_ptr(), s1._version,
           None if s2 is None else (s2.data_ptr(), s2._version), tuple(codes.shape))
    hit = _Q2T_CACHE.get(key)
    if hit is None:
        if len(_Q2T_CACHE) > 256:
            _Q2T_CACHE.clear()
        hit = q2t_from_ref(fmt, codes, s1, s2)
        _Q2T_CACHE[key] = hit
    return hit


def qmv_ternary_mps(x, w_packed, scales, bias=None) -> torch.Tensor:
    """``_METAL_MOD.qmv_ternary_mps`` (quant.py:298-317): y = x W^T (+ bias)
    for BitNet ternary; ``scales`` (N, K/64) per group, or one element for
    the per-tensor form."""
    w = _cuda(w_packed, "w_packed")
    s = _cuda(scales, "scales")
    fmt = L.W_TERNARY_PT if s.numel() == 1 else L.W_TERNARY_G64
    return lbgemm(x, _cached_q2t(fmt, w, s), bias=bias)


qmm_ternary_mps = qmv_ternary_mps


def qmv_q2_k_mps(x, w_packed, scales_biases, bias=None) -> torch.Tensor:
    """``_METAL_MOD.qmv_q2_k_mps`` (quant.py:406-425): y = x W^T (+ bias) for
    the reference's group-64 affine 2-bit format."""
    return lbgemm(x, _cached_q2t(L.W_Q2_G64, _cuda(w_packed, "w_packed"), _cuda(scales_biases, "scales_biases")),
                  bias=bias)


qmm_q2_k_mps = qmv_q2_k_mps


# ---------------------------------------------------------------- GEMV


def qgemm(x: torch.Tensor, W: Q4TWeight, bias: torch.Tensor | None = None, norm_w: torch.Tensor | None = None,
          eps: float = 1e-5, epilogue: int = L.EPI_STORE, out: torch.Tensor | None = None) -> torch.Tensor:
    """y[M, N] = x[M, K] W^T on the q4t kernel (M <= 64 per call; larger M is
    chunked).  ``norm_w`` fuses RMSNorm (fp32 weight) into the prologue;
    ``epilogue`` = EPI_RESIDUAL adds into ``out`` in place; EPI_SWIGLU needs a
    gate/up-interleaved weight and returns (M, N/2)."""
    x = _cuda(x, "x")
    if x.dtype != torch.float16:
        x = x.to(torch.float16)
    lead = x.shape[:-1]
    K = x.shape[-1]
    if K != W.K:
        raise RuntimeError(f"x has K={K}, weight has K={W.K}")
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    n_out = W.N // 2 if epilogue == L.EPI_SWIGLU else W.N
    if out is None:
        dt = torch.float32 if epilogue == L.EPI_F32 else torch.float16
        out = torch.empty((M, n_out), dtype=dt, device=x.device)
    o2 = out.view(M, n_out)
    lib = L.load()
    ws = _WS.get(lib.axb_qgemm_workspace_bytes(W.N, K, min(M, 64), W.group), x.device)
    nw = None if norm_w is None else _cuda(norm_w, "norm_w").float()
    b = None if bias is None else _cuda(bias, "bias").to(torch.float16)
    esz = o2.element_size()
    for m0 in range(0, M, 64):
        m = min(64, M - m0)
        d = L.QGemmDesc(fmt=W.fmt, group=W.group, words=W.words.data_ptr(), scales=W.scales.data_ptr(),
                        N=W.N, K=K, M=m, x=x2.data_ptr() + m0 * K * 2, ldx=K,
                        y=o2.data_ptr() + m0 * n_out * esz, ldy=n_out,
                        bias=None if b is None else b.data_ptr(), norm_w=None if nw is None else nw.data_ptr(),
                        eps=eps, epilogue=epilogue, gate_up_interleave=int(W.gate_up),
                        workspace=ws.data_ptr(), workspace_bytes=ws.numel(), pdl=0)
        L.call("axb_qgemm", C.byref(d), _stream())
    return out.view(*lead, n_out)


_TC_WS = _Workspace()


def qgemm_tc(x: torch.Tensor, W: Q4TWeight, bias: torch.Tensor | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """y[M, N] = x[M, K] W^T (+ bias) on the tcgen05 tensor-core kernel: the
    dense-contraction path for many tokens (tree verification, prefill
    chunks, large decode batches).  M <= 64 per launch; larger M is chunked.
    Weights are dequantized to the reference's fp16 values and accumulated in
    fp32."""
    x = _cuda(x, "x")
    if x.dtype != torch.float16:
        x = x.to(torch.float16)
    lead = x.shape[:-1]
    K = x.shape[-1]
    if K != W.K:
        raise RuntimeError(f"x has K={K}, weight has K={W.K}")
    if W.gate_up:
        raise RuntimeError("qgemm_tc stores rows in order: pass a weight packed without the gate/up interleave")
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    if out is None:
        out = torch.empty((M, W.N), dtype=torch.float16, device=x.device)
    o2 = out.view(M, W.N)
    lib = L.load()
    ws = _TC_WS.get(lib.axb_qgemm_tc_workspace_bytes(W.N, K, 64), x.device)
    b = None if bias is None else _cuda(bias, "bias").to(torch.float16)
    for m0 in range(0, M, 64):
        m = min(64, M - m0)
        d = L.QGemmDesc(fmt=W.fmt, group=W.group, words=W.words.data_ptr(), scales=W.scales.data_ptr(),
                        N=W.N, K=K, M=m, x=x2.data_ptr() + m0 * K * 2, ldx=K, y=o2.data_ptr() + m0 * W.N * 2,
                        ldy=W.N, bias=None if b is None else b.data_ptr(), norm_w=None, eps=0.0,
                        epilogue=L.EPI_STORE, gate_up_interleave=0, workspace=ws.data_ptr(),
                        workspace_bytes=ws.numel(), pdl=0)
        L.call("axb_qgemm_tc", C.byref(d), _stream())
    return out.view(*lead, W.N)


def qgemm_tc_status() -> int:
    """Synchronizes; AXB_ETIMEOUT if a bounded tensor-core wait ran out."""
    b = _TC_WS.bufs.get(torch.cuda.current_device())
    if b is None:
        return 0
    return L.load().axb_qgemm_tc_status(C.c_void_p(b.data_ptr()), _stream())


_MARLIN_CACHE: dict = {}


def _marlin_as_q4t(w_marlin: torch.Tensor, sb_marlin: torch.Tensor, n_out: int) -> Q4TWeight:
    # relayout once per (tensor storage, version): weights are constant in decode
    key = (w_marlin.data_ptr(), w_marlin._version, sb_marlin.data_ptr(), sb_marlin._version, n_out)
    hit = _MARLIN_CACHE.get(key)
    if hit is None:
        if len(_MARLIN_CACHE) > 256:
            _MARLIN_CACHE.clear()
        hit = q4t_from_marlin(w_marlin, sb_marlin, n_out)
        _MARLIN_CACHE[key] = hit
    return hit


def qmv_q4_marlin_mps(x, w_marlin, sb_marlin, n_out: int = -1, bias=None) -> torch.Tensor:
    """``_METAL_MOD.qmv_q4_marlin_mps`` (quant.py:648-654): y = x W^T (+ bias)
    for reference-layout MARLIN Q4.  ``n_out`` = -1 means 8 * N_tiles."""
    N = n_out if n_out is not None and n_out > 0 else w_marlin.shape[0] * 8
    W = _marlin_as_q4t(_cuda(w_marlin, "w_marlin"), _cuda(sb_marlin, "sb_marlin"), N)
    return qgemm(x, W, bias=bias)


qmm_q4_marlin_mps = qmv_q4_marlin_mps


def rmsnorm_infer_mps(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm (modules.py:30-43) with an fp32 weight, fp16 output."""
    x = _cuda(x, "x").to(torch.float16)
    K = x.shape[-1]
    out = torch.empty_like(x)
    L.call("axb_rmsnorm", _p(x), _p(_cuda(weight, "weight").float()), x.numel() // K, K, float(eps), _p(out),
           _stream())
    return out


def argmax_last_token_mps(logits: torch.Tensor) -> torch.Tensor:
    """Greedy argmax over the last dim (ties -> lowest index, as torch.argmax)."""
    x = _cuda(logits, "logits").to(torch.float16)
    n = x.shape[-1]
    rows = x.numel() // n
    out = torch.empty(rows, dtype=torch.int32, device=x.device)
    L.call("axb_argmax", _p(x), rows, n, n, _p(out), _stream())
    return out.view(x.shape[:-1]).long()


# ---------------------------------------------------------------- KV cache ops


def _kv_group_of(head_dim: int, scales: torch.Tensor | None) -> int:
    if scales is None:
        return 64
    return head_dim // scales.shape[-1]


def quantize_kv(x: torch.Tensor, kv_dtype: str, group: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """quantize_kv_fp8 / quantize_kv_int4 (quant.py:692-807) for one tensor:
    fp16 inputs follow the fp16 rule, fp32 inputs the fp32 rule."""
    x = _cuda(x, "x")
    if x.dtype not in (torch.float16, torch.float32):
        x = x.float()
    hd = x.shape[-1]
    rows = x.numel() // hd
    kt = L.KV_TYPES[kv_dtype]
    width = hd if kt == L.KV_FP8 else hd // 2
    q = torch.empty((*x.shape[:-1], width), dtype=torch.uint8, device=x.device)
    s = torch.empty((*x.shape[:-1], hd // group), dtype=torch.float16, device=x.device)
    L.call("axb_kv_quantize", _p(x), int(x.dtype == torch.float32), rows, hd, kt, group, _p(q), _p(s), _stream())
    return q, s


def quantize_kv_fp8(k, v):
    kq, ks = quantize_kv(k, "fp8")
    vq, vs = quantize_kv(v, "fp8")
    return kq, ks, vq, vs


def quantize_kv_int4(k, v):
    kq, ks = quantize_kv(k, "int4")
    vq, vs = quantize_kv(v, "int4")
    return kq, ks, vq, vs


def dequantize_kv(q: torch.Tensor, scales: torch.Tensor, kv_dtype: str, head_dim: int | None = None):
    q = _cuda(q, "q")
    s = _cuda(scales, "scales")
    kt = L.KV_TYPES[kv_dtype]
    hd = head_dim or (q.shape[-1] if kt == L.KV_FP8 else q.shape[-1] * 2)
    rows = q.numel() // q.shape[-1]
    out = torch.empty((*q.shape[:-1], hd), dtype=torch.float16, device=q.device)
    L.call("axb_kv_dequantize", _p(q), _p(s), rows, hd, kt, hd // s.shape[-1], _p(out), _stream())
    return out


def dequantize_kv_cache_fp8_mps(cache, scales, n_kv_head: int, seq_len: int, head_dim: int):
    return dequantize_kv(cache, scales, "fp8", head_dim)


def dequantize_kv_cache_int4_mps(cache, scales, n_kv_head: int, seq_len: int, head_dim: int):
    return dequantize_kv(cache, scales, "int4", head_dim)


def _as_cache4(t: torch.Tensor) -> torch.Tensor:
    return t if t.dim() == 4 else t.unsqueeze(0)


def _attention(q, k_cache, v_cache, k_scales, v_scales, kv_dtype, *, active_len=0, num_splits=0, masks=None,
               prefix_len=0, write_pos=0, T=1):
    q = _cuda(q, "q")
    kc = _as_cache4(_cuda(k_cache, "k_cache"))
    vc = _as_cache4(_cuda(v_cache, "v_cache"))
    kt = L.KV_TYPES[kv_dtype]
    Bc, Hkv, S = kc.shape[0], kc.shape[1], kc.shape[2]
    hd = q.shape[-1] if q.dim() == 4 else None
    if kt == L.KV_F16:
        hd = kc.shape[3]
    elif kt == L.KV_FP8:
        hd = kc.shape[3]
    else:
        hd = kc.shape[3] * 2
    if hd > 128 or hd % 2:
        raise ValueError(f"head_dim must be even and <= 128, got {hd}")
    Hq = q.numel() // (hd * T * Bc) if masks is not None else q.numel() // (hd * Bc)
    ks = None if kt == L.KV_F16 else _as_cache4(_cuda(k_scales, "k_scales"))
    vs = None if kt == L.KV_F16 else _as_cache4(_cuda(v_scales, "v_scales"))
    group = _kv_group_of(hd, ks)
    qf = q.contiguous()
    out = torch.empty((Bc * (T if masks is not None else 1), Hq * hd), dtype=torch.float16, device=q.device)
    lib = L.load()
    ws = _ATTN_WS.get(lib.axb_attn_workspace_bytes(Bc, Hq, Hkv, hd, S, kt, num_splits), q.device)
    mask_t = None
    if masks is not None:
        mask_t = torch.tensor([int(m) & 0xFFFFFFFFFFFFFFFF for m in masks], dtype=torch.uint64, device=q.device)
    d = L.AttnDesc(kv_type=kt, kv_group=group, B=Bc, n_head=Hq, n_kv_head=Hkv, head_dim=hd, max_seq=S,
                   max_batch=Bc, q=qf.data_ptr(), q_is_fp32=int(qf.dtype == torch.float32),
                   k_cache=kc.data_ptr(), v_cache=vc.data_ptr(),
                   k_scale=None if ks is None else ks.data_ptr(), v_scale=None if vs is None else vs.data_ptr(),
                   out=out.data_ptr(), active_len=active_len, num_splits=num_splits, T=T, prefix_len=prefix_len,
                   write_pos=write_pos, masks=None if mask_t is None else mask_t.data_ptr(), dev_params=None,
                   workspace=ws.data_ptr(), workspace_bytes=ws.numel(), pdl=0)
    L.call("axb_attention", C.byref(d), _stream())
    return out


def gqa_flash_decode_mps(q, k_cache, v_cache, active_len: int, num_splits: int = 0, k_scales=None, v_scales=None,
                         kv_dtype: str = "fp16"):
    """gqa_flash_decode_mps (ops.py:552-654): T_q = 1, all slots < active_len."""
    out = _attention(q, k_cache, v_cache, k_scales, v_scales, kv_dtype.lower(), active_len=active_len,
                     num_splits=num_splits)
    return out.view(q.shape)


def gqa_flash_decode_fp8_mps(q, k_cache, v_cache, k_scales, v_scales, active_len, num_splits=0):
    return gqa_flash_decode_mps(q, k_cache, v_cache, active_len, num_splits, k_scales, v_scales, "fp8")


def gqa_flash_decode_int4_mps(q, k_cache, v_cache, k_scales, v_scales, active_len, num_splits=0):
    return gqa_flash_decode_mps(q, k_cache, v_cache, active_len, num_splits, k_scales, v_scales, "int4")


def gqa_tree_verify_mps(q, k_cache, v_cache, tree_mask, prefix_len: int, write_pos: int, n_head: int,
                        num_splits: int = 0, k_scales=None, v_scales=None, kv_dtype: str = "fp16"):
    """gqa_tree_verify_mps (ops.py:657-797).  q: (T, Hq*hd) / (1, T, Hq*hd) or
    (1, Hq, T, hd); output (T, Hq*hd) laid out token-major.  Masks are up to
    64 bits (the reference's Metal path is limited to 32 nodes)."""
    masks = [int(m) for m in (tree_mask.tolist() if isinstance(tree_mask, torch.Tensor) else tree_mask)]
    T = len(masks)
    if T < 1 or T > 64:
        raise ValueError(f"tree verify supports 1..64 nodes, got {T}")
    if q.dim() == 4:
        q_tok = q.transpose(1, 2).reshape(1, T, -1)
    else:
        q_tok = q.reshape(1, T, -1)
    return _attention(q_tok, k_cache, v_cache, k_scales, v_scales, kv_dtype.lower(), masks=masks,
                      prefix_len=prefix_len, write_pos=write_pos, T=T)


def gqa_tree_verify_fp8_mps(q, k_cache, v_cache, k_scales, v_scales, tree_mask, prefix_len: int, write_pos: int,
                            n_head: int, num_splits: int = 0):
    """The FP8-cache tree verify in the argument order of the Metal entry
    point (ops.py:697-708)."""
    return gqa_tree_verify_mps(q, k_cache, v_cache, tree_mask, prefix_len, write_pos, n_head, num_splits, k_scales,
                               v_scales, "fp8")


def gqa_tree_verify_int4_mps(q, k_cache, v_cache, k_scales, v_scales, tree_mask, prefix_len: int, write_pos: int,
                             n_head: int, num_splits: int = 0):
    """The INT4-cache tree verify in the argument order of the Metal entry
    point (ops.py:715-726)."""
    return gqa_tree_verify_mps(q, k_cache, v_cache, tree_mask, prefix_len, write_pos, n_head, num_splits, k_scales,
                               v_scales, "int4")


def compact_tree_kv(cache: torch.Tensor, scales: torch.Tensor | None, write_pos: int, accepted: list[int],
                    cache_dtype: str):
    """compact_tree_kv_mps / compact_tree_kv_quant_mps (paged_cache.py:376-462)."""
    cache = _cuda(cache, "cache")
    L_, two, Bm, H, S, W = cache.shape
    row_bytes = W * cache.element_size()
    ng = 0 if scales is None else scales.shape[-1]
    acc = torch.tensor([int(a) for a in accepted], dtype=torch.int32, device=cache.device)
    L.call("axb_compact_kv", _p(cache), _p(scales), L_, Bm, H, S, row_bytes, ng, int(write_pos), _p(acc), len(accepted),
           _stream())


def compact_tree_kv_mps(cache, write_pos, accepted):
    compact_tree_kv(cache, None, write_pos, accepted, "fp16")


def compact_tree_kv_quant_mps(cache, scales, write_pos, accepted, cache_dtype):
    compact_tree_kv(cache, scales, write_pos, accepted, cache_dtype)


def rope_kv_cache_write(qkv, freqs_real, k_cache, v_cache, k_scales, v_scales, q_dim: int, kv_dim: int,
                        head_dim: int, start_pos: int, write_pos: int, kv_dtype: str = "fp16", qkv_bias=None):
    """rope_kv_cache_write_quantized (quant.py:896-1008) for one token: RoPE
    on Q and K in place in ``qkv`` (fp16) and K/V written (quantized) to slot
    ``write_pos``."""
    qkv = _cuda(qkv, "qkv")
    if qkv.dtype != torch.float16:
        raise RuntimeError("qkv must be fp16")
    n_head, n_kv = q_dim // head_dim, kv_dim // head_dim
    kc = _as_cache4(k_cache)
    fr = freqs_real if not torch.is_complex(freqs_real) else torch.view_as_real(freqs_real)
    fr = _cuda(fr, "freqs").float().contiguous()
    q_out = torch.empty((1, q_dim), dtype=torch.float32, device=qkv.device)
    kt = L.KV_TYPES[kv_dtype]
    ks = None if kt == L.KV_F16 else _as_cache4(k_scales)
    d = L.KvWriteDesc(kv_type=kt, kv_group=_kv_group_of(head_dim, ks), B=1, T=1, n_head=n_head, n_kv_head=n_kv,
                      head_dim=head_dim, max_seq=kc.shape[2], max_batch=kc.shape[0], qkv=qkv.data_ptr(),
                      bias=None if qkv_bias is None else _cuda(qkv_bias, "bias").half().data_ptr(),
                      rope=fr.data_ptr(), rope_len=fr.shape[0], rope_pos=start_pos, depths=None,
                      write_pos=write_pos, q_out=q_out.data_ptr(), dev_params=None, k_cache=kc.data_ptr(),
                      v_cache=_as_cache4(v_cache).data_ptr(), k_scale=None if ks is None else ks.data_ptr(),
                      v_scale=None if ks is None else _as_cache4(v_scales).data_ptr(), k_is_fp32=0)
    L.call("axb_rope_kv_write", C.byref(d), _stream())
    qkv.view(-1)[:q_dim].copy_(q_out.view(-1).to(torch.float16))


def rope_kv_cache_write_mps(qkv, freqs_real, k_cache, v_cache, q_dim, kv_dim, head_dim, start_pos, write_pos):
    rope_kv_cache_write(qkv, freqs_real, k_cache, v_cache, None, None, q_dim, kv_dim, head_dim, start_pos, write_pos)


def rope_kv_cache_write_fp8_mps(qkv, freqs_real, k_cache, v_cache, k_scales, v_scales, q_dim, kv_dim, head_dim,
                                start_pos, write_pos, qkv_bias=None):
    rope_kv_cache_write(qkv, freqs_real, k_cache, v_cache, k_scales, v_scales, q_dim, kv_dim, head_dim, start_pos,
                        write_pos, "fp8", qkv_bias)


def rope_kv_cache_write_int4_mps(qkv, freqs_real, k_cache, v_cache, k_scales, v_scales, q_dim, kv_dim, head_dim,
                                 start_pos, write_pos, qkv_bias=None):
    rope_kv_cache_write(qkv, freqs_real, k_cache, v_cache, k_scales, v_scales, q_dim, kv_dim, head_dim, start_pos,
                        write_pos, "int4", qkv_bias)


def rope_table(head_dim: int, max_seq_len: int, theta: float = 10000.0, rope_scaling: dict | None = None):
    """precompute_rope_frequencies (modules.py:46-92) as (S, hd/2, 2) fp32,
    computed with the same torch ops so the table is bit-identical."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    if rope_scaling is not None:
        rtype = rope_scaling.get("rope_type", rope_scaling.get("type", "default"))
        if rtype == "llama3":
            factor = float(rope_scaling["factor"])
            lo_f = float(rope_scaling.get("low_freq_factor", 1.0))
            hi_f = float(rope_scaling.get("high_freq_factor", 4.0))
            old = float(rope_scaling.get("original_max_position_embeddings", 8192))
            wavelen = 2.0 * math.pi / inv_freq
            inv_l = torch.where(wavelen > old / lo_f, inv_freq / factor, inv_freq)
            smooth = (old / wavelen - lo_f) / (hi_f - lo_f)
            smoothed = (1.0 - smooth) * inv_l / factor + smooth * inv_l
            medium = ~(wavelen < old / hi_f) & ~(wavelen > old / lo_f)
            inv_freq = torch.where(medium, smoothed, inv_l)
        elif rtype == "linear" and "factor" in rope_scaling:
            inv_freq = inv_freq / float(rope_scaling["factor"])
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return torch.view_as_real(torch.polar(torch.ones_like(freqs), freqs)).contiguous()
