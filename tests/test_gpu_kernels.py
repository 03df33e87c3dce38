"""CUDA kernels (through the C ABI) vs the oracle and the reference fixtures.

Bit-exact: every unpack / dequant / pack / relayout and the KV-cache
quantization.  Tolerance: GEMV and attention outputs against an fp32 torch
evaluation of the same (dequantized) operands, relative error < 2e-3 of the
output's max magnitude (the north-star layer tolerance).
"""

import os

import numpy as np
import pytest
import torch

import oracle as O
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


def _g(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="module")
def ax():
    from axiomlm_b200 import _lib, ops

    _lib.load()
    assert _lib.load().axb_check_device() == 0, "not an sm_100 device"
    return ops


def _cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _bits(t):
    return t.cpu().numpy().view(np.uint16) if t.dtype == torch.float16 else t.cpu().numpy()


def _rel(a, b):
    a = a.float()
    b = b.float()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-6))


# ------------------------------------------------------------------ formats

def test_marlin_dequant_bit_exact(ax):
    g = _g("quant.npz")
    for pfx in ("q4m", "q4m_clip"):
        dq = ax.dequantize_q4_marlin(_cu(g[f"{pfx}_w"]), _cu(g[f"{pfx}_sb"]), 256, 40)
        assert np.array_equal(_bits(dq), g[f"{pfx}_dq"].view(np.uint16))


@pytest.mark.parametrize("gate_up", [False, True])
def test_relayout_from_marlin_bit_exact(ax, gate_up):
    g = _g("quant.npz")
    W = ax.q4t_from_marlin(_cu(g["q4m_clip_w"]), _cu(g["q4m_clip_sb"]), 32 if gate_up else 40, gate_up=gate_up)
    ow, osc = O.q4t_from_marlin(g["q4m_clip_w"], g["q4m_clip_sb"], 32 if gate_up else 40, gate_up=gate_up)
    assert np.array_equal(W.words.cpu().numpy(), ow.reshape(-1))
    assert np.array_equal(_bits(W.scales), osc.reshape(-1).view(np.uint16))
    if not gate_up:
        # values are the reference's dequantized weights, bit for bit
        assert np.array_equal(_bits(W.dequant()), g["q4m_clip_dq"].view(np.uint16))


def test_relayout_from_legacy_q4g64_bit_exact(ax):
    """q4_legacy packs (pack_linear_q4_g64, quant.py:17-69): the relayout keeps
    the reference's codes, scales and biases, so the q4t dequant equals
    dequantize_q4_g64 bit for bit; the GEMV (qmv_q4_g64) agrees with an fp32
    matmul of those values, and the gate/up interleave keeps every row."""
    g = _g("quant.npz")
    W = ax.q4t_from_q4g64(_cu(g["q4g_w"]), _cu(g["q4g_sb"]))
    assert np.array_equal(_bits(W.dequant()), g["q4g_dq"].view(np.uint16))
    x = _cu(g["x"]).half()
    ref = x.float() @ torch.from_numpy(g["q4g_dq"]).cuda().float().t()
    assert _rel(ax.qmv_q4_g64(x, _cu(g["q4g_w"]), _cu(g["q4g_sb"])), ref) < REL_TOL
    # gate/up interleave of a seeded 2F x K legacy pack (rows g of a tile = gate j, g + 8 = up j)
    rng = np.random.default_rng(5)
    wp, sb = O.pack_q4_g64(rng.standard_normal((64, 256), dtype=np.float32) * 0.02)
    Wg = ax.q4t_from_q4g64(_cu(wp), _cu(sb), gate_up=True)
    Wp = ax.q4t_from_q4g64(_cu(wp), _cu(sb))
    dq_g, dq_p = Wg.dequant().float().cpu(), Wp.dequant().float().cpu()
    assert torch.equal(torch.sort(dq_g, 0).values, torch.sort(dq_p, 0).values)


@pytest.mark.parametrize("group,sym,gu", [(64, False, False), (128, True, False), (128, True, True), (64, True, True),
                                          (128, False, False)])
def test_q4t_pack_matches_oracle(ax, group, sym, gu):
    rng = np.random.default_rng(group + 2 * sym + 4 * gu)
    N, K = (48, 512) if gu else (40, 384 if group == 64 else 512)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[1, 5] = 0.4
    w[2, :group] = 0.0
    W = ax.pack_q4t(_cu(w), group, sym, gate_up=gu)
    ow, osc = O.q4t_pack(w, group, sym, gate_up=gu)
    assert np.array_equal(W.words.cpu().numpy(), ow.reshape(-1))
    assert np.array_equal(_bits(W.scales), osc.reshape(-1).view(np.uint16))
    dq = O.q4t_dequant(ow, osc, K, group, sym, N, gate_up=gu)
    assert np.array_equal(_bits(W.dequant()), dq.view(np.uint16))
    if not sym and group == 64 and not gu:
        # affine G64 RTN == the reference's q4_rtn MARLIN values
        wm, sb = O.pack_q4_marlin_rtn(w)
        assert np.array_equal(dq.view(np.uint16), O.dequant_q4_marlin(wm, sb, K, N).view(np.uint16))


def test_q8_pack_and_rows_bit_exact(ax):
    g = _g("quant.npz")
    p, s = ax.pack_q8_g64(_cu(g["W"]))
    assert np.array_equal(p.cpu().numpy(), g["q8_w"]) and np.array_equal(_bits(s), g["q8_sb"].view(np.uint16))
    rows = ax.dequant_q8_rows(_cu(g["q8_rows_idx"]), p, s)
    assert np.array_equal(_bits(rows), g["q8_rows"].view(np.uint16))


def test_ternary_and_q2_dequant_bit_exact(ax):
    g = _g("quant.npz")
    t = ax.dequantize_ternary(_cu(g["ter_w"]), _cu(g["ter_s"]), 256)
    assert np.array_equal(_bits(t), g["ter_dq"].view(np.uint16))
    q = ax.dequantize_q2_k(_cu(g["q2_w"]), _cu(g["q2_sb"]), 256)
    assert np.array_equal(_bits(q), g["q2_dq"].view(np.uint16))
    # per-tensor ternary (the format of the GEMV sweep's ternary case)
    w = (np.random.default_rng(3).standard_normal((16, 128)) * 0.02).astype(np.float32)
    pw, ps = O.ternary_pt_pack(w)
    t = ax.dequantize_ternary(_cu(pw), _cu(ps), 128)
    assert np.array_equal(_bits(t), O.ternary_pt_dequant(pw, ps).view(np.uint16))


# ------------------------------------------------------------------ KV quant

@pytest.mark.parametrize("hd", [64, 128])
def test_kv_quant_fp16_inputs_bit_exact(ax, hd):
    g = _g("kv.npz")
    x = _cu(g[f"x{hd}"])
    q, s = ax.quantize_kv(x, "fp8")
    ref_q, ref_s = g[f"fp8_q{hd}"], g[f"fp8_s{hd}"]
    ok = ref_s.view(np.uint16) != 0  # zero-scale groups: the reference stores NaN codes, we store zeros
    assert np.array_equal(_bits(s), ref_s.view(np.uint16))
    qg = q.cpu().numpy().reshape(*ref_s.shape, -1)
    assert np.array_equal(qg[ok], ref_q.reshape(*ref_s.shape, -1)[ok])
    assert np.array_equal(_bits(ax.dequantize_kv(q, s, "fp8")), g[f"fp8_dq{hd}"].view(np.uint16))
    q, s = ax.quantize_kv(x, "int4")
    assert np.array_equal(q.cpu().numpy(), g[f"i4_q{hd}"]) and np.array_equal(_bits(s), g[f"i4_s{hd}"].view(np.uint16))
    assert np.array_equal(_bits(ax.dequantize_kv(q, s, "int4")), g[f"i4_dq{hd}"].view(np.uint16))


@pytest.mark.parametrize("hd", [64, 128])
def test_kv_quant_fp32_inputs_bit_exact(ax, hd):
    g = _g("kv.npz")
    x = _cu(g[f"x32_{hd}"])
    q, s = ax.quantize_kv(x, "fp8")
    assert np.array_equal(q.cpu().numpy(), g[f"fp8_q32_{hd}"]) and np.array_equal(_bits(s), g[f"fp8_s32_{hd}"].view(np.uint16))
    q, s = ax.quantize_kv(x, "int4")
    assert np.array_equal(q.cpu().numpy(), g[f"i4_q32_{hd}"]) and np.array_equal(_bits(s), g[f"i4_s32_{hd}"].view(np.uint16))


@pytest.mark.parametrize("kv,group", [("fp8", 128), ("int4", 32)])
def test_kv_quant_baseline_granularities(ax, kv, group):
    x = (np.random.default_rng(group).standard_normal((3, 4, 7, 128)) * 1.3).astype(np.float32)
    q, s = ax.quantize_kv(_cu(x), kv, group)
    oq, os_ = (O.quant_kv_fp8(x, group) if kv == "fp8" else O.quant_kv_int4(x, group))
    assert np.array_equal(q.cpu().numpy(), oq) and np.array_equal(_bits(s), os_.view(np.uint16))
    dq = ax.dequantize_kv(q, s, kv, 128)
    odq = O.dequant_kv_fp8(oq, os_, group) if kv == "fp8" else O.dequant_kv_int4(oq, os_, group)
    assert np.array_equal(_bits(dq), odq.view(np.uint16))


def test_kv_quant_all_zero_group_finite(ax):
    x = torch.zeros(2, 128, dtype=torch.float16, device="cuda")
    x[1, 64:] = 1.0
    q, s = ax.quantize_kv(x, "fp8")
    dq = ax.dequantize_kv(q, s, "fp8")
    assert torch.isfinite(dq).all() and (dq[0] == 0).all() and (dq[1, 64:] == 1).all()


# ------------------------------------------------------------------ GEMV

def _torch_ref_gemv(x, w_dq, bias=None):
    y = x.float() @ w_dq.float().t()
    if bias is not None:
        y = y + bias.float()
    return y


def test_gemv_matches_reference_fixture(ax):
    g = _g("quant.npz")
    y = ax.qmv_q4_marlin_mps(_cu(g["x"]), _cu(g["q4m_w"]), _cu(g["q4m_sb"]), 40)
    assert _rel(y, torch.from_numpy(g["q4m_y"]).cuda()) < REL_TOL


@pytest.mark.parametrize("M", [1, 2, 5, 8, 16, 19, 32, 64])
@pytest.mark.parametrize("fmt", ["sym128", "aff64"])
def test_gemv_sweep(ax, M, fmt):
    torch.manual_seed(M)
    N, K = 2003, 1024
    w = torch.randn(N, K, device="cuda") * 0.02
    w[7, 3] = 1.0  # outlier row
    W = ax.pack_q4t(w, 128 if fmt == "sym128" else 64, fmt == "sym128")
    x = torch.randn(M, K, device="cuda").half()
    y = ax.qgemm(x, W)
    ref = _torch_ref_gemv(x, W.dequant())
    assert y.shape == (M, N)
    assert _rel(y, ref) < REL_TOL


def test_gemv_big_shapes_and_determinism(ax):
    torch.manual_seed(0)
    # every 8B decode shape at M = 1: QKV, o, down, gate_up and the lm_head
    for N, K in [(4096, 4096), (6144, 4096), (4096, 14336), (512, 14336), (28672, 4096), (128256, 4096)]:
        w = torch.randn(N, K, device="cuda") * 0.02
        W = ax.pack_q4t(w, 128, True)
        x = torch.randn(1, K, device="cuda").half()
        y1 = ax.qgemm(x, W)
        y2 = ax.qgemm(x, W)
        assert torch.equal(y1, y2)  # fixed-order split-K reduction
        assert _rel(y1, _torch_ref_gemv(x, W.dequant())) < REL_TOL


@pytest.mark.parametrize("N,K,M", [(40, 256, 3), (32000, 768, 1), (32000, 768, 5), (1000, 4096, 12)])
def test_q8_g64_gemv(ax, N, K, M):
    """qmv_q8_g64 (quant.py:201-233): the reference fixture's Q8 pack at its
    own size, then larger seeded packs (the tied lm_head of the reference's
    CPU-runnable tiny model among them), against an fp32 matmul of the oracle's
    dequantized weights (dequantize_q8_g64 values, pinned to the fixture)."""
    g = np.load(os.path.join(GOLDEN, "quant.npz"))
    if (N, K) == (40, 256):
        wp, sb = g["q8_w"], g["q8_sb"]
        assert np.array_equal(O.dequant_q8_g64(wp, sb, K), g["q8_dq"])
        x = torch.from_numpy(g["x"]).cuda().half()
    else:
        torch.manual_seed(N + K + M)
        wp, sb = O.pack_q8_g64(np.random.default_rng(N + M).standard_normal((N, K), dtype=np.float32) * 0.02)
        x = torch.randn(M, K, device="cuda").half()
    y = ax.qmv_q8_g64(x, torch.from_numpy(np.ascontiguousarray(wp)).cuda(), torch.from_numpy(sb).cuda())
    dq = torch.from_numpy(O.dequant_q8_g64(wp, sb, K)).cuda().float()
    ref = x.float() @ dq.t()
    assert y.shape == (M, N)
    assert _rel(y, ref) < REL_TOL


def test_gemv_epilogues(ax):
    torch.manual_seed(1)
    F, K = 512, 256
    gate = torch.randn(F, K, device="cuda") * 0.05
    up = torch.randn(F, K, device="cuda") * 0.05
    W = ax.pack_q4t(torch.cat([gate, up], 0), 64, False, gate_up=True)
    x = torch.randn(3, K, device="cuda").half()
    sw = ax.qgemm(x, W, epilogue=2)
    dq = W.dequant()
    gu = _torch_ref_gemv(x, dq).half().float()
    ref = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
    assert sw.shape == (3, F) and _rel(sw, ref) < REL_TOL
    # residual: x_res = fp16(x_res + fp16(W h))
    Wd = ax.pack_q4t(torch.randn(K, F, device="cuda") * 0.05, 128, True)
    res = torch.randn(3, K, device="cuda").half()
    exp = (res.float() + _torch_ref_gemv(sw, Wd.dequant()).half().float()).half()
    out = res.clone()
    ax.qgemm(sw, Wd, epilogue=1, out=out)
    assert _rel(out, exp) < REL_TOL


def test_gemv_fused_rmsnorm(ax):
    torch.manual_seed(2)
    K, N = 768, 2304
    W = ax.pack_q4t(torch.randn(N, K, device="cuda") * 0.02, 64, False)
    x = (torch.randn(4, K, device="cuda") * 3).half()
    nw = 1 + 0.1 * torch.randn(K, device="cuda")
    y = ax.qgemm(x, W, norm_w=nw, eps=1e-5)
    h = O.rmsnorm(x.cpu(), nw.cpu(), 1e-5).half().cuda()
    assert _rel(y, _torch_ref_gemv(h, W.dequant())) < REL_TOL
    assert torch.equal(ax.rmsnorm_infer_mps(x, nw, 1e-5).cpu(), h.cpu()) or _rel(ax.rmsnorm_infer_mps(x, nw, 1e-5), h) < 1e-3


# ------------------------------------------------------------------ attention

def test_decode_attention_matches_reference_fixture(ax):
    g = _g("attn.npz")
    q = _cu(g["q"])
    for kv, kc, vc, ks, vs, ref in [("fp16", "k", "v", None, None, "dec_fp16"),
                                    ("fp8", "kq8", "vq8", "ks8", "vs8", "dec_fp8"),
                                    ("int4", "kq4", "vq4", "ks4", "vs4", "dec_int4")]:
        out = ax.gqa_flash_decode_mps(q, _cu(g[kc]), _cu(g[vc]), 33, 0, None if ks is None else _cu(g[ks]),
                                      None if vs is None else _cu(g[vs]), kv)
        assert _rel(out, _cu(g[ref])) < REL_TOL, kv


@pytest.mark.parametrize("hd,Hq,Hkv,S,active", [(128, 32, 8, 4096, 4096), (64, 12, 12, 300, 257),
                                                 (128, 28, 4, 1000, 999), (64, 9, 3, 100, 1)])
@pytest.mark.parametrize("kv", ["fp16", "fp8", "int4", "fp8_head", "int4_g32"])
def test_decode_attention_vs_oracle(ax, hd, Hq, Hkv, S, active, kv):
    """Split-K decode attention against the oracle's SDPA over the cache the
    oracle's own quantizer produced: the reference formats (group 64) and the
    benchmark variants (one FP8 scale per (token, head); INT4 groups of 32)."""
    torch.manual_seed(hd + S)
    B = 2
    k = torch.randn(B, Hkv, S, hd, device="cuda").half()
    v = torch.randn(B, Hkv, S, hd, device="cuda").half()
    q = torch.randn(B, Hq, 1, hd, device="cuda")
    kvt, group = {"fp16": ("fp16", 64), "fp8": ("fp8", 64), "int4": ("int4", 64), "fp8_head": ("fp8", hd),
                  "int4_g32": ("int4", 32)}[kv]
    if kvt == "fp16":
        kc, vc, ks, vs = k, v, None, None
        kd, vd = k.float().cpu(), v.float().cpu()
    else:
        qf, dqf = (O.quant_kv_fp8, O.dequant_kv_fp8) if kvt == "fp8" else (O.quant_kv_int4, O.dequant_kv_int4)
        kq, ksc = qf(k.cpu().numpy(), group)
        vq, vsc = qf(v.cpu().numpy(), group)
        kc, ks, vc, vs = (torch.from_numpy(t).cuda() for t in (kq, ksc, vq, vsc))
        # the device quantizer writes the same codes and scales
        kc2, ks2 = ax.quantize_kv(k, kvt, group)
        assert torch.equal(kc2, kc) and torch.equal(ks2, ks), kv
        kd = torch.from_numpy(dqf(kq, ksc, group)).float()
        vd = torch.from_numpy(dqf(vq, vsc, group)).float()
        kv = kvt
    ref = O.attention_decode(q.cpu(), kd, vd, active)
    for splits in (0, 1, 7):
        out = ax._attention(q, kc, vc, ks, vs, kv, active_len=active, num_splits=splits)
        assert _rel(out.view(B, Hq, hd).cpu(), ref.view(B, Hq, hd)) < REL_TOL


def test_tree_attention_matches_reference_fixture(ax):
    g = _g("attn.npz")
    out = ax.gqa_tree_verify_mps(_cu(g["tq"]), _cu(g["k"]), _cu(g["v"]), g["tmask"].tolist(), 30, 30, 8)
    assert _rel(out, _cu(g["tree_fp16"])) < REL_TOL


@pytest.mark.parametrize("T", [1, 17, 64])
@pytest.mark.parametrize("kv", ["fp16", "fp8"])
def test_tree_attention_uint64_masks_vs_oracle(ax, T, kv):
    rng = np.random.default_rng(T)
    Hq, Hkv, hd, S, prefix = 16, 4, 128, 256, 150
    masks = [1]
    for u in range(1, T):
        masks.append(masks[int(rng.integers(0, u))] | (1 << u))
    k = torch.randn(1, Hkv, S, hd, device="cuda").half()
    v = torch.randn(1, Hkv, S, hd, device="cuda").half()
    q = torch.randn(1, T, Hq * hd, device="cuda")
    if kv == "fp16":
        kc, vc, ks, vs, kd, vd = k, v, None, None, k, v
    else:
        kc, ks = ax.quantize_kv(k, kv)
        vc, vs = ax.quantize_kv(v, kv)
        kd, vd = ax.dequantize_kv(kc, ks, kv, hd), ax.dequantize_kv(vc, vs, kv, hd)
    out = ax.gqa_tree_verify_mps(q, kc, vc, masks, prefix, prefix, Hq, k_scales=ks, v_scales=vs, kv_dtype=kv)
    q4 = q.view(1, T, Hq, hd).transpose(1, 2).cpu()
    ref = O.attention_tree(q4, kd.float().cpu(), vd.float().cpu(), masks, prefix, prefix)
    assert _rel(out.view(T, Hq * hd).cpu(), ref.transpose(1, 2).reshape(T, -1)) < REL_TOL


@pytest.mark.parametrize("hd,kv,group,Hq,Hkv,T,write_pos", [
    (64, "fp8", 64, 8, 8, 33, 150),      # MHA, head_dim 64
    (128, "fp8", 128, 32, 8, 64, 150),   # one scale per (token, head)
    (128, "int4", 32, 16, 2, 20, 200),   # 8:1 GQA, G32, tree slots apart from the prefix
    (128, "int4", 64, 16, 4, 5, 150),
    (64, "fp16", 64, 4, 1, 64, 180),     # 4:1 GQA over one KV head
])
def test_tree_attention_formats_vs_oracle(ax, hd, kv, group, Hq, Hkv, T, write_pos):
    """Tensor-core tree attention over every cache format, group size, GQA
    ratio and head size, with the tree's slots elsewhere in the cache."""
    rng = np.random.default_rng(T + hd)
    S, prefix = 256, 150
    masks = [1]
    for u in range(1, T):
        masks.append(masks[int(rng.integers(0, u))] | (1 << u))
    g = torch.Generator(device="cuda").manual_seed(T)
    k = torch.randn(1, Hkv, S, hd, device="cuda", generator=g).half()
    v = (torch.randn(1, Hkv, S, hd, device="cuda", generator=g) * 3).half()
    q = torch.randn(1, T, Hq * hd, device="cuda", generator=g)
    if kv == "fp16":
        kc, vc, ks, vs, kd, vd = k, v, None, None, k, v
    else:
        kc, ks = ax.quantize_kv(k, kv, group)
        vc, vs = ax.quantize_kv(v, kv, group)
        kd, vd = ax.dequantize_kv(kc, ks, kv, hd), ax.dequantize_kv(vc, vs, kv, hd)
    out = ax.gqa_tree_verify_mps(q, kc, vc, masks, prefix, write_pos, Hq, k_scales=ks, v_scales=vs, kv_dtype=kv)
    q4 = q.view(1, T, Hq, hd).transpose(1, 2).cpu()
    ref = O.attention_tree(q4, kd.float().cpu(), vd.float().cpu(), masks, prefix, write_pos)
    assert _rel(out.view(T, Hq * hd).cpu(), ref.transpose(1, 2).reshape(T, -1)) < REL_TOL


# ------------------------------------------------------------------ KV write / compaction

@pytest.mark.parametrize("kv,group", [("fp16", 64), ("fp8", 64), ("int4", 64), ("fp8", 128), ("int4", 32)])
def test_rope_kv_write_vs_oracle(ax, kv, group):
    from axiomlm_b200 import _lib as L
    import ctypes as C

    torch.manual_seed(5)
    Hq, Hkv, hd, S, B, T = 8, 2, 128, 64, 2, 3
    qkv = (torch.randn(B * T, (Hq + 2 * Hkv) * hd, device="cuda") * 0.7).half()
    rope = ax.rope_table(hd, 128).cuda()
    if kv == "fp16":
        kc = torch.zeros(B, Hkv, S, hd, dtype=torch.float16, device="cuda")
    else:
        kc = torch.zeros(B, Hkv, S, hd if kv == "fp8" else hd // 2, dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.zeros(B, Hkv, S, hd // group, dtype=torch.float16, device="cuda")
    vs = torch.zeros_like(ks)
    q_out = torch.empty(B * T, Hq * hd, device="cuda")
    rope_pos, wp = 37, 10
    d = L.KvWriteDesc(kv_type=L.KV_TYPES[kv], kv_group=group, B=B, T=T, n_head=Hq, n_kv_head=Hkv, head_dim=hd,
                      max_seq=S, max_batch=B, qkv=qkv.data_ptr(), bias=None, rope=rope.data_ptr(),
                      rope_len=rope.shape[0], rope_pos=rope_pos, depths=None, write_pos=wp, q_out=q_out.data_ptr(),
                      dev_params=None, k_cache=kc.data_ptr(), v_cache=vc.data_ptr(),
                      k_scale=ks.data_ptr() if kv != "fp16" else None, v_scale=vs.data_ptr() if kv != "fp16" else None,
                      k_is_fp32=1)
    L.call("axb_rope_kv_write", C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    # oracle: transformer.py:1105-1127 in fp32, then the fp32 quantization rule
    x = qkv.cpu().view(B, T, -1).float()
    f = torch.view_as_complex(rope[rope_pos:rope_pos + T].cpu().contiguous()).view(1, 1, T, -1)
    qh = x[..., :Hq * hd].view(B, T, Hq, hd).transpose(1, 2)
    kh = x[..., Hq * hd:(Hq + Hkv) * hd].view(B, T, Hkv, hd).transpose(1, 2)
    vh = x[..., (Hq + Hkv) * hd:].view(B, T, Hkv, hd).transpose(1, 2)
    qr = O.axb_oracle._rope_apply(qh, f)
    kr = O.axb_oracle._rope_apply(kh, f)
    assert torch.equal(q_out.cpu().view(B, T, Hq, hd).transpose(1, 2), qr)
    sl = slice(wp, wp + T)
    if kv == "fp16":
        assert torch.equal(kc[:, :, sl].cpu(), kr.half()) and torch.equal(vc[:, :, sl].cpu(), vh.half())
    else:
        fq = (lambda a: O.quant_kv_fp8(a, group)) if kv == "fp8" else (lambda a: O.quant_kv_int4(a, group))
        okq, oks = fq(kr.numpy())
        ovq, ovs = fq(vh.numpy())
        assert np.array_equal(kc[:, :, sl].cpu().numpy(), okq) and np.array_equal(_bits(ks[:, :, sl]), oks.view(np.uint16))
        assert np.array_equal(vc[:, :, sl].cpu().numpy(), ovq) and np.array_equal(_bits(vs[:, :, sl]), ovs.view(np.uint16))


def test_compact_tree_path_vs_oracle(ax):
    from axiomlm_b200.cache import StaticKVCache

    c = StaticKVCache(2, 40, 3, 2, 64, cache_dtype="fp8")
    c.cache.copy_(torch.randint(0, 255, c.cache.shape, dtype=torch.uint8))
    c.scales.copy_(torch.randn(c.scales.shape).half())
    ref_c, ref_s = c.cache.cpu().numpy().copy(), c.scales.cpu().numpy().copy()
    acc = [0, 2, 5, 6]
    c.compact_tree_path(30, acc, 34)
    src = [(30 + a) % 40 for a in acc]
    dst = [(30 + m) % 40 for m in range(len(acc))]
    st = ref_c[:, :, :, :, src].copy()
    ref_c[:, :, :, :, dst] = st
    ss = ref_s[:, :, :, :, src].copy()
    ref_s[:, :, :, :, dst] = ss
    assert np.array_equal(c.cache.cpu().numpy(), ref_c) and np.array_equal(c.scales.cpu().numpy(), ref_s)
    assert c.total_seen_tokens == [34] * 3


def test_argmax_ties_lowest_index(ax):
    x = torch.zeros(3, 1000, dtype=torch.float16, device="cuda")
    x[0, 17] = 5
    x[0, 900] = 5
    x[1, 999] = 1
    out = ax.argmax_last_token_mps(x)
    assert out.tolist() == [17, 999, 0]
