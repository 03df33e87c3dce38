"""Quantized decoder on the CUDA-graph runner: the drop-in for the reference's
quantized ``Transformer`` decode path.

Mirrors ``Transformer.quantize`` / ``_ensure_quant_weights`` /
``forward`` (T = 1 decode and T > 1 chunked prefill) /
``forward_tree_verify`` / ``get_decode_runner`` (axiomlm/models/transformer.py
276-352, 822-1008, 1415-1546, 581-784, 1202-1308), over ``libaxb.so``'s
runner (replacing MPSQuantizedDecodeRunner, mps_kernels.mm:2982-3737).
"""

from __future__ import annotations

import ctypes as C
import dataclasses
import json
from typing import Any

import torch

from . import _lib as L
from . import ops
from .cache import StaticKVCache

WEIGHT_FORMATS = {
    # reference q4_rtn: MARLIN RTN values, affine (scale, bias), group 64
    "q4_rtn": (L.W_Q4T_AFFINE, 64),
    # reference q4_legacy: the same round-to-nearest G64 values in another
    # layout (pack_linear_q4_g64, quant.py:17-69), so the same q4t packs
    "q4_legacy": (L.W_Q4T_AFFINE, 64),
    # the benchmark format: symmetric, group 128, fp16 scales (4.125 bits/weight)
    "q4_g128_sym": (L.W_Q4T_SYM, 128),
    # reference q8: every projection and the lm_head Q8_G64 in its own layout
    # (transformer.py:847-855), gate_up as cat(w_gate, w_up)
    "q8": (L.W_Q8_G64, 64),
    # reference q4 / q4_k_m: affine G64 with the clip search (ops.pack_q4_mse),
    # importance-weighted as _ensure_quant_weights weighs it (transformer.py:
    # 880-884, 931-941); q4_k_m keeps w_down and the lm_head Q8_G64
    "q4": (L.W_Q4T_AFFINE, 64),
    "q4_k_m": (L.W_Q4T_AFFINE, 64),
    # 2-bit: the reference's ternary / q2_k packings (group 64, quant.py:236-381)
    # and the benchmark-only per-tensor ternary and K-quant super-blocks; every
    # projection and an untied lm_head, gate_up as cat(w_gate, w_up)
    "ternary": (L.W_TERNARY_G64, 64),
    "q2_k": (L.W_Q2_G64, 64),
    "ternary_pt": (L.W_TERNARY_PT, 0),
    "q2k": (L.W_Q2K_SB256, 256),
}
_LOWBIT_FORMATS = (L.W_TERNARY_G64, L.W_Q2_G64, L.W_TERNARY_PT, L.W_Q2K_SB256)


def _vp_array(items):
    arr = (C.c_void_p * len(items))()
    for i, t in enumerate(items):
        arr[i] = None if t is None else (t if isinstance(t, int) else t.data_ptr())
    return arr


def _scale_ref(w, keep: list):
    """What the runner takes as a projection's scale pointer: the scales
    tensor, or for a 2-bit projection the address of its axb_q2t_meta (kept
    alive in ``keep`` until the runner has copied it)."""
    if isinstance(w, ops.Q2TWeight):
        m = w.runner_meta()
        keep.append(m)
        return C.addressof(m)
    return w.scales


_WEIGHT_TYPES = {c.__name__: c for c in (ops.Q4TWeight, ops.Q8Weight, ops.Q2TWeight)}


def clip_importance(layer: dict | None, which: str, ln_f: torch.Tensor | None = None) -> torch.Tensor | None:
    """The column importance the reference's clip search gets for a
    projection in its "q4" / "q4_k_m" modes (_ensure_quant_weights,
    transformer.py:880-884, 931-941): |ln_1| for c_attn ("qkv"), none for
    c_proj ("o"), |ln_2| for gate_up ("gu"), |w_gate row| * |w_up row| for
    w_down ("down"), |ln_f| for the lm_head ("lm")."""
    if which == "lm":
        return ln_f.float().abs()
    if which == "qkv":
        return layer["ln_1"].float().abs()
    if which == "gu":
        return layer["ln_2"].float().abs()
    if which == "down":
        return layer["w_gate"].float().norm(dim=1) * layer["w_up"].float().norm(dim=1)
    return None


def packed_kind(p: torch.Tensor, s: torch.Tensor) -> str:
    """Which of the reference's packings a (words, scales) pair is, by shape
    and dtype (_ensure_quant_weights, transformer.py:849-876):
    "marlin" ((N/8, K/64, 32, 2) int32 MARLIN ladder: q4, q4_k_m, q4_rtn),
    "ternary_g64" / "q2_g64" ((N, K/4) uint8 codes with (N, K/64) scales or
    (N, K/64, 2) scale / bias pairs: ternary, q2_k), "q8_g64" ((N, K/4)
    int32: q8, and w_down / lm_head in q4_k_m), "q4_g64" ((N, K/8) int32:
    q4_legacy)."""
    if p.ndim == 4:
        return "marlin"
    if p.ndim == 2 and s.ndim >= 2:
        k64 = s.shape[1] * 64
        if p.dtype == torch.uint8 and p.shape[1] * 4 == k64:
            return "q2_g64" if s.ndim == 3 else "ternary_g64"
        if p.dtype == torch.int32 and p.shape[1] * 4 == k64:
            return "q8_g64"
        if p.dtype == torch.int32 and p.shape[1] * 8 == k64:
            return "q4_g64"
    raise NotImplementedError(f"packed weight of {p.dtype} {tuple(p.shape)} / {tuple(s.shape)}")


def packed_to_tensors(packed: dict) -> tuple[dict, dict]:
    """A packed-weight dict as flat named tensors (on the host) and string
    metadata: each weight object's type and scalar fields, and which optional
    tensors are absent."""
    tensors: dict = {}
    meta: dict = {"n_layer": str(len(packed["layers"]))}

    def put(name, v):
        if v is None:
            meta[name] = "none"
        elif isinstance(v, torch.Tensor):
            # a host copy per name (a tied lm_head shares the embedding's storage)
            tensors[name] = v.detach().to("cpu", copy=True).contiguous()
        else:
            fields = {}
            for f in dataclasses.fields(v):
                x = getattr(v, f.name)
                if isinstance(x, torch.Tensor) or x is None:
                    put(f"{name}.{f.name}", x)
                else:
                    fields[f.name] = x
            meta[name] = json.dumps({"type": type(v).__name__, **fields})

    for i, ly in enumerate(packed["layers"]):
        for k in ("qkv", "o", "gu", "down", "ln_1", "ln_2", "qkv_b"):
            put(f"layers.{i}.{k}", ly.get(k))
    lm = packed["lm_head"]
    tied = isinstance(lm, ops.Q8Weight) and lm.words.data_ptr() == packed["emb_w"].data_ptr()
    for k in ("emb_w", "emb_s", "ln_f") + (() if tied else ("lm_head",)):
        put(k, packed[k])
    if tied:  # the embedding matrix is the lm_head: stored once, shared again on load
        meta["lm_head"] = json.dumps({"tied": True, "N": lm.N, "K": lm.K})
    return tensors, meta


def read_packed(path, device="cuda") -> tuple[dict, dict]:
    """(cfg, packed dict) from a file ``QuantizedDecoder.save_packed`` wrote,
    tensors on ``device``."""
    from safetensors import safe_open

    with safe_open(str(path), framework="pt", device="cpu") as f:
        meta = f.metadata() or {}
        if meta.get("format") != QuantizedDecoder._PACKED_FORMAT:
            raise ValueError(f"{path} is not a packed-weight file of this library")
        names = set(f.keys())
        dev = torch.device(device)

        def get(name):
            if name in names:
                return f.get_tensor(name).to(dev)
            m = meta.get(name)
            if m is None or m == "none":
                return None
            d = json.loads(m)
            if d.get("tied"):
                return ops.Q8Weight(get("emb_w"), get("emb_s"), d["N"], d["K"])
            cls = _WEIGHT_TYPES[d.pop("type")]
            for fld in dataclasses.fields(cls):
                if fld.name not in d:
                    d[fld.name] = get(f"{name}.{fld.name}")
            return cls(**d)

        layers = [{k: get(f"layers.{i}.{k}") for k in ("qkv", "o", "gu", "down", "ln_1", "ln_2", "qkv_b")}
                  for i in range(int(meta["n_layer"]))]
        packed = dict(layers=layers, **{k: get(k) for k in ("emb_w", "emb_s", "ln_f")})
        packed["lm_head"] = get("lm_head")
        if isinstance(packed["lm_head"], ops.Q8Weight) and json.loads(meta["lm_head"]).get("tied"):
            packed["lm_head"] = ops.Q8Weight(packed["emb_w"], packed["emb_s"], packed["lm_head"].N,
                                             packed["lm_head"].K)
    return json.loads(meta["cfg"]), packed


class QuantizedDecoder:
    """Packed weights + ``StaticKVCache`` + the CUDA-graph runner.

    ``cfg`` keys: n_layer, d_model, n_head, n_kv_head, ffn, vocab, eps, theta,
    rope_scaling (optional).  Build with ``from_weights`` (fp32 master
    weights, packed on the GPU) or ``from_reference`` (a reference
    ``Transformer`` after ``quantize()``: its own packed tensors are relaid
    out, so MSE-clipped "q4" models are served exactly as packed).
    """

    def __init__(self, cfg: dict, packed: dict, *, kv_dtype: str = "fp16", kv_group: int = 64, max_batch: int = 1,
                 max_seq: int = 1024, max_tokens: int = 64, ring_buffer: bool = False, rope_len: int | None = None,
                 device: str | torch.device = "cuda", use_graph: bool = True, tp=None):
        # tensor parallel (``tp``: an axiomlm_b200.tp.TensorParallel): ``cfg`` is
        # the whole model's; ``packed`` holds this rank's shards
        self.tp = tp
        world = tp.world if tp is not None else 1
        self.cfg = dict(cfg)
        self.device = torch.device(device)
        d, H, Hkv = cfg["d_model"], cfg["n_head"] // world, cfg["n_kv_head"] // world
        self.head_dim = d // cfg["n_head"]
        self.max_tokens = max_tokens
        self.use_graph = use_graph
        self.packed = packed
        self.cache = StaticKVCache(max_batch, max_seq, cfg["n_layer"], Hkv, self.head_dim, device=self.device,
                                   ring_buffer=ring_buffer, cache_dtype=kv_dtype, kv_group=kv_group)
        self.rope_len = rope_len or max(max_seq, cfg.get("block_size", 0))
        self.rope = ops.rope_table(self.head_dim, self.rope_len, cfg.get("theta", 10000.0),
                                   cfg.get("rope_scaling")).to(self.device)
        lay = packed["layers"]
        wq = lay[0]["qkv"]
        lm = packed["lm_head"]
        self.vocab_local = cfg["vocab"] // world
        c = L.ModelCfg(n_layer=cfg["n_layer"], d_model=d, n_head=H, n_kv_head=Hkv, head_dim=self.head_dim,
                       ffn=cfg["ffn"] // world, vocab=self.vocab_local, eps=float(cfg["eps"]), wfmt=wq.fmt,
                       group=wq.group, tp_world=world, tp_rank=tp.rank if tp is not None else 0,
                       lm_fmt=lm.fmt, lm_group=lm.group, kv_type=L.KV_TYPES[self.cache.cache_dtype],
                       kv_group=self.cache.kv_group, max_batch=max_batch, max_seq=max_seq, max_tokens=max_tokens,
                       rope_len=self.rope_len, has_qkv_bias=int(lay[0].get("qkv_b") is not None),
                       dn_fmt=lay[0]["down"].fmt, dn_group=lay[0]["down"].group)
        self._cfg_c = c
        lib = L.load()
        nbytes = lib.axb_runner_workspace_bytes(C.byref(c))
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        kc = self.cache.k_caches
        vc = self.cache.v_caches
        ks = self.cache.k_scales or [None] * cfg["n_layer"]
        vs = self.cache.v_scales or [None] * cfg["n_layer"]
        metas: list = []
        sr = lambda w: _scale_ref(w, metas)  # noqa: E731
        self._arrays = dict(
            qkv_w=_vp_array([x["qkv"].words for x in lay]), qkv_s=_vp_array([sr(x["qkv"]) for x in lay]),
            qkv_b=_vp_array([x.get("qkv_b") for x in lay]),
            o_w=_vp_array([x["o"].words for x in lay]), o_s=_vp_array([sr(x["o"]) for x in lay]),
            gu_w=_vp_array([x["gu"].words for x in lay]), gu_s=_vp_array([sr(x["gu"]) for x in lay]),
            dn_w=_vp_array([x["down"].words for x in lay]), dn_s=_vp_array([sr(x["down"]) for x in lay]),
            ln1=_vp_array([x["ln_1"] for x in lay]), ln2=_vp_array([x["ln_2"] for x in lay]),
            k_cache=_vp_array(kc), v_cache=_vp_array(vc), k_scale=_vp_array(ks), v_scale=_vp_array(vs))
        lm_s = sr(lm)
        p = L.ModelPtrs(emb_w=packed["emb_w"].data_ptr(), emb_s=packed["emb_s"].data_ptr(), lm_w=lm.words.data_ptr(),
                        lm_s=lm_s if isinstance(lm_s, int) else lm_s.data_ptr(), ln_f=packed["ln_f"].data_ptr(), rope=self.rope.data_ptr(),
                        tp_comm=tp.comm if tp is not None else None,
                        **{k: C.cast(v, C.POINTER(C.c_void_p)) for k, v in self._arrays.items()})
        h = C.c_void_p()
        L.call("axb_runner_create", C.byref(c), C.byref(p), C.c_void_p(self.workspace.data_ptr()), nbytes, C.byref(h))
        del metas  # copied by the runner
        self._h = h

        def view(which, dtype, shape):
            off, nb = C.c_size_t(), C.c_size_t()
            L.call("axb_runner_buffer", self._h, which, C.byref(off), C.byref(nb))
            return self.workspace[off.value: off.value + nb.value].view(dtype).view(*shape)

        rows = max_batch * max_tokens
        self.tokens = view(0, torch.int32, (rows,))
        self.logits_buf = view(1, torch.float16, (rows, self.vocab_local))  # this rank's vocab rows under tp
        self.argmax_buf = view(2, torch.int32, (rows,))
        self.norm_buf = view(3, torch.float32, (rows, d))
        self.error_buf = view(4, torch.int32, (1,))
        self._last_T = 1
        self.medusa_heads = None

    # ------------------------------------------------------------ builders
    @classmethod
    def from_weights(cls, cfg: dict, weights: dict, weight_format: str = "q4_rtn", **kw) -> "QuantizedDecoder":
        tp = kw.get("tp")
        if tp is not None and tp.world > 1:
            from .tp import local_dims, shard_weights

            local_dims(cfg, tp.world)  # divisibility checks
            weights = shard_weights(cfg, weights, tp.rank, tp.world)
        return cls._from_weights(cfg, weights, weight_format, **kw)

    @classmethod
    def _from_weights(cls, cfg: dict, weights: dict, weight_format: str = "q4_rtn", **kw) -> "QuantizedDecoder":
        """Pack fp32 master weights (``tests/golden/model_weights.make_weights``
        layout) on the GPU, following ``_ensure_quant_weights`` in q4_rtn
        mode (transformer.py:822-1008): projections and an untied lm_head in
        Q4, token embeddings in Q8_G64 (also the lm_head when the embeddings are
        tied), RMSNorm weights kept fp32.  ``weight_format="q8"`` packs every
        projection and the lm_head Q8_G64 (the reference's q8 mode); "ternary",
        "q2_k", "ternary_pt" and "q2k" pack them in a 2-bit format; "q4" and
        "q4_k_m" pack with the reference's clip search, c_attn weighted by
        |ln_1|, gate_up by |ln_2|, w_down by |w_gate row| * |w_up row| and the
        lm_head by |ln_f| ("q4"), or w_down and the lm_head in Q8_G64
        ("q4_k_m")."""
        dev = torch.device(kw.get("device", "cuda"))
        fmt, group = WEIGHT_FORMATS[weight_format]
        sym = fmt == L.W_Q4T_SYM
        tied = weights.get("lm_head") is None

        def g(t):
            return t.to(dev, torch.float32)

        mse = weight_format in ("q4", "q4_k_m")

        def q8(w):
            return ops.Q8Weight(*ops.pack_q8_g64(w), w.shape[0], w.shape[1])

        def pack(w, gate_up=False, imp=None):
            if fmt == L.W_Q8_G64:
                return q8(w)
            if fmt in _LOWBIT_FORMATS:
                return ops.pack_q2t(w, fmt)
            if mse:
                return ops.pack_q4_mse(w, imp, gate_up=gate_up)
            return ops.pack_q4t(w, group, sym, gate_up=gate_up)

        layers = []
        for lw in weights["layers"]:
            dl = {k: g(lw[k]) for k in ("w_gate", "w_up", "ln_1", "ln_2")}
            gu = torch.cat([dl["w_gate"], dl["w_up"]], 0)
            b = lw.get("c_attn_b")

            def imp(which):
                return clip_importance(dl, which) if mse else None

            down = q8(g(lw["w_down"])) if weight_format == "q4_k_m" else pack(g(lw["w_down"]), imp=imp("down"))
            layers.append(dict(
                qkv=pack(g(lw["c_attn"]), imp=imp("qkv")), o=pack(g(lw["c_proj"]), imp=imp("o")),
                gu=pack(gu, gate_up=True, imp=imp("gu")), down=down, ln_1=dl["ln_1"].contiguous(),
                ln_2=dl["ln_2"].contiguous(), qkv_b=None if b is None else b.to(dev, torch.float16).contiguous()))
            del gu, dl
        emb_w, emb_s = ops.pack_q8_g64(g(weights["wte"]))
        # tied embeddings (transformer.py:842-847): the Q8_G64 embedding matrix is the lm_head
        if tied:
            lm = ops.Q8Weight(emb_w, emb_s, emb_w.shape[0], emb_w.shape[1] * 4)
        elif weight_format == "q4_k_m":
            lm = q8(g(weights["lm_head"]))
        else:
            lm = pack(g(weights["lm_head"]), imp=clip_importance(None, "lm", g(weights["ln_f"])) if mse else None)
        packed = dict(layers=layers, emb_w=emb_w, emb_s=emb_s, lm_head=lm, ln_f=g(weights["ln_f"]).contiguous())
        dec = cls(cfg, packed, **kw)
        if weights.get("medusa"):
            from .medusa import MedusaHeads

            dec.add_medusa_heads(MedusaHeads.from_weights(weights["medusa"], weight_format, device=dev))
        return dec

    @classmethod
    def from_hf(cls, model_dir, weight_format: str = "q4_rtn", max_seq_len: int | None = None,
                dtype: torch.dtype = torch.float16, **kw) -> "QuantizedDecoder":
        """A local Hugging Face checkpoint (Llama-3 / SmolLM2 / Qwen2.5; the
        reference's load_hf_safetensors, hf_importer.py:199-305), packed on
        the GPU in ``weight_format``.  ``dtype`` is the load dtype the
        reference quantizes from (fp16 by default)."""
        from .hf_import import read_hf_checkpoint

        cfg, w = read_hf_checkpoint(model_dir, dtype=dtype, max_seq_len=max_seq_len)
        return cls.from_weights(cfg, w, weight_format, **kw)

    # ------------------------------------------------------------ packed-weight cache
    _PACKED_FORMAT = "axiomlm_b200.packed/1"

    def save_packed(self, path) -> None:
        """Write the packed weights (every format, as packed) and the model
        config to one safetensors file, so a large model is packed once;
        ``load_packed`` serves it again.  Medusa heads are not included."""
        from safetensors.torch import save_file

        tensors, meta = packed_to_tensors(self.packed)
        meta["cfg"] = json.dumps(self.cfg)
        meta["format"] = self._PACKED_FORMAT
        save_file(tensors, str(path), metadata=meta)

    @classmethod
    def load_packed(cls, path, **kw) -> "QuantizedDecoder":
        """A decoder over the weights ``save_packed`` wrote (no packing)."""
        cfg, packed = read_packed(path, kw.get("device", "cuda"))
        return cls(cfg, packed, **kw)

    @classmethod
    def from_reference(cls, model: Any, **kw) -> "QuantizedDecoder":
        """Serve a reference ``Transformer`` after ``model.quantize("q4" |
        "q4_k_m" | "q4_rtn" | "q4_legacy" | "q8")``, the modes its quantized
        forward and decode runner take (transformer.py:797-799, 1227-1236):
        its own packed tensors (``_ensure_quant_weights``) are served by
        ``from_packed``."""
        mc = model.config
        qw = model._ensure_quant_weights(torch.device("cpu"))
        H = mc.n_head
        cfg = dict(n_layer=mc.n_layer, d_model=mc.n_embd, n_head=H, n_kv_head=mc.n_kv_head or H,
                   ffn=qw["hidden_dim"], vocab=mc.vocab_size, eps=mc.rms_norm_eps, theta=mc.rope_theta,
                   rope_scaling=mc.rope_scaling, block_size=mc.block_size)
        return cls.from_packed(cfg, qw, [b.ln_1.weight for b in model.transformer.h],
                               [b.ln_2.weight for b in model.transformer.h], model.transformer.ln_f.weight, **kw)

    @classmethod
    def from_packed(cls, cfg: dict, qw: dict, ln_1: list, ln_2: list, ln_f, **kw) -> "QuantizedDecoder":
        """Serve the reference's packed tensors (the dict of
        ``_ensure_quant_weights``, transformer.py:822-1008) with its RMSNorm
        weights.  Per projection, by shape: MARLIN Q4 ("q4", "q4_k_m",
        "q4_rtn") and legacy Q4_G64 ("q4_legacy") are relaid out bit-exactly
        into q4t; Q8_G64 ("q8"; w_down in "q4_k_m") and a Q8_G64 lm_head (tied
        embeddings, "q8", "q4_k_m") run on the Q8 GEMV in the reference's own
        layout."""
        dev = torch.device(kw.get("device", "cuda"))
        H, Hkv, d = cfg["n_head"], cfg["n_kv_head"], cfg["d_model"]
        hd = d // H
        qkv_dim = (H + 2 * Hkv) * hd

        def rl(p, s, n, gu=False):
            p = torch.as_tensor(p)
            s = torch.as_tensor(s)
            kind = packed_kind(p, s)
            if kind == "marlin":
                return ops.q4t_from_marlin(p.to(dev), s.to(dev), n, gate_up=gu)
            if kind in ("ternary_g64", "q2_g64"):
                fmt = L.W_Q2_G64 if kind == "q2_g64" else L.W_TERNARY_G64
                return ops.q2t_from_ref(fmt, p.to(dev).contiguous(), s.to(dev).contiguous(), None, p.shape[1] * 4)
            if kind == "q8_g64":  # kept as packed
                return ops.Q8Weight(p.to(dev).contiguous(), s.to(dev).contiguous(), n, p.shape[1] * 4)
            return ops.q4t_from_q4g64(p.to(dev).contiguous(), s.to(dev).contiguous(), n, gate_up=gu)

        def f32(w):
            return torch.as_tensor(w).detach().to(dev, torch.float32).contiguous()

        layers = []
        for i in range(cfg["n_layer"]):
            cb = torch.as_tensor(qw["c_attn_b"][i]) if qw.get("c_attn_b") is not None else torch.empty(0)
            layers.append(dict(
                qkv=rl(qw["c_attn_p"][i], qw["c_attn_s"][i], qkv_dim), o=rl(qw["c_proj_p"][i], qw["c_proj_s"][i], d),
                gu=rl(qw["gu_p"][i], qw["gu_s"][i], 2 * cfg["ffn"], True),
                down=rl(qw["wd_p"][i], qw["wd_s"][i], d),
                ln_1=f32(ln_1[i]), ln_2=f32(ln_2[i]),
                qkv_b=cb.to(dev, torch.float16) if cb.numel() > 0 else None))
        lmh_p = torch.as_tensor(qw["lmh_p"])
        packed = dict(layers=layers, emb_w=torch.as_tensor(qw["wte_p"]).to(dev),
                      emb_s=torch.as_tensor(qw["wte_sb"]).to(dev),
                      lm_head=rl(lmh_p, qw["lmh_sb"], cfg["vocab"]), ln_f=f32(ln_f))
        dec = cls(cfg, packed, **kw)
        if qw.get("medusa_packs"):
            from .medusa import MedusaHeads

            dec.add_medusa_heads(MedusaHeads.from_packs(qw["medusa_packs"], d, cfg["vocab"], device=dev))
        return dec

    # ------------------------------------------------------------ steps
    @property
    def weight_bytes(self) -> int:
        p = self.packed
        n = p["emb_w"].numel() * 0  # embedding rows are gathered, not streamed
        n += p["lm_head"].nbytes
        for x in p["layers"]:
            n += x["qkv"].nbytes + x["o"].nbytes + x["gu"].nbytes + x["down"].nbytes
        return n

    def _step(self, B, T, rope_pos, write_pos, active_len, prefix_len, masks=None, depths=None):
        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        mp = dp = None
        if masks is not None:
            ma = (C.c_uint64 * T)(*[int(m) & 0xFFFFFFFFFFFFFFFF for m in masks])
            da = (C.c_int32 * T)(*[int(x) for x in depths])
            mp, dp = C.cast(ma, C.c_void_p), C.cast(da, C.c_void_p)
        L.call("axb_runner_step", self._h, B, T, rope_pos, write_pos, active_len, prefix_len, mp, dp,
               int(self.use_graph), st)
        self._last_T = T

    def _load_tokens(self, idx: torch.Tensor):
        n = idx.numel()
        self.tokens[:n].copy_(idx.reshape(-1).to(torch.int32), non_blocking=True)

    def decode_step(self, idx: torch.Tensor) -> torch.Tensor:
        """One T = 1 step for B sequences (idx (B, 1)); returns (B, 1, V) fp16
        logits (a view of the runner's buffer, valid until the next step)."""
        B = idx.shape[0]
        seen = self.cache.total_seen_tokens[0]
        wp, active, new_seen = self.cache.next_positions(1)
        self._load_tokens(idx)
        self._step(B, 1, seen % self.rope_len, wp, active, 0)
        self.cache.advance(new_seen)
        return self.logits_buf[:B].view(B, 1, -1)

    def prefill(self, idx: torch.Tensor) -> torch.Tensor:
        """T > 1 tokens per sequence, in chunks of max_tokens, each chunk a
        causal chain over the cached prefix; returns last-token logits."""
        B, T = idx.shape
        seen = self.cache.total_seen_tokens[0]
        if seen + T > self.cache.max_seq_len:
            raise RuntimeError("prefill beyond the cache capacity (ring wrap during prefill is not supported)")
        for t0 in range(0, T, self.max_tokens):
            n = min(self.max_tokens, T - t0)
            seen = self.cache.total_seen_tokens[0]
            masks = [(1 << (u + 1)) - 1 for u in range(n)]
            self._load_tokens(idx[:, t0:t0 + n].contiguous())
            self._step(B, n, seen % self.rope_len, seen, seen + n, seen, masks, list(range(n)))
            self.cache.advance(seen + n)
        last = self.logits_buf[: B * n].view(B, n, -1)[:, -1:, :]
        return last

    def forward(self, idx: torch.Tensor, return_all_logits: bool = False) -> torch.Tensor:
        idx = idx if idx.dim() == 2 else idx.view(1, -1)
        if idx.shape[1] == 1:
            return self.decode_step(idx)
        out = self.prefill(idx)
        return out

    def forward_tree_verify(self, idx: torch.Tensor, tree_depths: list[int], tree_mask: list[int]) -> torch.Tensor:
        """transformer.py:581-784 with uint64 masks (up to 64 nodes); K/V of the
        nodes land at [seen, seen + T); the caller commits with
        ``cache.compact_tree_path``.  Returns (B, T, V) fp16 logits."""
        idx = idx if idx.dim() == 2 else idx.view(1, -1)
        B, T = idx.shape
        seen = self.cache.total_seen_tokens[0]
        wp = (seen % self.cache.max_seq_len) if (self.cache.ring_buffer or seen >= self.cache.max_seq_len) else seen
        if wp + T > self.cache.max_seq_len or seen != wp:
            raise RuntimeError(f"tree verification needs contiguous tail capacity: write_pos={wp}, T={T}")
        self._load_tokens(idx)
        self._step(B, T, seen % self.rope_len, wp, seen + T, seen, tree_mask, tree_depths)
        return self.logits_buf[: B * T].view(B, T, -1)

    def forward_tree_verify_device(self, T: int, tree_depths: list[int], tree_mask: list[int]) -> torch.Tensor:
        """forward_tree_verify over the T tokens already in the runner's token
        buffer (``self.tokens``, written on the device by the Medusa draft)."""
        seen = self.cache.total_seen_tokens[0]
        wp = (seen % self.cache.max_seq_len) if (self.cache.ring_buffer or seen >= self.cache.max_seq_len) else seen
        if wp + T > self.cache.max_seq_len or seen != wp:
            raise RuntimeError(f"tree verification needs contiguous tail capacity: write_pos={wp}, T={T}")
        self._step(1, T, seen % self.rope_len, wp, seen + T, seen, tree_mask, tree_depths)
        return self.logits_buf[:T].view(1, T, -1)

    def compact_device(self, write_pos: int, result: torch.Tensor):
        """compact_tree_path with the accepted nodes and their count taken from
        a device tree-walk result block (no host round trip)."""
        c = self.cache
        cache = c.cache
        L_, two, Bm, H, S, W = cache.shape
        ng = 0 if c.scales is None else c.scales.shape[-1]
        L.call("axb_compact_kv_dev", C.c_void_p(cache.data_ptr()), ops._p(c.scales), L_, Bm, H, S,
               W * cache.element_size(), ng, int(write_pos), C.c_void_p(result.data_ptr() + 4 * L.TREE_RESULT_HDR),
               C.c_void_p(result.data_ptr()), min(L.TREE_MAX_NODES, S), ops._stream())

    # ------------------------------------------------------------ Medusa
    def add_medusa_heads(self, heads):
        """Attach quantized Medusa heads (an ``axiomlm_b200.medusa.MedusaHeads``),
        as Transformer.add_medusa_heads + quantize do (transformer.py:386-412)."""
        if heads.d != self.cfg["d_model"] or heads.vocab != self.vocab_local:
            raise ValueError("Medusa heads must map d_model -> vocab")
        if self.tp is not None and self.tp.world > 1:
            raise NotImplementedError("Medusa heads under tensor parallelism")
        self.medusa_heads = heads
        return self

    def forward_with_medusa(self, idx: torch.Tensor, kv_caches: Any = None, return_all_logits: bool = False,
                            return_medusa: bool = True):
        """transformer.py:447-520 (its decode-runner branch): the T tokens of
        one sequence as a causal chain, the cache counters moved past them,
        and the Medusa heads on the final-norm rows.  Returns (logits (1, T or
        1, V), per-head logits, ``kv_caches``); with T > 1 only the last
        position unless ``return_all_logits``."""
        idx = idx if idx.dim() == 2 else idx.view(1, -1)
        B, T = idx.shape
        if B != 1:
            raise ValueError("forward_with_medusa serves one sequence (as the reference's runner does)")
        seen = self.cache.total_seen_tokens[0]
        logits = self.forward_tree_verify(idx, list(range(T)), [(1 << (i + 1)) - 1 for i in range(T)])
        self.cache.advance(seen + T)
        x_norm = self.get_last_norm(T)
        if T > 1 and not return_all_logits:
            logits, x_norm = logits[:, -1:], x_norm[:, -1:]
        med = self.eval_medusa_heads(x_norm) if return_medusa and self.medusa_heads is not None else []
        return logits, med, kv_caches

    def get_decode_runner(self, cache: Any = None) -> "QuantizedDecoder":
        """transformer.py:1202: the decode runner bound to the cache; here the
        decoder is its own runner (bound to ``self.cache``)."""
        if cache is not None and cache is not self.cache:
            raise ValueError("this decoder's runner is bound to its own cache (dec.cache)")
        return self

    def eval_medusa_heads(self, x_norm: torch.Tensor) -> list[torch.Tensor]:
        """transformer.py:414-445: the heads' logits on final-norm rows."""
        if self.medusa_heads is None:
            return []
        return self.medusa_heads(x_norm)

    def get_last_norm(self, T: int | None = None) -> torch.Tensor:
        """Final-norm hidden states (fp32) of the last tree/prefill step."""
        T = T or self._last_T
        return self.norm_buf[:T].view(1, T, -1)

    def status(self) -> int:
        """The runner's error word (synchronizes): 0, or the status of the first
        problem a step met (AXB_EINVAL: an out-of-vocabulary token id,
        AXB_ETIMEOUT: a bounded device-side wait ran out)."""
        return int(self.error_buf.item())

    @property
    def uses_step_kernel(self) -> bool:
        """True when decode steps run as one persistent kernel launch."""
        return bool(L.load().axb_runner_uses_step_kernel(self._h))

    def argmax(self, rows: int) -> torch.Tensor:
        return self.argmax_buf[:rows]

    @torch.no_grad()
    def generate_greedy(self, prompt: torch.Tensor, n_new: int) -> list[int]:
        prompt = prompt.to(self.device).view(1, -1)
        logits = self.prefill(prompt)
        T = prompt.shape[1] - (prompt.shape[1] - 1) // self.max_tokens * self.max_tokens
        tok = self.argmax_buf[T - 1: T].clone()
        out = [tok]
        for _ in range(n_new - 1):
            self.decode_step(tok.view(1, 1))
            tok = self.argmax_buf[:1].clone()
            out.append(tok)
        return [int(t) for t in torch.cat(out).tolist()]

    def close(self):
        if getattr(self, "_h", None):
            L.call("axb_runner_destroy", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
