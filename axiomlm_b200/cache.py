"""``StaticKVCache`` on CUDA (mirror of axiomlm/engine/paged_cache.py:122-462).

Same constructor, buffers and bookkeeping fields as the reference
(``cache`` (L, 2, B, Hkv, S, hd | hd/2), ``scales`` (L, 2, B, Hkv, S, G),
``k_caches``/``v_caches``/``k_scales``/``v_scales`` per-layer views,
``total_seen_tokens``, ``layer_seq_lens``, ``ring_buffer``), plus one B200
extension: ``kv_group`` (elements per fp16 scale; 64 = the reference,
``head_dim`` = one scale per (token, head), 32 = group-32 INT4).
The cache is written by the CUDA decode runner, or through ``update`` (the
reference's per-layer write that returns the active window);
``compact_tree_path`` runs the compaction kernel.
"""

from __future__ import annotations

import torch

from . import ops


class StaticKVCache:
    def __init__(self, max_batch_size: int, max_seq_len: int, n_layer: int, n_kv_head: int, head_dim: int,
                 dtype: torch.dtype = torch.float16, device: torch.device | str | None = None,
                 ring_buffer: bool = False, cache_dtype: str = "fp16", kv_group: int = 64):
        device = torch.device(device if device is not None else "cuda")
        if device.type != "cuda":
            raise RuntimeError("axiomlm_b200.StaticKVCache lives in CUDA memory")
        self.max_batch_size = max_batch_size
        self.max_seq_len = max_seq_len
        self.n_layer = n_layer
        self.n_kv_head = n_kv_head
        self.head_dim = head_dim
        self.ring_buffer = ring_buffer
        self.cache_dtype = cache_dtype.lower()
        if self.cache_dtype not in ("fp16", "fp8", "int4"):
            raise ValueError(f"cache_dtype must be fp16, fp8 or int4, got {cache_dtype}")
        self.kv_group = kv_group if self.cache_dtype != "fp16" else 64
        if self.cache_dtype != "fp16" and head_dim % self.kv_group:
            raise ValueError(f"kv_group {kv_group} must divide head_dim {head_dim}")
        self.num_groups = max(1, head_dim // self.kv_group)
        shape = (n_layer, 2, max_batch_size, n_kv_head, max_seq_len)
        if self.cache_dtype == "fp16":
            self.cache = torch.zeros((*shape, head_dim), dtype=dtype, device=device)
            self.scales = None
        else:
            width = head_dim if self.cache_dtype == "fp8" else head_dim // 2
            self.cache = torch.zeros((*shape, width), dtype=torch.uint8, device=device)
            self.scales = torch.zeros((*shape, self.num_groups), dtype=torch.float16, device=device)
        self.k_caches = [self.cache[i, 0] for i in range(n_layer)]
        self.v_caches = [self.cache[i, 1] for i in range(n_layer)]
        self.k_scales = None if self.scales is None else [self.scales[i, 0] for i in range(n_layer)]
        self.v_scales = None if self.scales is None else [self.scales[i, 1] for i in range(n_layer)]
        self.layer_seq_lens = [0] * n_layer
        self.total_seen_tokens = [0] * n_layer

    def get_memory_bytes(self) -> int:
        total = self.cache.numel() * self.cache.element_size()
        if self.scales is not None:
            total += self.scales.numel() * self.scales.element_size()
        return total

    @property
    def seq_len(self) -> int:
        return self.total_seen_tokens[0]

    def reset(self):
        for i in range(self.n_layer):
            self.layer_seq_lens[i] = 0
            self.total_seen_tokens[i] = 0

    def next_positions(self, T: int) -> tuple[int, int, int]:
        """(write_pos, active_len, new_seen) for T new tokens, as the runner
        path computes them (transformer.py:1451-1461)."""
        seen = self.total_seen_tokens[0]
        S = self.max_seq_len
        write_pos = (seen % S) if (self.ring_buffer or seen >= S) else seen
        new_seen = seen + T
        return write_pos, min(new_seen, S), new_seen

    def advance(self, new_seen: int):
        active = min(new_seen, self.max_seq_len)
        self.total_seen_tokens[:] = [new_seen] * self.n_layer
        self.layer_seq_lens[:] = [active] * self.n_layer

    def update(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """paged_cache.py:218-361: write K and V of shape (B, n_kv_head, T,
        head_dim) at the layer's next positions and return the active window.

        Positions follow the reference: a monotonic write while the tokens fit
        (and the cache is not a ring); otherwise a ring write at seen % max_seq_len
        (wrapping to slot 0), or the last max_seq_len tokens when T alone fills
        the cache.  Each layer keeps its own ``total_seen_tokens`` and
        ``layer_seq_lens``.  FP8 / INT4 caches quantize the new rows with the
        CUDA kernels (fp16 inputs by the fp16 rule, fp32 by the fp32 rule) and
        return dequantized fp16 copies of the window, as the reference returns
        high-precision views for SDPA; an fp16 cache returns views of its
        buffers."""
        B, _, T, _ = k.shape
        seen = self.total_seen_tokens[layer_idx]
        S = self.max_seq_len
        kb, vb = self.k_caches[layer_idx], self.v_caches[layer_idx]
        quant = self.cache_dtype != "fp16"
        if quant:
            kq, ks = ops.quantize_kv(k, self.cache_dtype, self.kv_group)
            vq, vs = ops.quantize_kv(v, self.cache_dtype, self.kv_group)
            pairs = ((kb, kq), (vb, vq), (self.k_scales[layer_idx], ks), (self.v_scales[layer_idx], vs))
        else:
            pairs = ((kb, k), (vb, v))

        def put(dst0: int, src0: int, n: int):
            for dst, src in pairs:
                dst[:B, :, dst0:dst0 + n] = src[:, :, src0:src0 + n]

        new_seen = seen + T
        if not self.ring_buffer and new_seen <= S:
            put(seen, 0, T)
        elif T >= S:
            put(0, T - S, S)
        else:
            wp = seen % S
            first = min(T, S - wp)
            put(wp, 0, first)
            if T > first:
                put(0, first, T - first)
        active = min(new_seen, S)
        self.layer_seq_lens[layer_idx] = active
        self.total_seen_tokens[layer_idx] = new_seen
        if quant:
            return (ops.dequantize_kv(kb[:B, :, :active], self.k_scales[layer_idx][:B, :, :active], self.cache_dtype,
                                      self.head_dim),
                    ops.dequantize_kv(vb[:B, :, :active], self.v_scales[layer_idx][:B, :, :active], self.cache_dtype,
                                      self.head_dim))
        return kb[:B, :, :active], vb[:B, :, :active]

    def get_quantized_views(self, layer_idx: int):
        k_s = self.k_scales[layer_idx] if self.scales is not None else None
        v_s = self.v_scales[layer_idx] if self.scales is not None else None
        return self.k_caches[layer_idx], self.v_caches[layer_idx], k_s, v_s

    def compact_tree_path(self, write_pos: int, accepted_indices: list[int], new_total_seen: int | None = None):
        """paged_cache.py:376-462: move accepted tree slots into a contiguous run."""
        n = len(accepted_indices)
        if n > 0 and not all(int(accepted_indices[m]) == m for m in range(n)):
            ops.compact_tree_kv(self.cache, self.scales, int(write_pos), [int(a) for a in accepted_indices],
                                self.cache_dtype)
        if new_total_seen is not None:
            self.advance(new_total_seen)
