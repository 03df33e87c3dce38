"""``StaticKVCache.update`` (paged_cache.py:218-361) against the oracle's cache.

Each case writes a sequence of (B, Hkv, T, hd) chunks through ``update`` and
through ``OracleCache.write`` at the oracle's slot rule (the reference's
monotonic / ring / overflow positions), then checks after every call:

* the cached codes and scales bit-exact (the CUDA quantizer against the
  oracle's restatement of quantize_kv_fp8 / quantize_kv_int4);
* the returned window equal to the oracle's dequantized window (fp16 caches:
  the written values themselves);
* ``total_seen_tokens`` and ``layer_seq_lens`` as the reference keeps them.
"""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

CASES = [
    # kv, group, ring, S, chunk lengths, input dtype
    ("fp16", 64, False, 32, [20, 1, 3, 1], torch.float16),
    ("fp16", 64, True, 16, [10, 1, 9, 1, 20], torch.float16),
    ("fp8", 64, False, 32, [5, 1, 1, 7], torch.float16),
    ("fp8", 64, True, 16, [10, 1, 7, 20, 1], torch.float16),
    ("fp8", 128, False, 24, [8, 1, 1], torch.float32),
    ("int4", 64, True, 16, [12, 1, 5, 1], torch.float16),
    ("int4", 32, False, 40, [16, 1, 2], torch.float32),
    ("fp8", 64, False, 8, [6, 1, 3], torch.float16),  # runs past max_seq_len: wraps like the reference
]


@pytest.mark.parametrize("kv,group,ring,S,chunks,dtype", CASES)
def test_update_matches_oracle(kv, group, ring, S, chunks, dtype):
    from axiomlm_b200.cache import StaticKVCache

    B, H, hd = 2, 3, 128 if group == 128 else 64
    g = torch.Generator().manual_seed(S + len(chunks) + group)
    c = StaticKVCache(B, S, 1, H, hd, ring_buffer=ring, cache_dtype=kv, kv_group=group)
    oc = O.OracleCache(1, B, H, S, hd, kv, ring_buffer=ring, kv_group=group)
    for T in chunks:
        k = (torch.randn(B, H, T, hd, generator=g) * 2).to(dtype)
        v = (torch.randn(B, H, T, hd, generator=g) * 2).to(dtype)
        kd, vd = c.update(0, k.cuda(), v.cuda())
        slots = oc.slots(T)
        oc.write(0, k.numpy(), v.numpy(), slots)
        oc.seen += T
        active = min(oc.seen, S)
        assert c.total_seen_tokens[0] == oc.seen and c.layer_seq_lens[0] == active
        if kv == "fp16":
            assert torch.equal(c.k_caches[0].cpu(), torch.from_numpy(oc.k[0]))
            assert torch.equal(c.v_caches[0].cpu(), torch.from_numpy(oc.v[0]))
        else:
            assert np.array_equal(c.k_caches[0].cpu().numpy(), oc.k[0])
            assert np.array_equal(c.v_caches[0].cpu().numpy(), oc.v[0])
            assert np.array_equal(c.k_scales[0].cpu().numpy(), oc.ks[0])
            assert np.array_equal(c.v_scales[0].cpu().numpy(), oc.vs[0])
        rk, rv = oc.dequant(0, B, active)
        assert kd.shape == (B, H, active, hd)
        assert torch.equal(kd.float().cpu(), rk.float()) and torch.equal(vd.float().cpu(), rv.float())
