"""Micro-benchmarks of single ops on one GPU, timed with CUDA events over a
replayed CUDA graph (inputs rotated over copies larger than L2).

    python -m axiomlm_b200.microbench gemv   [--n N --k K --m M]      Q4 G128 GEMV (warp-level mma)
    python -m axiomlm_b200.microbench tc     [--n N --k K --m M]      Q4 GEMM on tcgen05
    python -m axiomlm_b200.microbench lowbit [--n N --k K --fmt F]    2-bit GEMV
    python -m axiomlm_b200.microbench tree   [--ctx C --nodes T --layers L]   8B-shape tree verification
    python -m axiomlm_b200.microbench medusa [--heads K] [--residual]      8B-shape Medusa draft step

Each prints one line: the op, its shape, microseconds per launch and the
algorithmic GB/s (and TF/s for the GEMMs).  The tree case prints ms per
verify step of T nodes over a C-token prefix.
"""

from __future__ import annotations

import argparse
import ctypes as C
import random

import torch


def _timed_graph(fn, reps: int = 20) -> float:
    st = torch.cuda.current_stream()
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    g.replay()
    e1.record(st)
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3 / reps


def _copies(nbytes: float) -> int:
    return max(1, int(400e6 // max(nbytes, 1.0)))


def bench_q4(kind: str, N: int, K: int, M: int) -> str:
    from . import ops

    W0 = ops.pack_q4t(torch.randn(N, K, device="cuda") * 0.02, 128, True)
    nc = _copies(W0.nbytes)
    Ws = [W0] + [ops.pack_q4t(torch.randn(N, K, device="cuda") * 0.02, 128, True) for _ in range(nc - 1)]
    x = torch.randn(M, K, device="cuda").half()
    out = torch.empty(M, N, device="cuda", dtype=torch.float16)
    f = ops.qgemm_tc if kind == "tc" else ops.qgemm
    t = _timed_graph(lambda i: f(x, Ws[i % nc], out=out))
    byts = W0.nbytes + 2 * M * K + 2 * M * N
    return (f"{kind} N={N} K={K} M={M}: {t * 1e6:.1f} us/launch, {byts / t / 1e9:.0f} GB/s, "
            f"{2 * M * N * K / t / 1e12:.1f} TF/s")


def bench_lowbit(fmt_name: str, N: int, K: int, M: int) -> str:
    from . import _lib as L
    from . import ops

    fmt = {"ternary_g64": L.W_TERNARY_G64, "ternary_pt": L.W_TERNARY_PT, "q2_g64": L.W_Q2_G64,
           "q2k": L.W_Q2K_SB256}[fmt_name]
    codes = torch.randint(0, 255, (N, K // 4), dtype=torch.uint8, device="cuda")
    s2 = None
    if fmt == L.W_TERNARY_G64:
        s1 = (torch.rand(N, K // 64, device="cuda") * 0.01).half()
    elif fmt == L.W_TERNARY_PT:
        s1 = torch.tensor([0.01], device="cuda").half()
    elif fmt == L.W_Q2_G64:
        s1 = (torch.rand(N, K // 64, 2, device="cuda") * 0.01).half()
    else:
        s1 = torch.randint(0, 255, (N, K // 16), dtype=torch.uint8, device="cuda")
        s2 = (torch.rand(N, K // 256, 2, device="cuda") * 0.01).half()
    W0 = ops.q2t_from_ref(fmt, codes, s1, s2, K)
    nc = _copies(W0.nbytes)
    Ws = [W0] + [ops.q2t_from_ref(fmt, codes, s1, s2, K) for _ in range(nc - 1)]
    x = torch.randn(M, K, device="cuda").half()
    out = torch.empty(M, N, device="cuda", dtype=torch.float16)
    t = _timed_graph(lambda i: ops.lbgemm(x, Ws[i % nc], out=out))
    return f"lowbit {fmt_name} N={N} K={K} M={M}: {t * 1e6:.1f} us/launch, {W0.nbytes / t / 1e9:.0f} GB/s"


def random_tree(nodes: int, max_depth: int = 6, max_children: int = 4, seed: int = 0):
    """Seeded random draft tree: depths and ancestor masks (node 0 is the root)."""
    rng = random.Random(seed)
    parents, depths, kids = [-1], [0], [0]
    while len(parents) < nodes:
        cand = [i for i in range(len(parents)) if depths[i] < max_depth and kids[i] < max_children]
        p = rng.choice(cand)
        parents.append(p)
        depths.append(depths[p] + 1)
        kids[p] += 1
        kids.append(0)
    masks = []
    for u in range(nodes):
        m, p = 1 << u, parents[u]
        while p >= 0:
            m |= 1 << p
            p = parents[p]
        masks.append(m)
    return depths, masks


def bench_tree(ctx: int, nodes: int, layers: int) -> str:
    from . import synth
    from .model import QuantizedDecoder

    cfg = dict(synth.CFG_8B, n_layer=layers)
    tmp = synth.build_decoder(cfg, 1, 64, ("fp8", 128))
    packed = tmp.packed
    tmp.close()
    dec = QuantizedDecoder(cfg, packed, kv_dtype="fp8", kv_group=128, max_batch=1, max_seq=ctx + 128,
                           max_tokens=64, rope_len=cfg["block_size"])
    g = torch.Generator(device="cuda").manual_seed(3)
    dec.prefill(torch.randint(0, cfg["vocab"], (1, ctx), generator=g, device="cuda"))
    depths, masks = random_tree(nodes)
    ids = torch.randint(0, cfg["vocab"], (1, nodes), generator=g, device="cuda")
    st = torch.cuda.current_stream()
    for _ in range(3):
        dec.forward_tree_verify(ids, depths, masks)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record(st)
    for _ in range(reps):
        dec.forward_tree_verify(ids, depths, masks)
    e1.record(st)
    e1.synchronize()
    t = e0.elapsed_time(e1) / reps
    status = dec.status()
    dec.close()
    return f"tree verify {nodes} nodes, prefix {ctx}, {layers} layers: {t:.2f} ms/step (status {status})"


def bench_medusa(heads: int, residual: bool) -> str:
    """The device work of one greedy speculative step besides the tree pass:
    walk + compaction, the K heads on the accepted leaf, their top-k and the
    next draft, over the default 17-node tree at the Llama-3-8B shape."""
    from . import _lib as L
    from . import ops
    from .medusa import DEFAULT_MEDUSA_TREE_CHOICES, DeviceTree, MedusaHeads, compile_medusa_tree, draft_tokens
    from .model import QuantizedDecoder

    from . import synth

    cfg = dict(synth.CFG_8B, n_layer=1)
    tmp = synth.build_decoder(cfg, 1, 64, ("fp8", 128))
    packed = tmp.packed
    tmp.close()
    dec = QuantizedDecoder(cfg, packed, kv_dtype="fp8", kv_group=128, max_batch=1, max_seq=4096, max_tokens=64,
                           rope_len=cfg["block_size"])
    d, V = cfg["d_model"], cfg["vocab"]
    g = torch.Generator(device="cuda").manual_seed(11)
    hs = [(ops.pack_q4t(torch.randn(d, d, device="cuda", generator=g) * 0.02, 128, True) if residual else None,
           ops.pack_q4t(torch.randn(V, d, device="cuda", generator=g) * 0.02, 128, True)) for _ in range(heads)]
    mh = MedusaHeads(hs)
    tree = DeviceTree(compile_medusa_tree(DEFAULT_MEDUSA_TREE_CHOICES, heads), "cuda")
    dec.prefill(torch.randint(0, V, (1, 1024), generator=g, device="cuda"))
    dec.forward_tree_verify(torch.randint(0, V, (1, tree.T), generator=g, device="cuda"), tree.depths, tree.masks)
    seen = dec.cache.total_seen_tokens[0]
    result = torch.zeros(L.TREE_RESULT_WORDS, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream()

    def walk():
        L.call("axb_tree_accept", tree.T, ops._p(tree.parent), ops._p(dec.tokens), ops._p(dec.argmax_buf), 64,
               ops._p(result), ops._stream())
        dec.compact_device(seen, result)

    def draft():
        topk = mh.draft(dec.norm_buf, tree.kmax, leaf_dev=result[1:2])
        draft_tokens(tree, topk, result[3:4], dec.tokens)

    def timed(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            fn()
        e1.record(st)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps * 1e3

    t_walk, t_draft = timed(walk), timed(draft)
    t_topk = timed(lambda: L.call("axb_topk_rows", C.c_void_p(mh.logits.data_ptr()), heads, V, V, tree.kmax,
                                  C.c_void_p(mh.topk.data_ptr()), ops._stream()))
    dec.close()
    return (f"medusa draft step ({heads} heads{', residual' if residual else ''}, {tree.T}-node tree): "
            f"walk+compact {t_walk:.1f} us, heads+top-k+draft {t_draft:.1f} us "
            f"({mh.nbytes / (t_draft - t_topk) / 1e3:.0f} GB/s over the head weights), top-k alone {t_topk:.1f} us")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("op", choices=["gemv", "tc", "lowbit", "tree", "medusa"])
    ap.add_argument("--n", type=int, default=28672)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--fmt", default="ternary_g64", choices=["ternary_g64", "ternary_pt", "q2_g64", "q2k"])
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--nodes", type=int, default=64)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--residual", action="store_true")
    a = ap.parse_args(argv)
    torch.cuda.set_device(0)
    if a.op in ("gemv", "tc"):
        print(bench_q4(a.op, a.n, a.k, a.m), flush=True)
    elif a.op == "lowbit":
        print(bench_lowbit(a.fmt, a.n, a.k, a.m), flush=True)
    elif a.op == "medusa":
        print(bench_medusa(a.heads, a.residual), flush=True)
    else:
        print(bench_tree(a.ctx, a.nodes, a.layers), flush=True)


if __name__ == "__main__":
    main()
