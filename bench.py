"""Decode throughput of the quantized hot path (the headline benchmark's metric).

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]
                    [--batch B] [--ctx C] [--layers L]

Workload (the 8B decode benchmark, one GPU): Llama-3-8B-shaped decoder (32 layers,
d 4096, 32/8 heads, head_dim 128, FFN 14336, vocab 128256), random N(0, 0.02)
weights quantized Q4 group-128 symmetric (4.125 bits/weight), FP8-e4m3 KV
cache with one fp16 scale per (token, head), a 4096-token context of random
token ids prefilled through the same runner, batch 1 per GPU.  A step is one
greedy decode step (embed -> 32 layers -> lm_head -> argmax) for every
sequence.  Under torchrun each rank runs its own batch (replicas, weak
scaling); the time is the max over ranks.

``--impl reference`` times the reference algorithm's CPU path (the oracle
restatement of ``_forward_quantized_sequence``: per-call dequant + F.linear,
SDPA over the dequantized FP8 cache) on the host cores, on a bounded sample of
the same step (one layer and 1/32 of the lm_head rows, scaled by 32).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from axiomlm_b200.synth import CFG_8B  # noqa: E402  (after the path insert)

METRIC = "decode tokens/s (Q4 8B-shape, FP8 KV, ctx 4096)"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
# DRAM bytes (read + write) per algorithmic byte of the step kernel, from one
# ncu capture of a smaller case (the 8B layer shapes, 4 layers, ctx 4096:
# 768.5 MB for 754.8 MB); the traffic of a full launch is this ratio times its
# algorithmic bytes.
STEP_TRAFFIC_RATIO = 1.018


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ------------------------------------------------------------------ distributed

def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples during the timed region (the recipe's clocks line)."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 4:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
                bits = int(parts[3], 16)
            except ValueError:
                continue
            for b, name in self.REASONS.items():
                if bits & b and name != "gpu_idle":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ our arm

def build_decoder(cfg, batch, ctx, kv, seed=0, tp=None, weights="q4_g128", ring=0):
    from axiomlm_b200.synth import build_decoder as bd

    return bd(cfg, batch, ctx, kv, seed=seed, tp=tp, weights=weights, ring=ring)


def fill_context(dec, batch, ctx, seed=1):
    from axiomlm_b200.synth import fill_context as fc

    fc(dec, batch, ctx, seed=seed)


def step_bytes(dec, batch):
    """Algorithmic HBM bytes of one decode step: every packed projection and
    the lm_head once, the KV cache of every sequence over the active window
    (codes + scales), the new K/V rows, embeddings rows; activations are
    negligible and excluded."""
    c = dec.cache
    active = c.layer_seq_lens[0]
    row = c.cache.shape[-1] * c.cache.element_size()
    kv = c.n_layer * 2 * batch * c.n_kv_head * active * row
    if c.scales is not None:
        kv += c.n_layer * 2 * batch * c.n_kv_head * active * c.scales.shape[-1] * 2
    emb = batch * dec.cfg["d_model"] * (1 + 2 / 64 * 2)
    return dec.weight_bytes + kv + emb


def gemv_roofline(dec, batch, reps=3):
    """Time every projection GEMV of one step eagerly (same kernel, same
    launch shape as in the graph) with CUDA events on the launching stream;
    report algorithmic bytes per launch / mean launch time."""
    from axiomlm_b200 import _lib as L
    from axiomlm_b200 import ops

    st = torch.cuda.current_stream()
    xs = {}

    def act(K):  # activations of the launch's width (tensor parallel: o and down take a shard)
        if K not in xs:
            xs[K] = torch.randn(batch, K, device="cuda").half()
        return xs[K]

    launches = []
    for lay in dec.packed["layers"]:
        launches += [(lay["qkv"], act(lay["qkv"].K), L.EPI_STORE), (lay["o"], act(lay["o"].K), L.EPI_STORE),
                     (lay["gu"], act(lay["gu"].K), L.EPI_SWIGLU), (lay["down"], act(lay["down"].K), L.EPI_STORE)]
    launches.append((dec.packed["lm_head"], act(dec.packed["lm_head"].K), L.EPI_STORE))
    tot_bytes = sum(W.nbytes + batch * W.K * 2 + batch * W.N * 2 for W, _, _ in launches)

    def lowbit(W):  # 2-bit projections: the 2-bit GEMV, its product stored (the runner's next pass applies SwiGLU)
        return isinstance(W, ops.Q2TWeight)

    outs = [torch.empty(batch, W.N // 2 if e == L.EPI_SWIGLU and not lowbit(W) else W.N, dtype=torch.float16,
                        device="cuda") for W, _, e in launches]

    def run(W, x, e, o):
        if lowbit(W):
            ops.lbgemm(x, W, out=o)
        else:
            ops.qgemm(x, W, epilogue=e, out=o)

    for (W, x, e), o in zip(launches[:8], outs):  # warm-up (allocates the workspace)
        run(W, x, e, o)
    torch.cuda.synchronize()
    # the launch sequence is captured once and replayed, so host launch cost
    # does not leak into the kernel time; same kernels and grids as the runner
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for (W, x, e), o in zip(launches, outs):
            run(W, x, e, o)
    g.replay()
    times = []
    for _ in range(reps):
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record(st)
        g.replay()
        ev1.record(st)
        ev1.synchronize()
        times.append(ev0.elapsed_time(ev1) / 1e3)
    del g
    t = min(times)
    per_launch_s = t / len(launches)
    per_launch_bytes = tot_bytes / len(launches)
    return per_launch_bytes, per_launch_s, len(launches)


def step_roofline(dec, batch, reps=20):
    """Time the decode-step kernel itself: the runner's step (one CUDA-graph
    replay: a tiny parameter kernel and the persistent step kernel) launched
    back to back at fixed positions, CUDA events on the launching stream.
    Algorithmic bytes per launch = step_bytes (weights, the KV window, the new
    K/V rows and embedding rows)."""
    c = dec.cache
    seen = c.total_seen_tokens[0]
    wp, active, _ = c.next_positions(1)
    st = torch.cuda.current_stream()
    for _ in range(3):
        dec._step(batch, 1, seen % dec.rope_len, wp, active, 0)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        dec._step(batch, 1, seen % dec.rope_len, wp, active, 0)
    e1.record(st)
    e1.synchronize()
    return step_bytes(dec, batch), e0.elapsed_time(e1) / 1e3 / reps, reps


def run_ours(args, rank, world):
    from axiomlm_b200 import _lib as L

    L.load()
    if L.load().axb_check_device() != 0:
        raise SystemExit(L.load().axb_last_error().decode())
    cfg = dict(CFG_8B)
    if args.layers:
        cfg["n_layer"] = args.layers
    kv = {"fp8_head": ("fp8", 128), "fp8_g64": ("fp8", 64), "fp16": ("fp16", 64), "int4_g32": ("int4", 32)}[args.kv]
    B = args.batch
    tp = None
    if args.tp > 1:  # every rank works on the same sequences: ids and positions must agree
        from axiomlm_b200.tp import TensorParallel

        if args.tp != world:
            raise SystemExit(f"--tp {args.tp} needs {args.tp} ranks under torchrun (got {world})")
        tp = TensorParallel.from_process_group()
    dec = build_decoder(cfg, B, args.ctx, kv, seed=1000 + (0 if tp else rank), tp=tp, weights=args.weights,
                        ring=args.ring)
    fill_context(dec, B, args.ctx, seed=2000 + (0 if tp else rank))
    st = torch.cuda.current_stream()
    tok = dec.argmax(B).view(B, 1).long()
    for _ in range(args.warmup):
        dec.decode_step(tok)
        tok = dec.argmax(B).view(B, 1).long()
    torch.cuda.synchronize()
    # ---- device-timed region: K greedy steps, inputs resident in HBM
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        barrier(world)
        torch.cuda.synchronize()
        ev0.record(st)
        for _ in range(args.steps):
            dec.decode_step(tok)
            tok = dec.argmax(B).view(B, 1).long()  # next input stays on the device
        ev1.record(st)
        torch.cuda.synchronize()
        barrier(world)
    t = max_over_ranks(ev0.elapsed_time(ev1) / 1e3, world)
    seqs = B if tp else world * B  # tensor parallel: the ranks share the same B sequences
    value = seqs * args.steps / t
    sbytes = step_bytes(dec, B)
    # ---- end to end through the public API, host buffers
    host_in = torch.zeros((B, 1), dtype=torch.int64).pin_memory()
    host_out = torch.zeros((B,), dtype=torch.int32).pin_memory()
    host_in.copy_(tok.cpu())
    dev_in = torch.empty((B, 1), dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        dev_in.copy_(host_in, non_blocking=True)
        dec.decode_step(dev_in)
        host_out.copy_(dec.argmax(B), non_blocking=True)
        st.synchronize()
        host_in[:, 0].copy_(host_out)
    e1.record(st)
    e1.synchronize()
    barrier(world)
    te = max_over_ranks(e0.elapsed_time(e1) / 1e3, world)
    e2e = {"value": seqs * args.steps / te, "unit": "tokens/s", "h2d_bytes_per_step": B * 8,
           "d2h_bytes_per_step": B * 4}
    # ---- roofline of the dominant kernel: the persistent step kernel (one
    # launch per step), or the Q4 GEMV when the per-kernel graph runs the step
    pk, pk_kind = peaks()
    step_kernel = dec.uses_step_kernel and B <= 8  # the persistent kernel takes decode batches of up to 8
    lowbit = args.weights != "q4_g128"
    if lowbit:  # 2-bit projections on the per-kernel graph: the 2-bit GEMV dominates
        bpl, spl, nl = gemv_roofline(dec, B)
        kname = f"lbgemv_kernel ({args.weights} GEMV, split-K) + its x-sum / reduce kernels"
    elif step_kernel:
        bpl, spl, nl = step_roofline(dec, B)
        kname = "step_kernel<SYM, GB=2, HD=128> (whole decode step, one persistent launch)"
    elif B > 16:  # many-token decode: the graph path with the tcgen05 projections; whole step timed
        bpl, spl, nl = step_roofline(dec, B)
        kname = "per-op CUDA graph step (qgemm_tc_kernel projections, split decode attention)"
    else:
        bpl, spl, nl = gemv_roofline(dec, B)
        kname = "qgemm_kernel<1,SYM,2,*> (Q4 G128 GEMV)"
    achieved = bpl / spl / 1e9
    out = None
    if rank == 0:
        # the runner counts the kernel nodes of the step's CUDA graph (+ its parameter kernel)
        launches_per_step = L.load().axb_runner_step_launches(dec._h, B, 1, 0)
        if launches_per_step < 0:  # no graph captured (cooperative launch outside a graph)
            launches_per_step = 2
        out = {
            "metric": METRIC if not (lowbit or args.ring) else
            f"decode tokens/s ({args.weights} 8B-shape, KV {args.kv}, ctx {args.ctx}"
            + (f", ring {args.ring})" if args.ring else ")"),
            "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
            "dtype": "w2a16 (fp32 accumulate)" if lowbit else "w4a16 (fp32 accumulate)",
            "data": "synthetic (seeded N(0,0.02) weights, uniform-random token ids)",
            "config": {"workload": f"Llama-3-8B-shape decode ({cfg['n_layer']} layers), "
                                   + {"q4_g128": "Q4 G128 sym", "ternary_pt": "BitNet ternary per-tensor",
                                      "q2k": "Q2_K 256 super-blocks"}[args.weights]
                                   + f", KV {args.kv}, ctx {args.ctx}"
                                   + (f" (ring window {args.ring})" if args.ring else "") + f", batch {B}"
                                   + (f" tensor-parallel x{world}" if tp else "/GPU"),
                       "global_batch": seqs, "seq_len": args.ctx,
                       "parallelism": f"tp{world}" if tp else f"replicas x{world}",
                       "l2": "inputs larger than L2 (weights %.2f GB per step)" % (dec.weight_bytes / 1e9)},
            "achieved_hbm_gbs": round(sbytes * B * args.steps / B / t / 1e9 / 1, 1) if world == 1 else None,
            "step_bytes": int(sbytes),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / pk["hbm_gbs"], 4),
                         "traffic": int(bpl * STEP_TRAFFIC_RATIO) if step_kernel else None,
                         "kernel": kname, "launches_timed": nl, "us_per_launch": round(spl * 1e6, 1),
                         "bytes_per_launch": int(bpl), "peak_kind": f"{pk_kind} (MEASURED_PEAKS.json hbm_gbs)"},
            "e2e": {k: (round(v, 2) if isinstance(v, float) else v) for k, v in e2e.items()},
            "clocks": clk.summary(), "gpu_launches": launches_per_step * args.steps,
        }
        if world == 1 and not args.no_cpu_baseline and not lowbit and not args.ring:
            out["cpu_baseline"] = cpu_baseline(cfg, B, args.ctx, kv, args)
    dec.close()
    if tp is not None:
        tp.close()
    return out


# ------------------------------------------------------------------ CPU (oracle) arm

def _cpu_sample_fns(cfg, B, ctx, kv):
    """Build the bounded CPU sample: one decoder layer of the step and 1/32 of
    the lm_head rows, packed in the reference's MARLIN layout (random codes;
    the dequant + F.linear cost does not depend on values)."""
    import numpy as np

    import oracle as O

    d, H, Hkv, F, V = cfg["d_model"], cfg["n_head"], cfg["n_kv_head"], cfg["ffn"], cfg["vocab"]
    hd = d // H
    rng = np.random.default_rng(0)

    def ladder(N, K):
        nt = (N + 7) // 8
        w = rng.integers(-2 ** 31, 2 ** 31 - 1, size=(nt, K // 64, 32, 2), dtype=np.int64).astype(np.int32)
        sb = (rng.standard_normal((nt, K // 64, 8, 2)) * 0.01).astype(np.float16)
        return torch.from_numpy(w), torch.from_numpy(sb)

    mats = {"qkv": ladder((H + 2 * Hkv) * hd, d), "o": ladder(d, H * hd), "gu": ladder(2 * F, d),
            "down": ladder(d, F), "lm": ladder(V // cfg["n_layer"], d)}
    kvq = torch.from_numpy(rng.integers(0, 120, size=(B, Hkv, ctx, hd), dtype=np.uint8))
    kvs = torch.from_numpy((rng.random((B, Hkv, ctx, hd // kv[1])) * 0.01).astype(np.float16))
    x = torch.randn(B, 1, d).half()

    def linear(name, inp, K, n):
        w, sb = mats[name]
        W = O.dequant_q4_marlin_torch(w, sb, K, n)  # quant.py:656-661: dequantized on every call
        return torch.nn.functional.linear(inp.half(), W)

    def sample():
        qkv = linear("qkv", x, d, (H + 2 * Hkv) * hd).float()
        q = qkv[..., : H * hd].view(B, 1, H, hd).transpose(1, 2)
        kd = torch.from_numpy(O.dequant_kv_fp8(kvq.numpy(), kvs.numpy(), kv[1])).float()
        vd = torch.from_numpy(O.dequant_kv_fp8(kvq.numpy(), kvs.numpy(), kv[1])).float()
        y = O.attention_decode(q, kd, vd, ctx).transpose(1, 2).reshape(B, 1, H * hd)
        o = linear("o", y, H * hd, d)
        gu = linear("gu", o, d, 2 * F).float()
        sw = torch.nn.functional.silu(gu[..., :F]) * gu[..., F:]
        dn = linear("down", sw, F, d)
        linear("lm", dn, d, V // cfg["n_layer"])

    return sample


def cpu_baseline(cfg, B, ctx, kv, args):
    """The reported CPU baseline beside our arm: one full decode step of the
    reference's own CPU path (reference_cpu), or, when the reference is not
    installed, the oracle restatement on a bounded sample."""
    import copy

    a = copy.copy(args)
    a.steps, a.warmup = 1, 1
    res = reference_cpu(a)
    if res is not None:
        t = sum(res["step_s"]) / res["steps"]
        return {"value": round(B / t, 4), "unit": "tokens/s", "cores": res["cores"], "kind": "reference",
                "sample": f"1 full {res['layers']}-layer decode step of {res['module']} after 1 warm-up step "
                          f"({t:.1f} s; one packed layer serving every layer slot; FP8 G64 cache, ctx {ctx})"}
    torch.set_num_threads(os.cpu_count() or 1)
    sample = _cpu_sample_fns(cfg, B, ctx, kv)
    sample()  # warm
    t0 = time.perf_counter()
    sample()
    t = time.perf_counter() - t0
    return {"value": round(B / (t * cfg["n_layer"]), 4), "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"1 of {cfg['n_layer']} layers + 1/{cfg['n_layer']} of lm_head rows per step "
                      f"(oracle restatement: per-call dequant + F.linear, SDPA over the dequantized FP8 cache, "
                      f"ctx {ctx}), x{cfg['n_layer']}"}


REF_ROOT = os.path.join(ROOT, "baseline", "_ref")  # the reference, installed offline (pip --target)


def _ref_step_worker(args):
    """The reference's own CPU decode path, timed on the host cores (run in a
    fresh process: no CUDA context, every core to torch's CPU kernels).

    A step is one greedy decode token at the bench config through
    ``Transformer.forward`` -> ``_forward_quantized_sequence``
    (axiomlm/models/transformer.py:1036-1200) after ``quantize("q4_rtn")``:
    every layer's ``qmv_q4_marlin`` (quant.py:637-661, which dequantizes the
    whole matrix on every call), RMSNorm, RoPE, ``StaticKVCache.update``
    (paged_cache.py:218-361, re-quantizing and dequantizing the FP8 window) and
    SDPA, then the lm_head.  To keep the set-up within seconds, one decoder
    layer is packed by the reference and its packed tensors serve all 32
    layer slots (the cost of a layer does not depend on the weight values);
    the 4096-token context is written straight into the reference's cache
    buffers as FP8 codes made by its own quantize_kv_fp8.  The reference's FP8
    cache has a scale per 64 elements (its only FP8 format)."""
    if not os.path.isdir(os.path.join(REF_ROOT, "axiomlm")):
        return None
    sys.path.insert(0, REF_ROOT)
    torch.set_num_threads(os.cpu_count() or 1)
    from axiomlm.engine.paged_cache import StaticKVCache
    from axiomlm.kernels.quant import quantize_kv_fp8
    from axiomlm.models.transformer import ModelConfig, Transformer

    cfg = dict(CFG_8B)
    if args.layers:
        cfg["n_layer"] = args.layers
    L, B, ctx = cfg["n_layer"], args.batch, args.ctx
    d, H, Hkv, F, V = cfg["d_model"], cfg["n_head"], cfg["n_kv_head"], cfg["ffn"], cfg["vocab"]
    hd = d // H
    n_steps, n_warm = max(1, min(args.steps, 2)), max(1, min(args.warmup, 1))
    t_setup = time.perf_counter()
    mc = ModelConfig(block_size=ctx + n_steps + n_warm + 8, vocab_size=V, n_layer=1, n_head=H, n_embd=d,
                     n_kv_head=Hkv, intermediate_size=F, rms_norm_eps=cfg["eps"], rope_theta=cfg["theta"],
                     tie_word_embeddings=False)
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        m = Transformer(mc, init_weights=False)
        for name, p in m.named_parameters():
            if p.dim() == 1:
                p.fill_(1.0)
            else:
                p.normal_(0.0, 0.02, generator=g)
        m.eval()
        m.quantize("q4_rtn")
        qw = m._ensure_quant_weights(torch.device("cpu"))
        for key in ("c_attn_p", "c_attn_s", "c_attn_b", "c_proj_p", "c_proj_s", "gu_p", "gu_s", "wd_p", "wd_s"):
            qw[key] = [qw[key][0]] * L
        m.transformer.h = torch.nn.ModuleList([m.transformer.h[0]] * L)
        m.config.n_layer = L
        cache = StaticKVCache(B, mc.block_size, L, Hkv, hd, dtype=torch.float16, device="cpu", cache_dtype="fp8")
        k = torch.randn(B, Hkv, ctx, hd, generator=g).half()
        v = torch.randn(B, Hkv, ctx, hd, generator=g).half()
        kq, ks, vq, vs = quantize_kv_fp8(k, v)
        for i in range(L):
            cache.k_caches[i][:, :, :ctx] = kq
            cache.v_caches[i][:, :, :ctx] = vq
            cache.k_scales[i][:, :, :ctx] = ks
            cache.v_scales[i][:, :, :ctx] = vs
        cache.total_seen_tokens = [ctx] * L
        cache.layer_seq_lens = [ctx] * L
        t_setup = time.perf_counter() - t_setup
        idx = torch.randint(0, V, (B, 1), generator=g)
        for _ in range(n_warm):
            logits, _, _ = m(idx, kv_caches=cache)
            idx = logits[:, -1].argmax(-1, keepdim=True)
        times = []
        for _ in range(n_steps):
            t0 = time.perf_counter()
            logits, _, _ = m(idx, kv_caches=cache)
            idx = logits[:, -1].argmax(-1, keepdim=True)
            times.append(time.perf_counter() - t0)
    return {"step_s": times, "setup_s": t_setup, "cores": torch.get_num_threads(), "layers": L, "batch": B,
            "steps": n_steps, "warmup": n_warm, "module": "axiomlm.models.transformer.Transformer (q4_rtn)"}


def reference_cpu(args):
    """Time the reference's CPU step in a child process (spawned fresh: no
    CUDA context is inherited); None when the reference is not installed."""
    import subprocess

    cmd = [sys.executable, os.path.abspath(__file__), "--ref-worker", "--batch", str(args.batch), "--ctx",
           str(args.ctx), "--steps", str(args.steps), "--warmup", str(args.warmup)]
    if args.layers:
        cmd += ["--layers", str(args.layers)]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    if r.returncode != 0 or not lines:
        sys.stderr.write(r.stderr[-2000:])
        return None
    return json.loads(lines[-1])


def run_reference(args, rank, world):
    """``--impl reference``: the reference's own CPU decode path, rank 0 only
    (other ranks exit without work).  Falls back to the oracle restatement
    only when the reference is not installed."""
    if rank != 0:
        return None
    cfg = dict(CFG_8B)
    if args.layers:
        cfg["n_layer"] = args.layers
    res = reference_cpu(args)
    if res is None:
        kv = {"fp8_head": ("fp8", 128), "fp8_g64": ("fp8", 64), "fp16": ("fp16", 64), "int4_g32": ("int4", 32)}[args.kv]
        torch.set_num_threads(os.cpu_count() or 1)
        sample = _cpu_sample_fns(cfg, args.batch, args.ctx, kv)
        for _ in range(args.warmup):
            sample()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            sample()
        t = (time.perf_counter() - t0) * cfg["n_layer"]
        steps, warm, ms = args.steps, args.warmup, t / args.steps * 1e3
        kind, sample_txt, cores = "port", (f"per step: 1 of {cfg['n_layer']} layers + 1/{cfg['n_layer']} of lm_head "
                                           f"rows, x{cfg['n_layer']} (oracle restatement; reference not installed)"), \
            torch.get_num_threads()
    else:
        steps, warm, cores = res["steps"], res["warmup"], res["cores"]
        t = sum(res["step_s"])
        ms = t / steps * 1e3
        kind = "reference"
        sample_txt = (f"{steps} full {res['layers']}-layer decode steps of {res['module']} on the host cores "
                      f"(one packed layer serving every layer slot; FP8 G64 cache, ctx {args.ctx}); "
                      f"per-step s: {', '.join('%.2f' % x for x in res['step_s'])}; set-up {res['setup_s']:.0f} s")
    v = args.batch * steps / t
    cb = {"value": round(v, 4), "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample_txt}
    return {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": round(ms, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (CPU)",
            "data": "synthetic", "config": {"workload": f"Llama-3-8B-shape decode ({cfg['n_layer']} layers), Q4 "
                                                        f"(reference MARLIN RTN layout), KV fp8 G64, ctx {args.ctx}, "
                                                        f"batch {args.batch}",
                                            "global_batch": args.batch, "seq_len": args.ctx,
                                            "parallelism": "CPU, rank 0 only"},
            "cpu_baseline": cb, "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--kv", default="fp8_head", choices=["fp8_head", "fp8_g64", "fp16", "int4_g32"])
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (debug only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel ranks (all ranks share one batch)")
    ap.add_argument("--weights", default="q4_g128", choices=["q4_g128", "ternary_pt", "q2k"],
                    help="projection and lm_head format (2-bit: the long-context low-bit configuration)")
    ap.add_argument("--ring", type=int, default=0, help="ring cache of this many slots (the sliding window)")
    ap.add_argument("--ref-worker", action="store_true", help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.ref_worker:  # child process of reference_cpu: CPU only
        res = _ref_step_worker(args)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.steps is None:
        args.steps = 200 if args.impl == "ours" else 5
    if args.warmup is None:
        args.warmup = 10 if args.impl == "ours" else 3
    args.warmup = max(args.warmup, 3)
    rank, world = dist_setup(args.gpus)
    if args.impl == "reference":
        out = run_reference(args, rank, world)
    else:
        out = run_ours(args, rank, world)
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
