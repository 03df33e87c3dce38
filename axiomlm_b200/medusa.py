"""Medusa speculative decoding on the B200 runner.

Mirrors the reference's speculative API:

* ``compile_medusa_tree`` / ``DEFAULT_MEDUSA_TREE_CHOICES``
  (engine/medusa.py:28-116);
* ``MedusaSpeculativeDecoder.generate`` (engine/medusa.py:119-537): greedy
  (temperature 0) tree and linear-chain verification;
* ``sample_without_replacement``, ``SequoiaTreeVerifier`` and
  ``fit_power_law_rejection_bound`` (speculative/sampling.py:20-446), the
  sampled (temperature > 0) regime;
* ``MedusaHeads``: the quantized Medusa heads of ``eval_medusa_heads``
  (models/transformer.py:414-445, models/medusa.py:20-54).

At temperature 0 a whole speculative step stays on the GPU: the runner's tree
step (logits and per-node argmax of every node), the greedy walk
(``axb_tree_accept``), the KV compaction with the count read on the device
(``axb_compact_kv_dev``), the Medusa heads on the last accepted node, a
per-head top-k and the next draft written straight into the runner's token
buffer.  The host reads back one small result block per step (the accepted
nodes and emitted tokens) where the reference pulls the (T, V) logits'
argmax through ``.tolist()``.  The sampled regime is host logic over the
device logits, as in the reference, drawing from the caller's generator in
the reference's order.
"""

from __future__ import annotations

import ctypes as C
import math
import time
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.nn.functional as F

from . import _lib as L
from . import ops

# engine/medusa.py:28-45: the reference's default draft tree (16 rank paths,
# 17 nodes with the root).  A data table: kept identical so that the default
# trees of the two implementations are the same tree.
DEFAULT_MEDUSA_TREE_CHOICES: list[tuple[int, ...]] = [
    (0,), (1,), (2,), (3,),
    (0, 0), (0, 1), (0, 2), (1, 0), (1, 1), (2, 0),
    (0, 0, 0), (0, 0, 1), (0, 1, 0), (0, 1, 1), (1, 0, 0),
    (0, 0, 0, 0),
]


# ------------------------------------------------------------------ the tree
def compile_medusa_tree(tree_choices, num_heads: int, max_nodes: int = 32) -> dict[str, Any]:
    """engine/medusa.py:48-116.  Every choice (a tuple of per-head top-k
    ranks, at most ``num_heads`` long) and all its prefixes become nodes,
    ordered by (depth, ranks); node 0 is the root.  ``max_nodes`` = 32
    reproduces the reference (31 paths and the root, 32-bit masks); up to 64
    uses the runner's 64-bit ancestor masks."""
    if not 2 <= max_nodes <= L.TREE_MAX_NODES:
        raise ValueError(f"max_nodes must be 2..{L.TREE_MAX_NODES}")
    nodes: set[tuple[int, ...]] = set()
    for choice in tree_choices:
        path = tuple(int(r) for r in choice)
        if 0 < len(path) <= num_heads:
            nodes.update(path[:n] for n in range(1, len(path) + 1))
    paths = sorted(nodes, key=lambda p: (len(p), p))[: max_nodes - 1]
    T = len(paths) + 1
    index = {(): 0}
    depths, masks, parent = [0] * T, [1] + [0] * (T - 1), [-1] * T
    children: list[list[int]] = [[] for _ in range(T)]
    head_idx, topk_rank = [-1] * T, [-1] * T
    max_topk = [1] * num_heads
    for u, path in enumerate(paths, start=1):
        index[path] = u
        p = index[path[:-1]]
        depths[u] = len(path)
        parent[u] = p
        children[p].append(u)
        head_idx[u] = len(path) - 1
        topk_rank[u] = path[-1]
        masks[u] = masks[p] | (1 << u)
        max_topk[len(path) - 1] = max(max_topk[len(path) - 1], path[-1] + 1)
    return {
        "num_nodes": T,
        "tree_depths": depths,
        "tree_mask": masks,
        "parent": parent,
        "children": children,
        "head_idx": head_idx,
        "topk_rank": topk_rank,
        "max_topk_per_head": max_topk,
        "max_depth": max(depths),
    }


def chain_tree(num_heads: int) -> dict[str, Any]:
    """The linear-chain draft (engine/medusa.py:383-418) as a tree: node j
    (1..num_heads) is head j-1's rank-0 token, a causal chain."""
    return compile_medusa_tree([(0,) * num_heads], num_heads, max_nodes=min(L.TREE_MAX_NODES, num_heads + 1))


def greedy_tree_walk(preds: list[int], verif_seq: list[int], children: list[list[int]], budget: int):
    """engine/medusa.py:312-330 on the host: (accepted nodes, emitted tokens)."""
    cur, accepted, emitted = 0, [0], []
    while len(emitted) < budget:
        tok = preds[cur]
        emitted.append(tok)
        nxt = next((c for c in children[cur] if verif_seq[c] == tok), None)
        if nxt is None or len(emitted) >= budget:
            break
        cur = nxt
        accepted.append(cur)
    return accepted, emitted


class DeviceTree:
    """A compiled tree's tables on the GPU (int32 parent / head / rank) plus
    the host lists the runner step takes (depths, 64-bit masks)."""

    def __init__(self, tree: dict[str, Any], device):
        self.tree = tree
        self.T = tree["num_nodes"]
        if self.T > L.TREE_MAX_NODES:
            raise ValueError(f"tree of {self.T} nodes exceeds {L.TREE_MAX_NODES}")
        par = tree["parent"]
        if par[0] != -1 or any(not 0 <= par[u] < u for u in range(1, self.T)):
            raise ValueError("tree parent table must have parent[0] = -1 and 0 <= parent[u] < u")
        self.depths = list(tree["tree_depths"])
        self.masks = list(tree["tree_mask"])
        self.max_topk = list(tree["max_topk_per_head"])
        self.kmax = max(self.max_topk)
        if self.kmax > L.TOPK_MAX:
            raise ValueError(f"a head's top-k of {self.kmax} exceeds {L.TOPK_MAX}")
        rank = [max(r, 0) for r in tree["topk_rank"]]
        head = [max(h, 0) for h in tree["head_idx"]]
        self.parent = torch.tensor(par, dtype=torch.int32, device=device)
        self.head_idx = torch.tensor(head, dtype=torch.int32, device=device)
        self.rank = torch.tensor(rank, dtype=torch.int32, device=device)


# ------------------------------------------------------------ Medusa heads
def _q4t_cat(ws: list[ops.Q4TWeight]) -> ops.Q4TWeight:
    """Rows of several q4t weights stacked into one (N of each a multiple of
    the 16-row tile): one GEMV serves heads that share their input."""
    w0 = ws[0]
    return ops.Q4TWeight(torch.cat([w.words for w in ws]), torch.cat([w.scales for w in ws]), sum(w.N for w in ws),
                         w0.K, w0.group, w0.fmt)


class MedusaHeads:
    """K quantized Medusa heads: head k maps a final-norm row x (fp32) to
    logits W_head_k h, with h = x + silu(fp16(W_res_k fp16(x))) when the head
    has a residual block (MedusaHead.forward, models/medusa.py:44-53, on the
    quantized path of eval_medusa_heads, transformer.py:420-441) and h = x
    otherwise.  Logits are fp16 values (the reference's _qlin output).

    Heads without residual blocks share their input, so their weights are
    stacked into one (K * V, d) GEMV; residual blocks are stacked the same
    way into one (K * d, d) GEMV."""

    def __init__(self, heads: list[tuple[ops.Q4TWeight | None, ops.Q4TWeight]], max_rows: int = 64):
        if not heads:
            raise ValueError("no Medusa heads")
        self.K = len(heads)
        self.res = [r for r, _ in heads]
        self.head = [h for _, h in heads]
        self.d = self.head[0].K
        self.vocab = self.head[0].N
        for r, h in heads:
            if h.K != self.d or h.N != self.vocab or (r is not None and (r.N != self.d or r.K != self.d)):
                raise ValueError("Medusa heads must all map d_model -> vocab (residual blocks d_model -> d_model)")
        dev = self.head[0].words.device
        self.device = dev
        self.max_rows = max_rows
        self.any_res = any(r is not None for r in self.res)
        same = len({(h.fmt, h.group) for h in self.head}) == 1
        self.head_stack = (_q4t_cat(self.head) if (not self.any_res and same and self.vocab % 16 == 0 and self.K > 1)
                           else None)
        res = [r for r in self.res if r is not None]
        self.res_stack = (_q4t_cat(res) if (len(res) == self.K and len({(r.fmt, r.group) for r in res}) == 1)
                          else None)
        R = max_rows
        self.x32 = torch.empty((R, self.d), dtype=torch.float32, device=dev)
        self.x16 = torch.empty((R, self.d), dtype=torch.float16, device=dev)
        self.r16 = torch.empty((R, self.K * self.d), dtype=torch.float16, device=dev) if self.any_res else None
        self.h16 = torch.empty((R, self.K * self.d), dtype=torch.float16, device=dev) if self.any_res else None
        self.logits = torch.empty((R, self.K, self.vocab), dtype=torch.float16, device=dev)
        self.topk = torch.empty((self.K, L.TOPK_MAX), dtype=torch.int32, device=dev)
        lib = L.load()
        ws = max(lib.axb_qgemm_workspace_bytes(w.N, w.K, min(R, 64), w.group)
                 for w in self.head + res + [x for x in (self.head_stack, self.res_stack) if x is not None])
        self.workspace = torch.zeros(ws, dtype=torch.uint8, device=dev)

    @property
    def num_heads(self) -> int:
        return self.K

    @property
    def nbytes(self) -> int:
        return sum(w.nbytes for w in self.head) + sum(r.nbytes for r in self.res if r is not None)

    # ---- builders
    @classmethod
    def from_weights(cls, heads: list[dict], weight_format: str = "q4_rtn", **kw) -> "MedusaHeads":
        """fp32 master weights ``[{"head": (V, d), "res": (d, d) or None}]``
        (MedusaHead.head.weight / res_block[0].weight), packed on the GPU the
        way the decoder packs its projections."""
        from .model import WEIGHT_FORMATS

        fmt, group = WEIGHT_FORMATS[weight_format]
        if fmt not in (L.W_Q4T_SYM, L.W_Q4T_AFFINE):
            raise NotImplementedError(f"Medusa heads are served in the Q4 formats, not {weight_format!r}")
        sym = fmt == L.W_Q4T_SYM
        dev = torch.device(kw.pop("device", "cuda"))
        packed = []
        for h in heads:
            r = h.get("res")
            packed.append((None if r is None else ops.pack_q4t(r.to(dev, torch.float32), group, sym),
                           ops.pack_q4t(h["head"].to(dev, torch.float32), group, sym)))
        return cls(packed, **kw)

    @classmethod
    def from_packs(cls, medusa_packs: list[dict], d: int, vocab: int, device="cuda", **kw) -> "MedusaHeads":
        """The reference's packed heads (``_ensure_quant_weights()["medusa_packs"]``,
        transformer.py:972-986: MARLIN Q4 ``res_p/res_s``, ``head_p/head_s``),
        relaid out bit-exactly."""
        dev = torch.device(device)
        out = []
        for hp in medusa_packs:
            if hp["head_p"].ndim != 4:
                raise NotImplementedError("Medusa heads must be MARLIN Q4 packs")
            r = None
            if hp.get("res_p") is not None and hp.get("res_s") is not None:
                r = ops.q4t_from_marlin(hp["res_p"].to(dev), hp["res_s"].to(dev), d)
            out.append((r, ops.q4t_from_marlin(hp["head_p"].to(dev), hp["head_s"].to(dev), vocab)))
        return cls(out, **kw)

    # ---- evaluation
    def _gemv(self, W: ops.Q4TWeight, x: int, ldx: int, M: int, y: int, ldy: int):
        d = L.QGemmDesc(fmt=W.fmt, group=W.group, words=W.words.data_ptr(), scales=W.scales.data_ptr(), N=W.N,
                        K=W.K, M=M, x=x, ldx=ldx, y=y, ldy=ldy, bias=None, norm_w=None, eps=0.0,
                        epilogue=L.EPI_STORE, gate_up_interleave=0, workspace=self.workspace.data_ptr(),
                        workspace_bytes=self.workspace.numel(), pdl=0)
        L.call("axb_qgemm", C.byref(d), ops._stream())

    def _run(self, M: int):
        """logits[:M] from x32 / x16 [:M] (already staged)."""
        K, d, V = self.K, self.d, self.vocab
        st = ops._stream()
        if self.any_res:
            if self.res_stack is not None:
                self._gemv(self.res_stack, self.x16.data_ptr(), d, M, self.r16.data_ptr(), K * d)
            else:
                for k, r in enumerate(self.res):
                    if r is not None:
                        self._gemv(r, self.x16.data_ptr(), d, M, self.r16.data_ptr() + 2 * k * d, K * d)
            for m in range(M):
                L.call("axb_medusa_silu_add", K, d, C.c_void_p(self.x32[m].data_ptr()),
                       C.c_void_p(self.r16[m].data_ptr()), C.c_void_p(self.h16[m].data_ptr()), st)
        if self.head_stack is not None:
            self._gemv(self.head_stack, self.x16.data_ptr(), d, M, self.logits.data_ptr(), K * V)
            return
        for k, h in enumerate(self.head):
            if self.res[k] is not None:
                x, ldx = self.h16.data_ptr() + 2 * k * d, K * d
            else:
                x, ldx = self.x16.data_ptr(), d
            self._gemv(h, x, ldx, M, self.logits.data_ptr() + 2 * k * V, K * V)

    @torch.no_grad()
    def __call__(self, x_norm: torch.Tensor) -> list[torch.Tensor]:
        """eval_medusa_heads (transformer.py:414-445): x_norm (..., d) fp32
        final-norm rows -> K logits tensors (..., V) fp16 (fresh tensors)."""
        x = ops._cuda(x_norm, "x_norm")
        lead = x.shape[:-1]
        rows = x.reshape(-1, self.d).float()
        outs = []
        for m0 in range(0, rows.shape[0], self.max_rows):
            m = min(self.max_rows, rows.shape[0] - m0)
            self.x32[:m].copy_(rows[m0:m0 + m])
            self.x16[:m].copy_(rows[m0:m0 + m])
            self._run(m)
            outs.append(self.logits[:m].clone())
        lg = torch.cat(outs) if outs else self.logits[:0]
        return [lg[:, k].reshape(*lead, self.vocab) for k in range(self.K)]

    def draft(self, norm: torch.Tensor, kmax: int, leaf_dev: torch.Tensor | None = None, leaf: int = -1) -> torch.Tensor:
        """Device pipeline: heads on final-norm row ``leaf`` (a device int32
        scalar in ``leaf_dev`` or a host index) and their top-``kmax`` token
        ids, (K, kmax) int32 in ``self.topk`` (no host synchronization)."""
        st = ops._stream()
        L.call("axb_medusa_leaf", C.c_void_p(norm.data_ptr()), self.d, ops._p(leaf_dev), int(leaf),
               C.c_void_p(self.x32.data_ptr()), C.c_void_p(self.x16.data_ptr()), st)
        self._run(1)
        k = min(kmax, self.vocab)
        L.call("axb_topk_rows", C.c_void_p(self.logits.data_ptr()), self.K, self.vocab, self.vocab, k,
               C.c_void_p(self.topk.data_ptr()), st)
        return self.topk.view(-1)[: self.K * k].view(self.K, k)


def topk_rows(x: torch.Tensor, k: int) -> torch.Tensor:
    """Top-k indices of each fp16 row on the GPU (value descending, ties to the
    lower index): the greedy regime of sample_without_replacement."""
    x = ops._cuda(x, "x")
    if x.dtype != torch.float16:
        raise RuntimeError("topk_rows needs fp16 rows")
    rows = x.reshape(-1, x.shape[-1])
    out = torch.empty((rows.shape[0], k), dtype=torch.int32, device=x.device)
    L.call("axb_topk_rows", ops._p(rows), rows.shape[0], rows.shape[1], rows.shape[1], k, ops._p(out), ops._stream())
    return out.view(*x.shape[:-1], k)


def tree_accept(tree: DeviceTree, verif: torch.Tensor, preds: torch.Tensor, budget: int,
                result: torch.Tensor | None = None) -> torch.Tensor:
    """axb_tree_accept on device int32 token / argmax rows; returns the result
    block (AXB_TREE_RESULT_WORDS int32)."""
    if result is None:
        result = torch.empty(L.TREE_RESULT_WORDS, dtype=torch.int32, device=verif.device)
    L.call("axb_tree_accept", tree.T, ops._p(tree.parent), ops._p(verif), ops._p(preds), int(budget), ops._p(result),
           ops._stream())
    return result


def draft_tokens(tree: DeviceTree, topk: torch.Tensor, root: torch.Tensor, tokens: torch.Tensor):
    """Next draft into ``tokens`` (device int32): node 0 = *root, node u = the
    rank topk_rank[u] token of head head_idx[u] (topk: (K, kmax) int32)."""
    L.call("axb_draft_tokens", tree.T, ops._p(tree.head_idx), ops._p(tree.rank), ops._p(topk), topk.shape[1],
           ops._p(root), ops._p(tokens), ops._stream())


# ---------------------------------------------------------- sampled regime
def sample_without_replacement(logits: torch.Tensor, num_samples: int, temperature: float = 0.0,
                               generator: torch.Generator | None = None) -> torch.Tensor:
    """speculative/sampling.py:20-81: greedy top-k at temperature <= 1e-6,
    else Gumbel-top-k over logits / T with uniforms from ``generator`` (drawn
    on the CPU when the generator lives there, as the reference does on a
    device it cannot draw on)."""
    V = logits.size(-1)
    k = max(0, min(num_samples, V))
    if k == 0:
        return torch.empty(list(logits.shape[:-1]) + [0], dtype=torch.long, device=logits.device)
    if temperature <= 1e-6:
        return torch.topk(logits, k=k, dim=-1).indices
    u = _uniform(logits.shape, logits.device, generator)
    u = u.clamp(min=1e-10, max=1.0 - 1e-10)
    gumbel = -torch.log(-torch.log(u))
    return torch.topk(logits.float() / temperature + gumbel, k=k, dim=-1).indices


def _uniform(shape, device, generator):
    if generator is None:
        return torch.rand(shape, device=device, dtype=torch.float32)
    try:
        return torch.rand(shape, device=device, generator=generator, dtype=torch.float32)
    except RuntimeError:
        return torch.rand(shape, device="cpu", generator=generator, dtype=torch.float32).to(device)


@dataclass
class VerificationStepResult:
    """speculative/sampling.py:84-93."""

    accepted: bool
    accepted_token: int
    accepted_candidate_idx: int | None
    is_fallback: bool
    rejected_tokens: list[int] = field(default_factory=list)
    acceptance_probs: list[float] = field(default_factory=list)


class SequoiaTreeVerifier:
    """speculative/sampling.py:96-376: Sequoia's Algorithm 2, candidates
    sampled without replacement verified against the target distribution
    with the exact residual update P <- (P - Q)+ / |(P - Q)+|.  Host logic
    over (device) logits; random draws come from ``generator`` in the
    reference's order."""

    def __init__(self, temperature: float = 0.0, generator: torch.Generator | None = None):
        self.temperature = float(temperature)
        self.generator = generator

    def _rand_scalar(self, device) -> float:
        return float(_uniform((), device, self.generator).item())

    def _multinomial_scalar(self, probs: torch.Tensor) -> int:
        p = probs.to(device="cpu", dtype=torch.float32)
        if self.generator is not None:
            try:
                return int(torch.multinomial(p, num_samples=1, generator=self.generator).item())
            except RuntimeError:
                pass
        return int(torch.multinomial(p, num_samples=1).item())

    def verify_candidates(self, target_logits: torch.Tensor, candidates: list[int],
                          draft_logits: torch.Tensor | None = None,
                          temperature: float | None = None) -> VerificationStepResult:
        """sampling.py:146-269 for the K candidates of one node."""
        temp = self.temperature if temperature is None else float(temperature)
        K = len(candidates)
        if temp <= 1e-6:  # greedy: only the first candidate is tested
            best = int(target_logits.argmax(dim=-1).item())
            if K > 0 and candidates[0] == best:
                return VerificationStepResult(True, candidates[0], 0, False, [], [1.0])
            return VerificationStepResult(False, best, None, True, [candidates[0]] if K else [], [0.0] if K else [])
        V = target_logits.size(-1)
        p = F.softmax(target_logits.float() / temp, dim=-1)
        if draft_logits is not None:
            q = F.softmax(draft_logits.float() / temp, dim=-1)
        else:
            q = torch.zeros_like(p)
            if K:
                q[candidates] = 1.0 / K
        rejected: list[int] = []
        alphas: list[float] = []
        for i, cand in enumerate(candidates):
            pv, qv = p[cand].item(), q[cand].item()
            alpha = min(1.0, max(0.0, pv / max(1e-9, qv)))
            alphas.append(alpha)
            if self._rand_scalar(target_logits.device) <= alpha:
                return VerificationStepResult(True, cand, i, False, rejected, alphas)
            rejected.append(cand)
            resid = torch.clamp(p - q, min=0.0)
            mass = resid.sum().item()
            if mass <= 1e-9:  # target residual exhausted: the candidate stands
                return VerificationStepResult(True, cand, i, False, rejected[:-1], alphas)
            p = resid / mass
            q[cand] = 0.0
            qm = q.sum().item()
            q = q / qm if qm > 1e-9 else torch.ones_like(q) / V
        return VerificationStepResult(False, self._multinomial_scalar(p), None, True, rejected, alphas)

    def verify_tree_step(self, tree_logits: torch.Tensor, compiled_tree: dict[str, Any], verif_seq: list[int],
                         medusa_logits_leaf=None, temperature: float | None = None,
                         max_accept: int | None = None):
        """sampling.py:271-376: walk from the root verifying each node's
        children (in order) as one candidate set; returns (accepted nodes,
        emitted tokens, stats)."""
        temp = self.temperature if temperature is None else float(temperature)
        children = compiled_tree["children"]
        limit = max_accept if max_accept is not None else len(verif_seq)
        cur, accepted, emitted = 0, [0], []
        tested = acc_total = 0
        attempts: list[int] = []
        rejections: list[int] = []
        while len(emitted) < limit:
            kids = children[cur]
            logits = tree_logits[cur]
            if not kids:  # a leaf: the final token comes from the target alone
                if temp <= 1e-6:
                    emitted.append(int(logits.argmax(dim=-1).item()))
                else:
                    emitted.append(self._multinomial_scalar(F.softmax(logits.float() / temp, dim=-1)))
                break
            cands = [verif_seq[c] for c in kids]
            res = self.verify_candidates(logits, cands, None, temp)
            tested += len(cands)
            emitted.append(res.accepted_token)
            while len(attempts) < len(cands):
                attempts.append(0)
                rejections.append(0)
            for r in range(len(cands)):
                attempts[r] += 1
                if not (res.accepted and res.accepted_candidate_idx == r):
                    rejections[r] += 1
            if not (res.accepted and res.accepted_candidate_idx is not None):
                break
            cur = kids[res.accepted_candidate_idx]
            accepted.append(cur)
            acc_total += 1
        stats = {
            "tested_candidates": tested,
            "accepted_draft_tokens": acc_total,
            "rejection_rates_per_rank": [rejections[i] / attempts[i] if attempts[i] else 0.0
                                         for i in range(len(attempts))],
            "emitted_count": len(emitted),
        }
        return accepted, emitted, stats


def fit_power_law_rejection_bound(rejection_rates: list[float]) -> dict[str, float]:
    """sampling.py:378-446: least-squares fit of ln r_k = ln a - b ln k over
    the rates strictly inside (1e-6, 1 - 1e-6)."""
    pts = [(math.log(k), math.log(r)) for k, r in enumerate(rejection_rates, start=1) if 1e-6 < r < 1.0 - 1e-6]
    if len(pts) < 2:
        return {"exponent_b": 0.0, "scale_a": 1.0, "r_squared": 0.0, "valid": False}
    n = len(pts)
    mx = sum(x for x, _ in pts) / n
    my = sum(y for _, y in pts) / n
    sxx = sum((x - mx) ** 2 for x, _ in pts)
    syy = sum((y - my) ** 2 for _, y in pts)
    sxy = sum((x - mx) * (y - my) for x, y in pts)
    if sxx < 1e-12:
        return {"exponent_b": 0.0, "scale_a": math.exp(my), "r_squared": 0.0, "valid": False}
    slope = sxy / sxx
    return {"exponent_b": float(-slope), "scale_a": float(math.exp(my - slope * mx)),
            "r_squared": float(sxy * sxy / (sxx * syy)) if syy > 1e-12 else 1.0, "valid": True}


# ----------------------------------------------------------------- decoder
class MedusaSpeculativeDecoder:
    """engine/medusa.py:119-537 over a ``QuantizedDecoder`` with
    ``medusa_heads`` attached (``decoder.add_medusa_heads``).  Batch 1."""

    def __init__(self, num_heads: int = 3, temperature: float = 0.0, tree_choices=None, max_nodes: int = 32):
        self.num_heads = num_heads
        self.temperature = temperature
        self.tree_choices = tree_choices
        self.max_nodes = max_nodes

    @torch.no_grad()
    def generate(self, model, prompt_tokens: list[int], max_new_tokens: int = 64, cache=None, device=None,
                 tree_choices=None, temperature: float | None = None, generator: torch.Generator | None = None):
        """Returns (prompt + generated tokens, stats) like the reference.  With
        ``cache`` None the decoder's cache starts empty; passing the
        decoder's own ``cache`` continues from its contents.  At temperature
        0 the stats add ``accepted_nodes``: the accepted node ids of every
        verification pass."""
        heads: MedusaHeads | None = getattr(model, "medusa_heads", None)
        if heads is None or heads.num_heads == 0:
            raise ValueError("Model does not have Medusa heads attached. Call model.add_medusa_heads() first.")
        if cache is None:
            model.cache.reset()
        elif cache is not model.cache:
            raise ValueError("the decoder serves its own StaticKVCache; pass model.cache or None")
        temp = float(self.temperature if temperature is None else temperature)
        choices = tree_choices if tree_choices is not None else self.tree_choices
        K = heads.num_heads
        tree = compile_medusa_tree(choices, K, self.max_nodes) if choices is not None else None
        use_tree = tree is not None and tree["num_nodes"] > 1
        if use_tree and tree["num_nodes"] > model.max_tokens:
            raise ValueError(f"tree of {tree['num_nodes']} nodes exceeds the runner's max_tokens {model.max_tokens}")
        if K + 1 > model.max_tokens:
            raise ValueError("the linear chain needs max_tokens >= num_heads + 1")
        if temp <= 1e-6:
            return self._generate_greedy(model, heads, list(prompt_tokens), max_new_tokens, tree, use_tree)
        return self._generate_sampled(model, heads, list(prompt_tokens), max_new_tokens, tree, use_tree, temp,
                                      generator)

    # ---- shared pieces
    @staticmethod
    def _prefill(model, prompt: list[int]) -> int:
        """Runs the prompt; returns the runner row of its last token."""
        ids = torch.tensor([prompt], dtype=torch.long, device=model.device)
        model.prefill(ids)
        T = len(prompt)
        return T - (T - 1) // model.max_tokens * model.max_tokens - 1

    @staticmethod
    def _stats(prompt_len, generated, elapsed, calls, drafted, accepted, nodes, temp, rank_rej):
        new = len(generated) - prompt_len
        avg_rej = [float(sum(v) / len(v)) for v in rank_rej if v]
        return {
            "new_tokens": new,
            "elapsed_seconds": elapsed,
            "tokens_per_second": new / elapsed if elapsed > 0 else 0.0,
            "ms_per_token": elapsed / new * 1000.0 if new > 0 else 0.0,
            "forward_calls": calls,
            "tokens_per_forward_call": new / calls if calls > 0 else 0.0,
            "mean_accepted_length": new / calls if calls > 0 else 0.0,
            "tree_nodes_per_step": nodes,
            "drafted_tokens": drafted,
            "accepted_draft_tokens": accepted,
            "acceptance_rate_pct": accepted / drafted * 100.0 if drafted > 0 else 0.0,
            "temperature": temp,
            "rejection_rates_per_rank": avg_rej,
            "power_law_fit": fit_power_law_rejection_bound(avg_rej),
        }

    # ---- temperature 0: the device pipeline
    def _generate_greedy(self, model, heads: MedusaHeads, prompt, max_new, tree, use_tree):
        dev = model.device
        cache = model.cache
        dtree = DeviceTree(tree, dev) if use_tree else None
        chain = DeviceTree(chain_tree(heads.num_heads), dev)
        kmax = dtree.kmax if use_tree else 1
        result = torch.zeros(L.TREE_RESULT_WORDS, dtype=torch.int32, device=dev)
        host = torch.zeros(L.TREE_RESULT_WORDS, dtype=torch.int32, pin_memory=True)
        done = torch.cuda.Event()
        K = heads.num_heads

        row = self._prefill(model, prompt)
        root = model.argmax_buf[row:row + 1]
        topk = heads.draft(model.norm_buf, kmax, leaf=row)
        first = torch.cat([root, topk[:, 0]]).cpu().tolist()  # the prefill's token and per-head argmax
        generated = prompt + [first[0]]
        draft_candidates = first[1:]
        draft_tokens(dtree if use_tree else chain, topk, root, model.tokens)
        target = len(prompt) + max_new
        calls, drafted, accepted_total = 1, 0, 0
        # engine/medusa.py:383-418: once the tree no longer fits the cache the
        # chain takes over, its first draft being the prefill-time per-head
        # argmax (the tree steps never refresh those); later chain drafts come
        # from the heads at the last accepted node
        linear_started = False
        trace: list[list[int]] = []  # accepted node ids of every verification pass
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        while len(generated) < target:
            seen = cache.total_seen_tokens[0]
            if use_tree and seen + dtree.T <= cache.max_seq_len:
                dt, T = dtree, dtree.T
                step_draft = min(tree["max_depth"], target - len(generated))
            else:
                k_cand = min(K, target - len(generated))
                dt, T = chain, k_cand + 1
                step_draft = k_cand
                if use_tree and not linear_started:
                    stale = torch.tensor([generated[-1]] + draft_candidates[:k_cand], dtype=torch.int32)
                    model.tokens[:T].copy_(stale)
                    linear_started = True
            budget = target - len(generated)
            model.forward_tree_verify_device(T, dt.depths[:T], dt.masks[:T])
            calls += 1
            drafted += step_draft
            L.call("axb_tree_accept", T, ops._p(dt.parent), ops._p(model.tokens), ops._p(model.argmax_buf),
                   budget, ops._p(result), ops._stream())
            model.compact_device(seen, result)
            host.copy_(result, non_blocking=True)
            done.record()
            # the next draft's heads run while the host reads the result
            topk = heads.draft(model.norm_buf, kmax, leaf_dev=result[1:2])
            done.synchronize()
            n = int(host[0])
            e0 = L.TREE_RESULT_HDR + L.TREE_MAX_NODES
            generated.extend(host[e0:e0 + n].tolist())
            trace.append(host[L.TREE_RESULT_HDR:L.TREE_RESULT_HDR + n].tolist())
            accepted_total += max(0, n - 1)
            cache.advance(seen + n)
            if len(generated) >= target:
                break
            if use_tree and seen + n + dtree.T <= cache.max_seq_len:
                draft_tokens(dtree, topk, result[3:4], model.tokens)
            elif not use_tree or linear_started:
                draft_tokens(chain, topk, result[3:4], model.tokens)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        nodes = tree["num_nodes"] if use_tree else 1 + K
        stats = self._stats(len(prompt), generated, elapsed, calls, drafted, accepted_total, nodes, 0.0, [])
        stats["accepted_nodes"] = trace
        return generated, stats

    # ---- temperature > 0: host logic over the device logits
    def _generate_sampled(self, model, heads: MedusaHeads, prompt, max_new, tree, use_tree, temp, generator):
        cache = model.cache
        verifier = SequoiaTreeVerifier(temperature=temp, generator=generator)
        K = heads.num_heads
        row = self._prefill(model, prompt)
        base = model.logits_buf[row].float()
        probs = torch.softmax(base / temp, dim=-1).cpu()
        next_tok = int(torch.multinomial(probs, 1, generator=generator).item()) if generator is not None else \
            int(torch.multinomial(probs, 1).item())
        generated = prompt + [next_tok]
        target = len(prompt) + max_new
        med = heads(model.norm_buf[row:row + 1].view(1, 1, -1))

        def tree_topk(med_list, pos):
            return [sample_without_replacement(med_list[h][0, pos, :], min(tree["max_topk_per_head"][h], heads.vocab),
                                               temp, generator).tolist() for h in range(K)]

        draft = [int(sample_without_replacement(med[k][:, -1, :], 1, temp, generator).squeeze(-1).item())
                 for k in range(K)]
        ttopk = tree_topk(med, -1) if use_tree else []
        calls, drafted, acc_total = 1, 0, 0
        rank_rej: list[list[float]] = []
        t0 = time.perf_counter()
        while len(generated) < target:
            seen = cache.total_seen_tokens[0]
            if use_tree and seen + tree["num_nodes"] <= cache.max_seq_len:
                T = tree["num_nodes"]
                verif = [generated[-1]] + [ttopk[tree["head_idx"][u]][min(tree["topk_rank"][u],
                                                                           len(ttopk[tree["head_idx"][u]]) - 1)]
                                           for u in range(1, T)]
                logits = model.forward_tree_verify(torch.tensor([verif], device=model.device),
                                                   tree["tree_depths"], tree["tree_mask"])
                calls += 1
                drafted += min(tree["max_depth"], target - len(generated))
                acc_nodes, emitted, st = verifier.verify_tree_step(logits[0], tree, verif, temperature=temp,
                                                                   max_accept=target - len(generated))
                generated.extend(emitted)
                for r, rate in enumerate(st["rejection_rates_per_rank"]):
                    while len(rank_rej) <= r:
                        rank_rej.append([])
                    rank_rej[r].append(rate)
                acc_total += max(0, len(acc_nodes) - 1)
                cache.compact_tree_path(seen, acc_nodes, seen + len(acc_nodes))
                if len(generated) >= target:
                    break
                leaf = acc_nodes[-1]
                ttopk = tree_topk(heads(model.norm_buf[leaf:leaf + 1].view(1, 1, -1)), 0)
                continue
            k_cand = min(len(draft), target - len(generated))
            if k_cand <= 0:
                break
            cand = draft[:k_cand]
            verif = [generated[-1]] + cand
            T = len(verif)
            logits = model.forward_tree_verify(torch.tensor([verif], device=model.device), list(range(T)),
                                               [(1 << (u + 1)) - 1 for u in range(T)])
            calls += 1
            drafted += k_cand
            n_acc = last = 0
            for j in range(k_cand):
                res = verifier.verify_candidates(logits[0, j], [cand[j]], None, temp)
                generated.append(res.accepted_token)
                n_acc += 1
                last = j
                if not res.accepted or len(generated) >= target:
                    break
            acc_total += max(0, n_acc - 1)
            cache.advance(seen + n_acc)
            if len(generated) >= target:
                break
            med = heads(model.norm_buf[last:last + 1].view(1, 1, -1))
            draft = [int(sample_without_replacement(med[k][0, 0], 1, temp, generator).item()) for k in range(K)]
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        nodes = tree["num_nodes"] if use_tree else 1 + K
        return generated, self._stats(len(prompt), generated, elapsed, calls, drafted, acc_total, nodes, temp,
                                      rank_rej)
