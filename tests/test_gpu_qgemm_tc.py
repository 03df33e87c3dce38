"""The tcgen05 W4A16 GEMM (large-M path: tree verification, prefill, decode
batches) through the C ABI, against an fp32 evaluation of the dequantized
weights (relative error < 2e-3 of the output's max magnitude) and against the
warp-level GEMV on the same inputs."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


@pytest.fixture(scope="module")
def ax():
    from axiomlm_b200 import _lib, ops

    assert _lib.load().axb_check_device() == 0, "not an sm_100 device"
    return ops


def _rel(y, ref):
    y, ref = y.float().cpu(), ref.float().cpu()
    return float((y - ref).abs().max() / ref.abs().max().clamp(min=1e-6))


def _case(ax, N, K, M, sym, bias=False, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * 0.02
    W = ax.pack_q4t(w.cuda(), 128 if sym else 64, sym)
    x = torch.randn(M, K, generator=g).half()
    b = (torch.randn(N, generator=g) * 0.1).half() if bias else None
    y = ax.qgemm_tc(x.cuda(), W, bias=None if b is None else b.cuda())
    assert ax.qgemm_tc_status() == 0
    ref = x.float() @ W.dequant().float().cpu().t()
    if b is not None:
        ref = ref + b.float()
    return y, ref, W, x


def test_smallest_case(ax):
    y, ref, _, _ = _case(ax, 128, 128, 16, True)
    assert _rel(y, ref) < REL_TOL, _rel(y, ref)


@pytest.mark.parametrize("sym", [True, False])
@pytest.mark.parametrize("M", [1, 16, 33, 64])
def test_against_dequant(ax, sym, M):
    y, ref, _, _ = _case(ax, 2003, 768, M, sym, bias=True, seed=M)
    assert _rel(y, ref) < REL_TOL, f"sym={sym} M={M}: rel {_rel(y, ref):.2e}"


@pytest.mark.parametrize("N,K", [(4096, 4096), (6144, 4096), (4096, 14336)])
def test_split_k_shapes(ax, N, K):
    """8B projection shapes: few 128-row blocks, so K is split across CTAs
    and the partials meet in split order."""
    y, ref, W, x = _case(ax, N, K, 64, True, seed=N + K)
    assert _rel(y, ref) < REL_TOL, f"{N}x{K}: rel {_rel(y, ref):.2e}"
    # deterministic, and the split counters are back at zero for the next call
    y2 = ax.qgemm_tc(x.cuda(), W)
    assert torch.equal(y, y2)


def test_matches_warp_level_gemv(ax):
    y, _, W, x = _case(ax, 1024, 1024, 64, True, seed=5)
    y_mma = ax.qgemm(x.cuda(), W)
    assert _rel(y, y_mma) < REL_TOL


def test_more_than_64_tokens_chunked(ax):
    y, ref, _, _ = _case(ax, 512, 512, 100, True, seed=9)
    assert _rel(y, ref) < REL_TOL


@pytest.mark.parametrize("N,K", [(256, 448), (2003, 320), (130, 64)])
def test_odd_k_block_counts(ax, N, K):
    """Splits whose k-block count is odd (a ring slot holding a single k-block),
    a single k-block in all, and a row count that ends inside a tile."""
    y, ref, _, _ = _case(ax, N, K, 40, False, bias=True, seed=N)
    assert _rel(y, ref) < REL_TOL, f"{N}x{K}: rel {_rel(y, ref):.2e}"
