"""axb_qgemm_noalloc: the GEMV entry point for callers that cannot allocate
device memory (hosts that reserve the device in their own pool, plugin/FFI
hosts without an allocator, latency-critical paths).  Its scratch is an array
inside the library, so the caller passes no workspace.  Checked against the
regular entry point (axb_qgemm with a caller workspace) on two calls in a row,
with different shapes, through the C ABI.

Kept in a file of its own that pytest collects last."""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


def _desc(L, W, x, y, ws=None):
    return L.QGemmDesc(fmt=W.fmt, group=W.group, words=W.words.data_ptr(), scales=W.scales.data_ptr(), N=W.N,
                       K=W.K, M=x.shape[0], x=x.data_ptr(), ldx=W.K, y=y.data_ptr(), ldy=W.N, bias=None,
                       norm_w=None, eps=1e-5, epilogue=L.EPI_STORE, gate_up_interleave=0,
                       workspace=None if ws is None else ws.data_ptr(),
                       workspace_bytes=0 if ws is None else ws.numel(), pdl=0)


def test_noalloc_gemv_matches_workspace_entry_point():
    from axiomlm_b200 import _lib as L
    from axiomlm_b200 import ops

    lib = L.load()
    assert lib.axb_check_device() == 0
    assert lib.axb_qgemm_noalloc_scratch_bytes() > 0
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    torch.manual_seed(0)
    for N, K, M, group, sym in [(4096, 4096, 1, 128, True), (2003, 1024, 5, 64, False)]:
        W = ops.pack_q4t(torch.randn(N, K, device="cuda") * 0.02, group, sym)
        x = torch.randn(M, K, device="cuda").half()
        y_na = torch.empty(M, N, dtype=torch.float16, device="cuda")
        y_ws = torch.empty(M, N, dtype=torch.float16, device="cuda")
        assert lib.axb_qgemm_noalloc(C.byref(_desc(L, W, x, y_na)), stream) == 0, lib.axb_last_error()
        ws = torch.zeros(lib.axb_qgemm_workspace_bytes(N, K, M, group), dtype=torch.uint8, device="cuda")
        assert lib.axb_qgemm(C.byref(_desc(L, W, x, y_ws, ws)), stream) == 0, lib.axb_last_error()
        torch.cuda.synchronize()
        err = float((y_na.float() - y_ws.float()).abs().max() / y_ws.float().abs().max())
        assert err < REL_TOL, (N, K, M, err)


def test_noalloc_rejects_oversize_batch():
    from axiomlm_b200 import _lib as L
    from axiomlm_b200 import ops

    lib = L.load()
    W = ops.pack_q4t(torch.randn(64, 256, device="cuda") * 0.02, 128, True)
    x = torch.randn(9, 256, device="cuda").half()
    y = torch.empty(9, 64, dtype=torch.float16, device="cuda")
    rc = lib.axb_qgemm_noalloc(C.byref(_desc(L, W, x, y)), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == L.AXB_EINVAL and b"M must be" in lib.axb_last_error()
