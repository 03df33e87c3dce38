"""axb_qgemm_noalloc: the GEMV entry point for callers that cannot allocate
device memory (hosts that reserve the device in their own pool, plugin/FFI
hosts without an allocator, latency-critical paths).  Its scratch is an array
inside the library, so the caller passes no workspace.

Checked against the regular entry point (axb_qgemm with a caller workspace)
through the C ABI, two calls in a row per case.  Both run the same
deterministic kernel on the same grid, so the outputs must be bit-identical.
The cases cover the plain store, the fused RMSNorm staging, the SwiGLU
epilogue over gate/up-interleaved weights, a dependent (PDL) launch, and
repeated same-shape calls whose tiles are split across CTAs (the tile
counters in the shared array must return to zero between calls).

Kept in a file of its own that pytest collects last."""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _desc(L, W, x, y, ws=None, norm_w=None, epilogue=None, gate_up=0, pdl=0):
    return L.QGemmDesc(fmt=W.fmt, group=W.group, words=W.words.data_ptr(), scales=W.scales.data_ptr(), N=W.N,
                       K=W.K, M=x.shape[0], x=x.data_ptr(), ldx=W.K, y=y.data_ptr(), ldy=y.shape[1], bias=None,
                       norm_w=None if norm_w is None else norm_w.data_ptr(), eps=1e-5,
                       epilogue=L.EPI_STORE if epilogue is None else epilogue, gate_up_interleave=gate_up,
                       workspace=None if ws is None else ws.data_ptr(),
                       workspace_bytes=0 if ws is None else ws.numel(), pdl=pdl)


CASES = [
    # N, K, M, group, sym, kind, pdl
    (4096, 4096, 1, 128, True, "store", 0),
    (2003, 1024, 5, 64, False, "store", 0),
    (4096, 4096, 3, 128, True, "norm", 0),
    (2 * 1792, 4096, 2, 128, True, "swiglu", 0),
    (4096, 4096, 1, 128, True, "store", 1),
    (28672, 4096, 8, 128, True, "store", 0),
]


@pytest.mark.parametrize("N,K,M,group,sym,kind,pdl", CASES)
def test_noalloc_gemv_matches_workspace_entry_point(N, K, M, group, sym, kind, pdl):
    from axiomlm_b200 import _lib as L
    from axiomlm_b200 import ops

    lib = L.load()
    assert lib.axb_check_device() == 0
    assert lib.axb_qgemm_noalloc_scratch_bytes() > 0
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator(device="cuda").manual_seed(N + K + M)
    W = ops.pack_q4t(torch.randn(N, K, device="cuda", generator=g) * 0.02, group, sym, gate_up=(kind == "swiglu"))
    norm_w = torch.rand(K, device="cuda", generator=g) + 0.5 if kind == "norm" else None
    epi = L.EPI_SWIGLU if kind == "swiglu" else L.EPI_STORE
    n_out = N // 2 if kind == "swiglu" else N
    ws = torch.zeros(lib.axb_qgemm_workspace_bytes(N, K, M, group), dtype=torch.uint8, device="cuda")
    for call in range(2):  # two calls in a row: the shared array must be reusable
        x = torch.randn(M, K, device="cuda", generator=g).half()
        y_na = torch.full((M, n_out), float("nan"), dtype=torch.float16, device="cuda")
        y_ws = torch.full((M, n_out), float("nan"), dtype=torch.float16, device="cuda")
        kw = dict(norm_w=norm_w, epilogue=epi, gate_up=int(kind == "swiglu"), pdl=pdl)
        assert lib.axb_qgemm_noalloc(C.byref(_desc(L, W, x, y_na, **kw)), stream) == 0, lib.axb_last_error()
        assert lib.axb_qgemm(C.byref(_desc(L, W, x, y_ws, ws, **kw)), stream) == 0, lib.axb_last_error()
        assert lib.axb_qgemm_noalloc_status(stream) == 0, lib.axb_last_error()
        assert lib.axb_qgemm_status(C.c_void_p(ws.data_ptr()), stream) == 0, lib.axb_last_error()
        assert not torch.isnan(y_ws).any(), (call, "workspace entry point left outputs unwritten")
        assert torch.equal(y_na, y_ws), (N, K, M, kind, call,
                                         float((y_na.float() - y_ws.float()).abs().max()))


def test_noalloc_rejects_oversize_batch():
    from axiomlm_b200 import _lib as L
    from axiomlm_b200 import ops

    lib = L.load()
    W = ops.pack_q4t(torch.randn(64, 256, device="cuda") * 0.02, 128, True)
    x = torch.randn(9, 256, device="cuda").half()
    y = torch.empty(9, 64, dtype=torch.float16, device="cuda")
    rc = lib.axb_qgemm_noalloc(C.byref(_desc(L, W, x, y)), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == L.AXB_EINVAL and b"M must be" in lib.axb_last_error()
