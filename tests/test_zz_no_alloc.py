"""GPU test of the allocation-free cross-entropy entry point.

``oxi_linear_ce_fwd_noalloc`` serves callers that cannot allocate device
memory themselves (a runtime that reserves all device memory up front, or
code that must not let cudaMalloc/cudaFree synchronise the device): it keeps
its scratch in a fixed file-scope device array.  This test calls it through
its exported C symbol and compares it with the regular entry point (which
uses caller-allocated scratch), on two calls in a row so that the contents
left in the shared scratch by the first call cannot leak into the second.

The file name makes pytest collect it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from oxidizr_b200 import _ext
    _ext.load()  # build/load the extension module first
    lib = ctypes.CDLL(_ext.so_path())
    f = lib.oxi_linear_ce_fwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                  ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_void_p]
    lib.oxi_linear_ce_noalloc_last_error.restype = ctypes.c_char_p
    lib.oxi_linear_ce_noalloc_status.restype = ctypes.c_int
    lib.oxi_linear_ce_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_int)]
    return lib


def _status(lib):
    word = ctypes.c_int(-1)
    rc = lib.oxi_linear_ce_noalloc_status(ctypes.byref(word))
    return rc, word.value


def _regular(x, w, tg):
    """The existing entry point: caller-allocated partials + finish kernel."""
    from oxidizr_b200.ops._C import ext, status
    M, V = x.shape[0], w.shape[0]
    nt = (V + 255) // 256
    pm = torch.empty(M, nt, device="cuda")
    ps = torch.empty_like(pm)
    tl = torch.zeros(M, device="cuda")
    ext().gemm_ce(x, w, tg, pm, ps, tl, None, 1.0, status("cuda"))
    lse = torch.empty(M, device="cuda")
    loss = torch.empty(M, device="cuda")
    ext().ce_finish(pm, ps, tl, tg, lse, loss)
    return loss, lse


def _noalloc(lib, x, w, tg):
    M, K = x.shape
    V = w.shape[0]
    loss = torch.full((M,), float("nan"), device="cuda")
    lse = torch.full((M,), float("nan"), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.oxi_linear_ce_fwd_noalloc(x.data_ptr(), M, K, x.stride(0), w.data_ptr(), V, w.stride(0),
                                       tg.data_ptr(), loss.data_ptr(), lse.data_ptr(), st)
    assert rc == 0, lib.oxi_linear_ce_noalloc_last_error()
    return loss, lse


def test_noalloc_matches_regular_entry_point_twice():
    lib = _lib()
    torch.manual_seed(11)
    cases = [(300, 256, 5003), (1000, 512, 4099)]
    for i, (M, K, V) in enumerate(cases):
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn(V, K, device="cuda") / K ** 0.5).bfloat16()
        tg = torch.randint(0, V, (M,), device="cuda")
        tg[::7] = -1  # ignored rows
        ref_loss, ref_lse = _regular(x, w, tg)
        loss, lse = _noalloc(lib, x, w, tg)
        torch.cuda.synchronize()
        assert torch.allclose(loss, ref_loss, atol=1e-4, rtol=1e-4), f"call {i}"
        assert torch.allclose(lse, ref_lse, atol=1e-4, rtol=1e-4), f"call {i}"
        # and against the fp32 PyTorch statement of the same math
        logits = x.float() @ w.float().t()
        full = torch.logsumexp(logits, -1)
        assert torch.allclose(lse, full, atol=2e-3, rtol=1e-4)
        valid = tg >= 0
        ce = full - logits.gather(1, tg.clamp_min(0)[:, None])[:, 0]
        assert torch.allclose(loss[valid], ce[valid], atol=2e-3, rtol=1e-3)
        assert torch.all(loss[~valid] == 0)
        # the kernels recorded no error (status word read back after the sync)
        assert _status(lib) == (0, 0), lib.oxi_linear_ce_noalloc_last_error()


def test_noalloc_rejects_oversized_problem():
    lib = _lib()
    M, K, V = 70000, 64, 1000  # more rows than the fixed scratch holds
    x = torch.empty(8, K, device="cuda", dtype=torch.bfloat16)
    w = torch.empty(V, K, device="cuda", dtype=torch.bfloat16)
    tg = torch.zeros(8, device="cuda", dtype=torch.int64)
    out = torch.empty(8, device="cuda")
    rc = lib.oxi_linear_ce_fwd_noalloc(x.data_ptr(), M, K, K, w.data_ptr(), V, K, tg.data_ptr(), out.data_ptr(),
                                       out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"too large" in lib.oxi_linear_ce_noalloc_last_error()


def _raw_call(lib, x_ptr, M, K, ldx, w_ptr, V, ldw, tg_ptr, loss_ptr, lse_ptr):
    return lib.oxi_linear_ce_fwd_noalloc(x_ptr, M, K, ldx, w_ptr, V, ldw, tg_ptr, loss_ptr, lse_ptr,
                                         torch.cuda.current_stream().cuda_stream)


def test_noalloc_argument_paths_launch_nothing():
    """Zero rows, bad strides, null pointers and the partials limit are
    answered before any kernel is queued; outputs stay untouched."""
    lib = _lib()
    K, V = 64, 1000
    x = torch.zeros(8, K, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(V, K, device="cuda", dtype=torch.bfloat16)
    tg = torch.zeros(8, device="cuda", dtype=torch.int64)
    loss = torch.full((8,), 7.0, device="cuda")
    lse = torch.full((8,), 7.0, device="cuda")
    args = (x.data_ptr(), 8, K, K, w.data_ptr(), V, K, tg.data_ptr(), loss.data_ptr(), lse.data_ptr())
    # M = 0: nothing to do
    a = list(args)
    a[1] = 0
    assert _raw_call(lib, *a) == 0
    # row stride shorter than a row
    a = list(args)
    a[3] = K - 8
    assert _raw_call(lib, *a) == 2
    # null output pointer
    a = list(args)
    a[8] = None
    assert _raw_call(lib, *a) == 2
    # rows within the row limit but M * ceil(V / 256) partials beyond the partials limit
    max_rows, max_part = ctypes.c_int64(), ctypes.c_int64()
    lib.oxi_linear_ce_noalloc_limits(ctypes.byref(max_rows), ctypes.byref(max_part))
    M = 60000
    Vbig = 256 * (max_part.value // M + 1)
    assert M <= max_rows.value and M * (Vbig // 256) > max_part.value
    a = list(args)
    a[1], a[5] = M, Vbig
    assert _raw_call(lib, *a) == 1
    assert b"too large" in lib.oxi_linear_ce_noalloc_last_error()
    torch.cuda.synchronize()
    assert torch.all(loss == 7.0) and torch.all(lse == 7.0)
