"""The allocation-free RMSNorm backward entry point, called through its C symbol.

Some hosts cannot let a library allocate device memory on its own schedule
(a fixed device-memory budget, or a calling context where a driver
allocation could block or fail); ``ts_rms_norm_bwd_noalloc`` serves them by
keeping its scratch in a fixed device array. This test checks it against the
regular entry point on two calls in a row. The file is collected last on
purpose, so a failure here never hides the other tests.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from thundersync_b200.ops._ext import native, so_path

    native()  # make sure the extension (and its device code) is loaded
    lib = ctypes.CDLL(so_path())
    fn = lib.ts_rms_norm_bwd_noalloc
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    err = lib.ts_noalloc_last_error
    err.restype = ctypes.c_char_p
    return fn, err


def test_noalloc_rms_norm_backward_matches_regular_entry_point():
    from thundersync_b200.ops._ext import native

    fn, err = _lib()
    torch.manual_seed(11)
    for call, (rows, cols) in enumerate([(1000, 2048), (333, 4096)]):
        x = torch.randn(rows, cols, device="cuda", dtype=torch.bfloat16)
        w = (1 + 0.1 * torch.randn(cols, device="cuda")).to(torch.bfloat16)
        dy = torch.randn(rows, cols, device="cuda", dtype=torch.bfloat16)
        _, rstd = native().rms_norm_fwd(x, w, 1e-6, False)
        dx_ref, dw_ref = native().rms_norm_bwd(dy, x, w, rstd, False)
        dx = torch.empty_like(x)
        dw = torch.empty(cols, device="cuda", dtype=torch.float32)
        stream = torch.cuda.current_stream().cuda_stream
        rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(),
                rows, cols, 0, stream)
        assert rc == 0, err()
        torch.cuda.synchronize()
        assert torch.equal(dx, dx_ref), f"call {call}: dx differs"
        torch.testing.assert_close(dw, dw_ref, rtol=1e-5, atol=1e-5, msg=f"call {call}: dw differs")


def test_noalloc_rejects_sizes_beyond_its_scratch():
    fn, err = _lib()
    x = torch.zeros(4, 4104, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(4104, device="cuda", dtype=torch.float32)
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), out.data_ptr(), x.data_ptr(), out.data_ptr(), 4, 4104, 0,
            torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"limit" in err()
