"""The allocation-free RMSNorm backward entry point, called through its C symbol.

Some hosts cannot let a library allocate device memory on its own schedule
(a fixed device-memory budget, or a calling context where a driver
allocation could block or fail); ``ts_rms_norm_bwd_noalloc`` serves them by
keeping its scratch in a fixed device array. This test checks it against the
regular entry point on two calls in a row, for bf16 and fp32 rows, and checks
that what it cannot serve is refused on the host before anything launches.
The file is collected last on purpose, so a failure here never hides the
other tests.
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


def _call(fn, dy, x, w, rstd, dx, dw, rows, cols, dtype_code):
    return fn(dy, x, w, rstd, dx, dw, rows, cols, dtype_code, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("dtype,code,shapes", [
    (torch.bfloat16, 0, [(1000, 2048), (333, 4096)]),
    (torch.float32, 1, [(257, 1024), (64, 2048)]),
])
def test_noalloc_rms_norm_backward_matches_regular_entry_point(dtype, code, shapes):
    from thundersync_b200.ops._ext import native

    fn, err = _lib()
    torch.manual_seed(11)
    for call, (rows, cols) in enumerate(shapes):
        x = torch.randn(rows, cols, device="cuda", dtype=dtype)
        w = (1 + 0.1 * torch.randn(cols, device="cuda")).to(dtype)
        dy = torch.randn(rows, cols, device="cuda", dtype=dtype)
        _, rstd = native().rms_norm_fwd(x, w, 1e-6, False)
        dx_ref, dw_ref = native().rms_norm_bwd(dy, x, w, rstd, False)
        dx = torch.empty_like(x)
        dw = torch.empty(cols, device="cuda", dtype=torch.float32)
        rc = _call(fn, dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(),
                   rows, cols, code)
        assert rc == 0, err()
        torch.cuda.synchronize()
        assert torch.equal(dx, dx_ref), f"{dtype} call {call}: dx differs"
        torch.testing.assert_close(dw, dw_ref, rtol=1e-5, atol=1e-5, msg=f"{dtype} call {call}: dw differs")


def test_noalloc_zero_rows_clears_dw():
    fn, err = _lib()
    dw = torch.full((1024,), 7.0, device="cuda", dtype=torch.float32)
    rc = _call(fn, None, None, None, None, None, dw.data_ptr(), 0, 1024, 0)
    assert rc == 0, err()
    torch.cuda.synchronize()
    assert torch.count_nonzero(dw).item() == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    fn, err = _lib()
    x = torch.zeros(4, 4104, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(4104, device="cuda", dtype=torch.float32)
    p = x.data_ptr()
    assert _call(fn, p, p, p, out.data_ptr(), p, out.data_ptr(), 4, 4104, 0) == 2
    assert b"limit" in err()
    xf = torch.zeros(4, 2052, device="cuda", dtype=torch.float32)
    outf = torch.empty(2052, device="cuda", dtype=torch.float32)
    pf = xf.data_ptr()
    assert _call(fn, pf, pf, pf, outf.data_ptr(), pf, outf.data_ptr(), 4, 2052, 1) == 2
    assert b"limit" in err()


def test_noalloc_rejects_misaligned_and_null_pointers():
    fn, err = _lib()
    x = torch.zeros(4, 1032, device="cuda", dtype=torch.bfloat16)
    dw = torch.empty(1024, device="cuda", dtype=torch.float32)
    rstd = torch.ones(4, device="cuda", dtype=torch.float32)
    p = x.data_ptr()
    # an offset view two elements in: 4-byte aligned, not 16-byte aligned
    bad = x.view(-1)[2:].data_ptr()
    assert _call(fn, bad, p, p, rstd.data_ptr(), p, dw.data_ptr(), 4, 1024, 0) == 1
    assert b"aligned" in err()
    assert _call(fn, p, p, p, None, p, dw.data_ptr(), 4, 1024, 0) == 1
    assert b"null" in err()
    assert _call(fn, p, p, p, rstd.data_ptr(), p, None, 4, 1024, 0) == 1
