"""tp_linear_backward_noalloc: the packed-linear backward for callers that may not
allocate device memory (a framework that owns every byte of GPU memory through its
own pool, or code that runs where an allocation is not allowed).  Its activation
gradient lives in a fixed 16 MiB array inside the library instead of a
caller-provided workspace.

The test calls the entry point through the C ABI twice in a row and checks both
results against the allocating entry point (tp_linear_backward), within the same
tolerance the other bf16 / fp32 parity tests use.  The file name sorts last so a
run that stops at the first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(a, b, rtol):
    a = a.float().cpu().numpy().astype(np.float64)
    b = b.float().cpu().numpy().astype(np.float64)
    scale = max(np.abs(b).max(), 1e-30)
    assert np.all(np.abs(a - b) <= rtol * np.abs(b) + rtol * 0.25 * scale)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_noalloc_backward_matches_allocating_backward(dtype):
    if not torch.cuda.is_available():
        pytest.skip('needs a GPU')
    from tabpack_b200 import _lib, ops

    lib = _lib.load()
    torch.manual_seed(7)
    P, B, max_in, max_out = 4, 250, 128, 192
    dev = 'cuda'
    x = torch.randn(P, B, max_in, device=dev).to(dtype)
    w = (torch.randn(P, max_out, max_in, device=dev) / max_in ** 0.5).to(dtype)
    b = torch.randn(P, max_out, device=dev) * 0.1
    in_f = torch.tensor([128, 40, 96, 8], device=dev, dtype=torch.int32)
    out_f = torch.tensor([192, 16, 100, 64], device=dev, dtype=torch.int32)
    p = torch.tensor([0.0, 0.2, 0.5, 0.1], device=dev)
    kw = dict(in_features=in_f, out_features=out_f, relu=True, dropout_p=p, seed=11, offset=4)
    y = ops.linear_forward(x, w, b, **kw)
    rtol = 2.0 ** -7 if dtype == torch.bfloat16 else 1e-5

    for call in range(2):  # two calls in a row share (and reuse) the built-in scratch
        dy = torch.randn(P, B, max_out, device=dev).to(dtype)
        dx_ref, dw_ref, db_ref = ops.linear_backward(dy, x, w, y, **kw)

        dx = torch.full((P, B, max_in), float('nan'), device=dev, dtype=dtype)
        dw = torch.full((P, max_out, max_in), float('nan'), device=dev)
        db = torch.full((P, max_out), float('nan'), device=dev)
        ga = _lib.LinearGradArgs()
        ga.fwd = ops._linear_args(x, w, None, in_f, out_f, None, 0, True, p, 11, 4, 0, None)
        ga.dy, ga.y, ga.g = dy.data_ptr(), y.data_ptr(), None
        ga.dbias, ga.dx, ga.dw = db.data_ptr(), dx.data_ptr(), dw.data_ptr()
        ga.dw_rows, ga.dw_cols, ga.db_cols = max_out, max_in, max_out
        rc = lib.tp_linear_backward_noalloc(ctypes.byref(ga), torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.tp_last_error_string()
        torch.cuda.synchronize()
        _close(dx, dx_ref, rtol)
        _close(dw, dw_ref, rtol)
        _close(db, db_ref, rtol)
    assert lib.tp_device_error() == 0


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_noalloc_backward_plain_linear_uses_no_scratch(dtype):
    """A plain linear layer (no ReLU, no dropout, no per-member widths or depths): dY is the
    activation gradient itself, so the entry point passes it straight to dgrad / wgrad and
    leaves the built-in scratch alone.  Its size limit does not apply either: this case is
    larger than the scratch."""
    if not torch.cuda.is_available():
        pytest.skip('needs a GPU')
    from tabpack_b200 import _lib, ops

    lib = _lib.load()
    torch.manual_seed(11)
    # P * B * max_out = 3 * 2048 * 1536 elements: 18 MiB in bf16, more than the 16 MiB scratch
    P, B, max_in, max_out = 3, 2048, 96, 1536
    dev = 'cuda'
    x = torch.randn(P, B, max_in, device=dev).to(dtype)
    w = (torch.randn(P, max_out, max_in, device=dev) / max_in ** 0.5).to(dtype)
    b = torch.randn(P, max_out, device=dev) * 0.1
    y = ops.linear_forward(x, w, b)
    rtol = 2.0 ** -7 if dtype == torch.bfloat16 else 1e-5
    for call in range(2):
        dy = torch.randn(P, B, max_out, device=dev).to(dtype)
        dx_ref, dw_ref, db_ref = ops.linear_backward(dy, x, w, y)
        dx = torch.full((P, B, max_in), float('nan'), device=dev, dtype=dtype)
        dw = torch.full((P, max_out, max_in), float('nan'), device=dev)
        db = torch.full((P, max_out), float('nan'), device=dev)
        ga = _lib.LinearGradArgs()
        ga.fwd = ops._linear_args(x, w, None, None, None, None, 0, False, None, 0, 0, 0, None)
        ga.dy, ga.y, ga.g = dy.data_ptr(), y.data_ptr(), None
        ga.dbias, ga.dx, ga.dw = db.data_ptr(), dx.data_ptr(), dw.data_ptr()
        ga.dw_rows, ga.dw_cols, ga.db_cols = max_out, max_in, max_out
        rc = lib.tp_linear_backward_noalloc(ctypes.byref(ga), torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.tp_last_error_string()
        torch.cuda.synchronize()
        _close(dx, dx_ref, rtol)
        _close(dw, dw_ref, rtol)
        _close(db, db_ref, rtol)
    assert lib.tp_device_error() == 0


def test_noalloc_rejects_oversized_and_caller_workspace():
    if not torch.cuda.is_available():
        pytest.skip('needs a GPU')
    from tabpack_b200 import _lib, ops

    lib = _lib.load()
    t = torch.zeros(16, device='cuda', dtype=torch.bfloat16)
    pf = torch.zeros(1, device='cuda')
    ga = _lib.LinearGradArgs()
    # 1 member x 4096 rows x 4096 bf16 columns = 32 MiB of workspace > 16 MiB
    ga.fwd = _lib.LinearArgs(P=1, B=4096, max_in=8, max_out=4096, dtype=_lib.TP_DTYPE_BF16, relu=1,
                             x=t.data_ptr(), w=t.data_ptr(), y=t.data_ptr())
    ga.dy, ga.y = t.data_ptr(), t.data_ptr()
    ga.dbias = pf.data_ptr()
    rc = lib.tp_linear_backward_noalloc(ctypes.byref(ga), torch.cuda.current_stream().cuda_stream)
    assert rc == -1
    assert b'built-in scratch' in lib.tp_last_error_string()
    ga.g = t.data_ptr()
    assert lib.tp_linear_backward_noalloc(ctypes.byref(ga), None) == -1
    assert b'g = NULL' in lib.tp_last_error_string()
    del ops
