"""ssd_linear_noalloc: the linear entry point for callers that cannot
allocate device memory.

Some callers cannot call cudaMalloc when they run a projection (a server
that reserves all device memory up front, a plain C caller with no
allocator of its own). ssd_linear_noalloc runs the same fused GEMM as
ssd_linear with its split-K scratch in a fixed array inside the library
instead of a caller workspace. These tests call it through the C ABI and
compare it with ssd_linear on the same inputs, twice in a row (the shared
array keeps the previous call's contents), and check that oversized calls
are refused. The file is named to be collected last.
"""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _args(x, w, out=None, resid=None, epilogue=3):
    from ssd import _lib as L
    from ssd import ops

    wp = (C.c_void_p * 3)(w.data_ptr(), None, None)
    rows = (C.c_int64 * 3)(w.shape[0], 0, 0)
    bp = (C.c_void_p * 3)(None, None, None)
    return [x.data_ptr(), x.stride(0), x.shape[0], x.shape[1], 1, wp, rows, bp, L.SEG_CONCAT, epilogue, 0,
            out.data_ptr() if out is not None else None, out.stride(0) if out is not None else 0,
            resid.data_ptr() if resid is not None else None, resid.stride(0) if resid is not None else 0,
            ops.dtype_code(w.dtype)]


def _noalloc(x, w, status, **kw):
    from ssd import _lib as L

    L.call("ssd_linear_noalloc", *_args(x, w, **kw), status.data_ptr(), torch.cuda.current_stream().cuda_stream)


def _with_workspace(x, w, ws, **kw):
    from ssd import _lib as L

    L.call("ssd_linear", *_args(x, w, **kw), ws.ptr, ws.nbytes, None, None, ws.status.data_ptr(),
           torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("dtype,T,N,K", [(torch.bfloat16, 33, 4096, 4096), (torch.bfloat16, 1, 14336, 4096),
                                         (torch.float32, 7, 2048, 2048)])
def test_noalloc_matches_workspace_entry_point(dtype, T, N, K):
    from ssd import ops

    ws = ops.Workspace(DEV, max_rows=64, vocab=1, max_head_rows=1)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(7)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(dtype)
    for call in range(2):  # two calls in a row, different inputs
        x = torch.randn(T, K, generator=g, device=DEV).to(dtype)
        ref = torch.empty(T, N, dtype=torch.float32, device=DEV)
        got = torch.full((T, N), float("nan"), dtype=torch.float32, device=DEV)
        _with_workspace(x, w, ws, out=ref)
        _noalloc(x, w, status, out=got)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-5)
        # and the residual epilogue on the same call pattern
        r0 = torch.randn(T, N, generator=g, device=DEV)
        r_ref, r_got = r0.clone(), r0.clone()
        _with_workspace(x, w, ws, resid=r_ref, epilogue=1)
        _noalloc(x, w, status, resid=r_got, epilogue=1)
        torch.cuda.synchronize()
        torch.testing.assert_close(r_got, r_ref, rtol=1e-4, atol=1e-5)


def test_noalloc_rejects_oversized_calls():
    from ssd import _lib as L

    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    w = torch.zeros(256, 128, dtype=torch.bfloat16, device=DEV)
    x = torch.zeros(65, 128, dtype=torch.bfloat16, device=DEV)
    out = torch.empty(65, 256, dtype=torch.float32, device=DEV)
    with pytest.raises(L.SSDError, match="outside 1..64"):
        _noalloc(x, w, status, out=out)
