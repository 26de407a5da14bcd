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


def _args(x, ws_, out=None, resid=None, epilogue=3, layout=0):
    from ssd import _lib as L
    from ssd import ops

    ws_ = list(ws_)
    wp = (C.c_void_p * 3)(*[w.data_ptr() for w in ws_], *([None] * (3 - len(ws_))))
    rows = (C.c_int64 * 3)(*[w.shape[0] for w in ws_], *([0] * (3 - len(ws_))))
    bp = (C.c_void_p * 3)(None, None, None)
    return [x.data_ptr(), x.stride(0), x.shape[0], x.shape[1], len(ws_), wp, rows, bp, layout, epilogue, 0,
            out.data_ptr() if out is not None else None, out.stride(0) if out is not None else 0,
            resid.data_ptr() if resid is not None else None, resid.stride(0) if resid is not None else 0,
            ops.dtype_code(ws_[0].dtype)]


def _noalloc(x, w, status, **kw):
    from ssd import _lib as L

    L.call("ssd_linear_noalloc", *_args(x, w, **kw), status.data_ptr(), torch.cuda.current_stream().cuda_stream)


def _with_workspace(x, w, ws, **kw):
    from ssd import _lib as L

    L.call("ssd_linear", *_args(x, w, **kw), ws.ptr, ws.nbytes, None, None, ws.status.data_ptr(),
           torch.cuda.current_stream().cuda_stream)


# (dtype, T, weight segments [(rows, K)], layout): decode-sized calls at the
# largest documented row count (64) for every Llama-3-8B projection shape
# (q/k/v as three segments, o_proj, gate/up as a pair, down, a 128k-row
# vocabulary head), a verify-sized call, a 1-row call and fp32 calls.
SHAPES = [
    (torch.bfloat16, 33, [(4096, 4096)], 0),
    (torch.bfloat16, 1, [(14336, 4096)], 0),
    (torch.bfloat16, 64, [(4096, 4096), (1024, 4096), (1024, 4096)], 0),
    (torch.bfloat16, 64, [(4096, 4096)], 0),
    (torch.bfloat16, 64, [(14336, 4096), (14336, 4096)], 1),
    (torch.bfloat16, 64, [(4096, 14336)], 0),
    (torch.bfloat16, 64, [(128256, 4096)], 0),
    (torch.float32, 7, [(2048, 2048)], 0),
    (torch.float32, 64, [(2048, 8192)], 0),
]


@pytest.mark.parametrize("dtype,T,segs,layout", SHAPES)
def test_noalloc_matches_workspace_entry_point(dtype, T, segs, layout):
    from ssd import ops

    ws = ops.Workspace(DEV, max_rows=64, vocab=1, max_head_rows=1)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(7)
    K = segs[0][1]
    w = [(torch.randn(n, k, generator=g, device=DEV) * 0.02).to(dtype) for n, k in segs]
    N = sum(n for n, _ in segs)
    # the gate/up pair runs with its SwiGLU epilogue (bf16 [T, F] out), the
    # only epilogue of the pair layout; everything else stores fp32
    pair = layout == 1
    epi, odt, ncol = (2, dtype, N // 2) if pair else (3, torch.float32, N)
    for call in range(2):  # two calls in a row, different inputs
        x = torch.randn(T, K, generator=g, device=DEV).to(dtype)
        ref = torch.empty(T, ncol, dtype=odt, device=DEV)
        got = torch.full((T, ncol), float("nan"), dtype=odt, device=DEV)
        _with_workspace(x, w, ws, out=ref, layout=layout, epilogue=epi)
        _noalloc(x, w, status, out=got, layout=layout, epilogue=epi)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-5)
        if len(w) == 1:  # and the residual epilogue on the same call pattern
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
        _noalloc(x, [w], status, out=out)
