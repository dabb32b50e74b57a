"""The statistics entry point that allocates nothing (sm_stats_accumulate_noalloc).

It serves callers that cannot allocate device memory -- for example a
statistics hook running inside another framework's training step, holding
only the tensors it was handed while that framework's allocator owns the rest
of HBM.  Called through the C-ABI and compared with the workspace entry point
(sm_stats_accumulate) within the statistics tolerance (1e-5 relative), on two
calls in a row that reuse the library's shared scratch array.  This file is
collected last so a failure here leaves every other test already run.
"""
import ctypes

import pytest
import torch

from sandmuon_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
SM_STATS_NOALLOC_MAX_COLS = (1 << 19) // 2
TOL = 1e-5


def _noalloc(rows, sum_sq, total):
    lib = _lib.load()
    rc = lib.sm_stats_accumulate_noalloc(
        ctypes.c_void_p(rows.data_ptr()), _lib.DTYPE_CODES[rows.dtype], rows.shape[0], rows.shape[1],
        rows.stride(0), rows.stride(1), ctypes.c_void_p(sum_sq.data_ptr()),
        ctypes.c_void_p(0 if total is None else total.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream))
    return rc


def _with_workspace(rows, sum_sq, total):
    lib = _lib.load()
    nbytes = lib.sm_stats_workspace_bytes(rows.shape[0], rows.shape[1])
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=DEV)
    rc = lib.sm_stats_accumulate(
        ctypes.c_void_p(rows.data_ptr()), _lib.DTYPE_CODES[rows.dtype], rows.shape[0], rows.shape[1],
        rows.stride(0), rows.stride(1), ctypes.c_void_p(sum_sq.data_ptr()),
        ctypes.c_void_p(0 if total is None else total.data_ptr()), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
        ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream))
    torch.cuda.synchronize(DEV)
    return rc


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


# The last two cases are >= 128 MB per call, where inputs take the one-launch
# TMA reduction whose completion counters live in the shared array too: two
# such calls back to back show that each call starts from cleared counters.
@pytest.mark.parametrize("dtype,cols,rows_first,rows_second", [
    (torch.float32, 768, 16384, 300),
    (torch.bfloat16, 3072, 4096, 16384),
    (torch.float16, 37, 1000, 5),
    (torch.float32, 200000, 6, 3),
    (torch.float32, 768, 65536, 49152),
    (torch.bfloat16, 3072, 32768, 24576),
])
def test_noalloc_matches_workspace_entry_point_on_two_calls_in_a_row(dtype, cols, rows_first, rows_second):
    _lib.ensure_device(DEV)
    g = torch.Generator(device="cpu").manual_seed(cols)
    batches = [(torch.randn(n, cols, generator=g) * 2 + 0.3).to(dtype).to(DEV) for n in (rows_first, rows_second)]
    sq_a, s_a = torch.zeros(cols, device=DEV), torch.zeros(cols, device=DEV)
    sq_b, s_b = torch.zeros(cols, device=DEV), torch.zeros(cols, device=DEV)
    for rows in batches:
        assert _noalloc(rows, sq_a, s_a) == 0, _lib.last_error()
        assert _with_workspace(rows, sq_b, s_b) == 0, _lib.last_error()
        torch.cuda.synchronize(DEV)
        assert rel(sq_a, sq_b) < TOL
        assert rel(s_a, s_b) < TOL
    sq_c = torch.zeros(cols, device=DEV)
    assert _noalloc(batches[0], sq_c, None) == 0, _lib.last_error()
    torch.cuda.synchronize(DEV)
    assert rel(sq_c, batches[0].float().square().sum(0)) < TOL
    assert _lib.device_status(DEV) == 0


def test_noalloc_rejects_more_columns_than_its_scratch_holds():
    _lib.ensure_device(DEV)
    rows = torch.zeros(2, 8, device=DEV)
    out = torch.zeros(8, device=DEV)
    lib = _lib.load()
    rc = lib.sm_stats_accumulate_noalloc(ctypes.c_void_p(rows.data_ptr()), 0, 2, SM_STATS_NOALLOC_MAX_COLS + 1,
                                         SM_STATS_NOALLOC_MAX_COLS + 1, 1, ctypes.c_void_p(out.data_ptr()),
                                         ctypes.c_void_p(0), ctypes.c_void_p(0))
    assert rc == 1
    assert "at most" in _lib.last_error()
    assert torch.equal(out, torch.zeros(8, device=DEV))
