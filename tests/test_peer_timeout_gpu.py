"""Failure detection of the peer-memory collectives on one GPU, without a fault: a wait for another
rank's rows runs out and the kernel returns with TC_DEVERR_PEER_TIMEOUT set.

Two regions of this GPU stand in for ranks 0 and 1 of a two-rank group; nothing plays rank 1, so
the words (sums) and the arrivals (gather) it would write never come. Each kernel's wait is bounded
(about a second), after which it records the error bit, finishes with what it has, and the context
stays usable: a normal launch afterwards works and the bit reads back once.
"""
import ctypes

import pytest
import torch

from threadcut_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
PEER_TIMEOUT = 4  # TC_DEVERR_PEER_TIMEOUT


def _regions(nbytes):
    L = _lib.lib()
    ptrs = []
    for _ in range(2):
        handle = (ctypes.c_uint8 * L.tc_peer_handle_bytes())()
        p = ctypes.c_void_p()
        assert L.tc_peer_alloc(nbytes, ctypes.byref(p), handle) == 0
        ptrs.append(p.value)
    return ptrs


def _free(ptrs):
    torch.cuda.synchronize()
    for p in ptrs:
        _lib.lib().tc_peer_free(ctypes.c_void_p(p))


def test_sum_wait_for_a_missing_rank_times_out():
    torch.cuda.set_device(DEV)
    L = _lib.lib()
    _lib.device_errors(clear=True)
    hidden, k = 256, 64
    ptrs = _regions(L.tc_allreduce_region_bytes(2, hidden))
    arr = (ctypes.c_void_p * 2)(*ptrs)
    x = torch.randn(1, k, device=DEV).to(torch.bfloat16)
    w = torch.randn(hidden, k, device=DEV).to(torch.bfloat16)
    h = torch.randn(1, hidden, device=DEV).to(torch.bfloat16)
    nw = torch.ones(hidden, device=DEV).to(torch.bfloat16)
    out = torch.empty_like(h)
    st = torch.cuda.current_stream().cuda_stream
    assert L.tc_gemv_allreduce(x.data_ptr(), w.data_ptr(), hidden, k, arr, 2, 0, _lib.TC_BF16, st) == 0
    assert L.tc_allreduce_add_rmsnorm(h.data_ptr(), nw.data_ptr(), out.data_ptr(), hidden, 1e-6, ptrs[0], 2,
                                      _lib.TC_BF16, st) == 0
    assert _lib.device_errors(clear=True) == PEER_TIMEOUT
    assert torch.isfinite(out.float()).all()
    y = x.float() @ w.float().t()  # the context still works
    torch.cuda.synchronize()
    assert torch.isfinite(y).all() and _lib.device_errors(clear=True) == 0
    _free(ptrs)


def test_gather_wait_for_a_missing_rank_times_out():
    torch.cuda.set_device(DEV)
    L = _lib.lib()
    _lib.device_errors(clear=True)
    rows, d = 8, 128
    ptrs = _regions(L.tc_gather_region_bytes(2, rows, d))
    arr = (ctypes.c_void_p * 2)(*ptrs)
    o = torch.randn(rows, d, device=DEV)
    lse = torch.randn(rows, device=DEV)
    out = torch.empty(rows, d, device=DEV).to(torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream
    assert L.tc_peer_gather_merge(o.data_ptr(), lse.data_ptr(), out.data_ptr(), None, rows, d, d, arr, 2, 0,
                                  _lib.TC_BF16, st) == 0
    assert _lib.device_errors(clear=True) == PEER_TIMEOUT
    torch.cuda.synchronize()
    assert _lib.device_errors(clear=True) == 0
    _free(ptrs)


def test_residual_sum_wait_for_a_missing_rank_times_out():
    """The residual form: each CTA of the projection waits for rank 1's words of its own rows, which
    never come; every wait runs out, the residual gets rank 0's part alone, the bit is set."""
    torch.cuda.set_device(DEV)
    L = _lib.lib()
    _lib.device_errors(clear=True)
    hidden, k = 256, 64
    ptrs = _regions(L.tc_allreduce_region_bytes(2, hidden))
    arr = (ctypes.c_void_p * 2)(*ptrs)
    x = torch.randn(1, k, device=DEV).to(torch.bfloat16)
    w = torch.randn(hidden, k, device=DEV).to(torch.bfloat16)
    h = torch.zeros(1, hidden, device=DEV).to(torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream
    assert L.tc_gemv_allreduce_residual(x.data_ptr(), w.data_ptr(), hidden, k, arr, 2, 0, h.data_ptr(),
                                        _lib.TC_BF16, st) == 0
    assert _lib.device_errors(clear=True) == PEER_TIMEOUT
    mine = (x.float() @ w.float().t()).to(torch.bfloat16)
    torch.testing.assert_close(h.float(), mine.float(), rtol=2 ** -7, atol=1e-2)
    torch.cuda.synchronize()
    assert _lib.device_errors(clear=True) == 0
    _free(ptrs)
