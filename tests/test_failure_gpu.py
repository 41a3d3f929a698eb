"""Failure detection on the GPU without a GPU fault.

The fused decode kernel synchronises its CTAs with a grid barrier whose wait
is bounded.  The test hook qmoe_debug_grid_barrier makes that wait run out (it
waits for one CTA that never arrives, for 1 ms): the kernel must return, the
call must report QMOE_ERR_TIMEOUT through qmoe_check_errors and through a
registered host-mapped error word, and after qmoe_workspace_init the same
workspace must compute the block correctly again.
"""
import ctypes

import pytest

from gpu_util import assert_close, oracle_run
from qmoe import _lib, synth

pytestmark = pytest.mark.gpu

EF_TIMEOUT = 4


def _block_call(blk, dims, x, out, ws):
    dc, c = dims.c(), blk.c()
    return _lib.lib().qmoe_block_forward(ctypes.byref(c), ctypes.byref(dc), x.data_ptr(), out.data_ptr(), None,
                                         x.shape[0], ws.data_ptr(), ws.numel(), None)


def test_grid_barrier_wait_runs_out(cuda):
    import torch

    L = _lib.lib()
    dims = synth.Dims()
    dc = dims.c()
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=77, device="cuda")
    x = synth.inputs(1, dims.d_model, seed=77, tag=3)
    out = torch.full_like(x, float("nan"))
    nws = L.qmoe_workspace_size(ctypes.byref(dc), 1)
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    _lib.check(L.qmoe_workspace_init(ws.data_ptr(), nws, None))
    # a host-mapped error word (pinned, device-visible through UVA)
    sink = torch.zeros(1, dtype=torch.int32).pin_memory()
    _lib.check(L.qmoe_workspace_set_error_sink(ws.data_ptr(), sink.data_ptr(), None))

    _lib.check(L.qmoe_debug_grid_barrier(1_000_000, 1))
    try:
        _lib.check(_block_call(blk, dims, x, out, ws), "block_forward")
        torch.cuda.synchronize()  # returns: the wait ran out instead of hanging
    finally:
        _lib.check(L.qmoe_debug_grid_barrier(0, 0))
    assert int(sink[0]) & EF_TIMEOUT, int(sink[0])
    err = (ctypes.c_uint32 * 2)()
    assert L.qmoe_check_errors(ws.data_ptr(), ctypes.byref(dc), err, None) == _lib.QMOE_ERR_TIMEOUT
    assert err[0] & EF_TIMEOUT

    # re-initialised, the same workspace computes the block correctly
    _lib.check(L.qmoe_workspace_init(ws.data_ptr(), nws, None))
    _lib.check(_block_call(blk, dims, x, out, ws), "block_forward")
    torch.cuda.synchronize()
    assert L.qmoe_check_errors(ws.data_ptr(), ctypes.byref(dc), err, None) == _lib.QMOE_OK
    want = oracle_run(blk, x.cpu().numpy())
    assert_close(out.cpu().numpy(), want["out"], "block after a timed-out call")
