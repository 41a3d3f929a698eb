"""Helpers shared by the GPU parity tests: run the product through its C-ABI
and the oracle / reference path on the same bytes."""
from __future__ import annotations

import ctypes
import os

import numpy as np

from oracle import oracle as orc
from qmoe import _lib, synth

# tolerance on outputs: max-abs 1e-3 / rel 1e-2 (an element passes under either bound)
ATOL, RTOL = 1e-3, 1e-2


def oracle_threads():
    orc.set_threads(max(1, min(32, os.cpu_count() or 1)))


class Run:
    """One block_forward call through the C-ABI with its workspace."""

    def __init__(self, blk: synth.Block, max_tokens: int = 8):
        import torch
        self.blk = blk
        self.dims = blk.dims.c()
        self.ws_bytes = _lib.lib().qmoe_workspace_size(ctypes.byref(self.dims), max_tokens)
        assert self.ws_bytes > 0
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device="cuda")
        _lib.check(_lib.lib().qmoe_workspace_init(self.ws.data_ptr(), self.ws_bytes, None))

    def forward(self, x, residual=None):
        import torch
        T = x.shape[0]
        out = torch.full_like(x, float("nan"))
        c = self.blk.c()
        st = _lib.lib().qmoe_block_forward(ctypes.byref(c), ctypes.byref(self.dims), x.data_ptr(), out.data_ptr(),
                                           None if residual is None else residual.data_ptr(), T,
                                           self.ws.data_ptr(), self.ws_bytes, None)
        _lib.check(st, "block_forward")
        torch.cuda.synchronize()
        return out

    def staged(self, x, residual=None):
        """The same block through the three stage entry points (router_topk,
        expert_gateup, down_combine): the two-kernel expert path."""
        import torch
        T = x.shape[0]
        out = torch.full_like(x, float("nan"))
        c = self.blk.c()
        L = _lib.lib()
        ws, wb, dp = self.ws.data_ptr(), self.ws_bytes, ctypes.byref(self.dims)
        _lib.check(L.qmoe_router_topk(ctypes.byref(c), dp, x.data_ptr(), T, None, None, ws, wb, None), "router_topk")
        _lib.check(L.qmoe_expert_gateup(ctypes.byref(c), dp, x.data_ptr(), T, ws, wb, None), "expert_gateup")
        _lib.check(L.qmoe_down_combine(ctypes.byref(c), dp, T, out.data_ptr(),
                                       None if residual is None else residual.data_ptr(), ws, wb, None),
                   "down_combine")
        torch.cuda.synchronize()
        return out

    def view(self, which, T, count, dtype):
        import torch
        p = _lib.lib().qmoe_ws_view(self.ws.data_ptr(), ctypes.byref(self.dims), T, which)
        off = p - self.ws.data_ptr()
        nbytes = count * np.dtype(dtype).itemsize
        return self.ws[off:off + nbytes].cpu().numpy().view(dtype)

    def check_errors(self):
        err = (ctypes.c_uint32 * 2)()
        st = _lib.lib().qmoe_check_errors(self.ws.data_ptr(), ctypes.byref(self.dims), err, None)
        return st, int(err[0]), int(err[1])


def oracle_run(blk: synth.Block, x_host: np.ndarray):
    return orc.moe_forward({n: blk.host_bytes(n) for n in synth.TENSORS}, blk.types, blk.dims, x_host,
                           blk.host_bias())


def assert_close(got, want, what=""):
    """The north-star bound: every element within max-abs ATOL or rel RTOL of
    the oracle (orc.tolerance_report)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    rep = orc.tolerance_report(got, want, ATOL, RTOL)
    if not rep["within_tol"]:
        diff = np.abs(got - want)
        bad = ~((diff <= ATOL) | (diff <= RTOL * np.abs(want))) | ~np.isfinite(got)
        i = np.argwhere(bad)[0]
        raise AssertionError(f"{what}: {rep['n_outside']} of {rep['n']} outside {rep['tol']}; "
                             f"first at {tuple(i)}: got {got[tuple(i)]} want {want[tuple(i)]}; "
                             f"max abs err {rep['max_abs_err']:.3e}, max rel err {rep['max_rel_err']:.3e}")
    return rep
