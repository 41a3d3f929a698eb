"""qmoe_dispatch_noalloc (fixed device scratch, no workspace argument) against
qmoe_dispatch (caller's workspace) on the same top-k ids: identical offsets,
permutation and inverse permutation, on two calls in a row.  Kept in a file
of its own that is collected last, so it runs both alone and after the other
GPU tests in one process."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from qmoe import _lib

pytestmark = pytest.mark.gpu

CASES = [(1, 8, 256), (37, 8, 256), (4096, 8, 256), (5, 6, 64), (300, 2, 7)]


def _run(fn_name, d_idx, T, k, E, ws=None):
    import torch
    off = torch.full((E + 1,), -7, dtype=torch.int32, device="cuda")
    perm = torch.full((T * k,), -7, dtype=torch.int32, device="cuda")
    inv = torch.full((T * k,), -7, dtype=torch.int32, device="cuda")
    L = _lib.lib()
    if fn_name == "qmoe_dispatch":
        st = L.qmoe_dispatch(d_idx.data_ptr(), T, k, E, off.data_ptr(), perm.data_ptr(), inv.data_ptr(),
                             ws.data_ptr(), ws.numel(), None)
    else:
        st = L.qmoe_dispatch_noalloc(d_idx.data_ptr(), T, k, E, off.data_ptr(), perm.data_ptr(), inv.data_ptr(),
                                     None)
    _lib.check(st, fn_name)
    torch.cuda.synchronize()
    return off.cpu().numpy(), perm.cpu().numpy(), inv.cpu().numpy()


@pytest.mark.parametrize("T,k,E", CASES)
def test_noalloc_dispatch_matches_workspace_dispatch(T, k, E):
    import torch
    rng = np.random.default_rng(T * 1000 + k * 10 + E)
    idx = rng.integers(0, E, size=(T, k)).astype(np.int32)
    idx[::5, 0] = -1  # invalid slots are left out of the permutation by both
    d_idx = torch.from_numpy(idx).cuda()
    ws = torch.empty(E * 32 * 4, dtype=torch.uint8, device="cuda")
    want = _run("qmoe_dispatch", d_idx, T, k, E, ws)
    for _ in range(2):  # two calls in a row share (and re-clear) the fixed scratch
        got = _run("qmoe_dispatch_noalloc", d_idx, T, k, E)
        for g, w in zip(got, want):
            assert np.array_equal(g, w)


def test_noalloc_dispatch_rejects_more_experts_than_its_scratch_holds():
    import torch
    d_idx = torch.zeros(8, dtype=torch.int32, device="cuda")
    buf = torch.zeros(1024, dtype=torch.int32, device="cuda")
    st = _lib.lib().qmoe_dispatch_noalloc(d_idx.data_ptr(), 1, 8, 257, buf.data_ptr(), buf.data_ptr(),
                                          buf.data_ptr(), None)
    assert st == _lib.QMOE_ERR_UNSUPPORTED
