"""The expert-parallel C-ABI over NCCL (include/qmoe_ep.h, libqmoe_ep.so):
the host side a C++ caller links to run the MoE block with its experts
sharded over the GPUs of a node.  On CPU: the library loads, exports every
declared symbol and rejects bad arguments without touching a GPU.  On GPUs
(at least two): one process per GPU, a communicator from qmoe_ep_unique_id /
qmoe_ep_comm_init, qmoe_ep_forward on each rank's tokens against the 1-GPU
qmoe_block_forward on all tokens -- routing and outputs bit-identical -- for
the all-to-all return and the peer-memory return, on two calls in a row."""
from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

import pytest

from qmoe import _lib, ep, synth

HEADER = Path(__file__).resolve().parent.parent / "include" / "qmoe_ep.h"
SEED = 5151


def test_ep_library_exports_every_declared_symbol():
    L = _lib.ep_lib()
    decl = sorted(set(re.findall(r"QMOE_API\s+[\w\s\*]+?\b(qmoe_\w+)\s*\(", HEADER.read_text())))
    assert len(decl) == 7
    for name in decl:
        assert hasattr(L, name), name
    assert sorted(n for n, _, _ in _lib.EP_SIGNATURES) == decl


def test_ep_argument_checks_without_gpu():
    L = _lib.ep_lib()
    dc = synth.Dims().c()
    out = ctypes.c_void_p()
    assert L.qmoe_ep_init(None, ctypes.byref(dc), 1024, 0, ctypes.byref(out)) == _lib.QMOE_ERR_ARG
    assert L.qmoe_ep_init(ctypes.c_void_p(0x1000), ctypes.byref(dc), 8, 0, ctypes.byref(out)) == _lib.QMOE_ERR_ARG
    assert L.qmoe_ep_forward(None, None, None, None, None, None, 1e-6, None, None, 100, None) == _lib.QMOE_ERR_ARG
    assert L.qmoe_ep_finalize(None) == _lib.QMOE_ERR_ARG
    assert L.qmoe_ep_comm_init(None, 2, 0, ctypes.byref(out)) == _lib.QMOE_ERR_ARG
    idb = (ctypes.c_uint8 * 128)()
    assert L.qmoe_ep_comm_init(idb, 2, 2, ctypes.byref(out)) == _lib.QMOE_ERR_ARG
    assert L.qmoe_ep_is_direct(None) == 0
    assert _lib.status_string(_lib.QMOE_ERR_COMM) == "collective communication error"


def _worker(rank, world, uid, t_local, flags, q):
    import torch
    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from test_ep_gpu import _reference  # 1-GPU block: out and top-k ids
    L = _lib.ep_lib()
    comm = ctypes.c_void_p()
    _lib.check(L.qmoe_ep_comm_init((ctypes.c_uint8 * 128).from_buffer_copy(uid), world, rank, ctypes.byref(comm)),
               "ep_comm_init")
    dims = synth.Dims()
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=SEED)  # the same bytes on every rank
    full, dc = blk.c(), dims.c()
    lb, _ = ep.local_block(full, dc, rank, world)
    ctx = ctypes.c_void_p()
    _lib.check(L.qmoe_ep_init(comm, ctypes.byref(dc), t_local, flags, ctypes.byref(ctx)), "ep_init")
    direct = L.qmoe_ep_is_direct(ctx)
    T = t_local * world
    sl = slice(rank * t_local, (rank + 1) * t_local)
    results = []
    for xs, rs in ((41, 42), (43, 44)):  # two calls: the second reuses every exchange buffer
        x_all = synth.inputs(T, dims.d_model, seed=xs, tag=7)
        r_all = synth.inputs(T, dims.d_model, seed=rs, tag=8)
        want, _ = _reference(blk, x_all, r_all)
        x, res = x_all[sl].contiguous(), r_all[sl].contiguous()
        out = torch.full_like(x, float("nan"))
        st = L.qmoe_ep_forward(ctx, ctypes.byref(full), ctypes.byref(lb), None, x.data_ptr(), None, 1e-6,
                               res.data_ptr(), out.data_ptr(), t_local, None)
        torch.cuda.synchronize()
        results.append((st, float((out - want[sl]).abs().max()), bool(torch.equal(out, want[sl]))))
    # a batch over max_tokens on one rank: every rank gets the same error, none hangs
    big = torch.zeros(t_local + (16 if rank == 0 else 0), dims.d_model, device="cuda")
    ob = torch.empty_like(big)
    st_big = L.qmoe_ep_forward(ctx, ctypes.byref(full), ctypes.byref(lb), None, big.data_ptr(), None, 1e-6, None,
                               ob.data_ptr(), big.shape[0], None)
    torch.cuda.synchronize()
    _lib.check(L.qmoe_ep_finalize(ctx), "ep_finalize")
    _lib.check(L.qmoe_ep_comm_destroy(comm), "ep_comm_destroy")
    q.put((rank, direct, results, st_big))


def _worlds():
    try:
        import torch
        n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:  # noqa: BLE001
        n = 0
    return sorted({2, min(n, 8)}) if n >= 2 else [2]


@pytest.mark.gpu
@pytest.mark.parametrize("world", _worlds())
@pytest.mark.parametrize("flags", [0, _lib.QMOE_EP_DIRECT], ids=["all_to_all_return", "direct_return"])
def test_ep_abi_nccl(world, flags):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    uid = (ctypes.c_uint8 * 128)()
    _lib.check(_lib.ep_lib().qmoe_ep_unique_id(uid), "ep_unique_id")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, bytes(uid), 160, flags, q)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    for rank, direct, results, st_big in sorted(q.get() for _ in range(world)):
        assert direct == (1 if flags else 0), rank
        for call, (st, max_err, exact) in enumerate(results):
            assert st == 0, (rank, call, _lib.status_string(st))
            assert max_err <= 1e-3, (rank, call, max_err)
            assert exact, (rank, call, max_err)
        assert st_big == _lib.QMOE_ERR_ARG, (rank, st_big)
