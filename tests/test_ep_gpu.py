"""Expert parallelism on the GPU: the qmoe_ep_* entry points against the
1-GPU qmoe_block_forward on the same bytes -- routing bit-identical, outputs
bit-identical too (each row's grouped-GEMM result and the combine order do
not depend on where the row ran), checked here within the north-star
tolerance and for exact equality.

test_ep_shards_on_one_gpu runs every shard of a G-way split on one GPU (no
exchange; the rows a rank would receive are gathered locally);
test_ep_nccl runs ExpertParallelMoE with one process per GPU over NCCL and
needs at least two GPUs."""
from __future__ import annotations

import ctypes
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

import ep_plan_ref
from qmoe import _lib, ep, synth

from gpu_util import assert_close

pytestmark = pytest.mark.gpu

SEED = 4242


def _poison(be):
    """Fill a backend's workspaces with a non-zero pattern (then re-initialise
    the control words) so that nothing can pass by reading memory left behind
    by an earlier call."""
    import torch
    for buf in (be.ws, be.rws, be.scratch, be.send_rows, be.send_meta, be.pair_pos):
        buf.view(torch.uint8).fill_(0xA5)
    _lib.check(_lib.lib().qmoe_workspace_init(be.ws.data_ptr(), be.ws_bytes, None))
    _lib.check(_lib.lib().qmoe_workspace_init(be.rws.data_ptr(), be.rws_bytes, None))


def _poison_peer(be, dist):
    """Fill this rank's IPC receive and return buffers (direct return) with the
    same pattern, then wait for every rank: a call can only pass if its own
    pushes and copies landed, not by reading a previous call's data."""
    import torch
    if getattr(be, "peer_ptrs", None) is None:
        return
    me, d, k = be.rank_, be.dims.d_model, be.dims.top_k
    for ptr, n in ((be.peer_ptrs[me], be.pair_pos.numel() * d * 2), (be.peer_rows[me], be.recv_cap * d * 2),
                   (be.peer_meta[me], be.recv_cap * k * 4)):
        torch.as_tensor(ep._DevicePtr(ptr, n), device="cuda").fill_(0xA5)
    torch.cuda.synchronize()
    dist.barrier()


def _reference(blk, x, residual):
    """1-GPU prefill block: out and the top-k ids of every token."""
    import torch
    T = x.shape[0]
    dc = blk.dims.c()
    n = _lib.lib().qmoe_workspace_size(ctypes.byref(dc), T)
    ws = torch.empty(n, dtype=torch.uint8, device=x.device)
    _lib.check(_lib.lib().qmoe_workspace_init(ws.data_ptr(), n, None))
    out = torch.empty_like(x)
    c = blk.c()
    _lib.check(_lib.lib().qmoe_block_forward(ctypes.byref(c), ctypes.byref(dc), x.data_ptr(), out.data_ptr(),
                                             residual.data_ptr(), T, ws.data_ptr(), n, None), "block_forward")
    p = _lib.lib().qmoe_ws_view(ws.data_ptr(), ctypes.byref(dc), T, _lib.WS_TOPK_IDX)
    off = p - ws.data_ptr()
    k = blk.dims.top_k
    idx = ws[off:off + T * k * 4].view(torch.int32).view(T, k).clone()
    torch.cuda.synchronize()
    return out, idx


@pytest.mark.parametrize("G,types,bias,direct,placed", [(2, synth.Q4K_TYPES, False, False, False),
                                                       (8, synth.MIXED_TYPES, True, False, False),
                                                       (4, synth.Q4K_TYPES, True, True, False),
                                                       (8, synth.Q4K_TYPES, True, True, True)],
                         ids=["g2_q4k", "g8_mixed_bias", "g4_q4k_direct_return", "g8_q4k_direct_balanced_placement"])
def test_ep_shards_on_one_gpu(cuda, G, types, bias, direct, placed):
    """Every rank of a G-way split on one GPU: the send layout bit-exact
    against tests/ep_plan_ref.py, each rank's chunk through its local experts,
    the chunks' outputs concatenated in rank order as the all-to-all returns
    them, then the combine -- equal to the 1-GPU block."""
    import torch
    dims = synth.Dims()
    T = 300
    k, d = dims.top_k, dims.d_model
    blk = synth.Block(dims, types, seed=SEED, bias=bias)
    x = synth.inputs(T, d, seed=17, tag=3)
    residual = synth.inputs(T, d, seed=18, tag=4)
    want, want_idx = _reference(blk, x, residual)

    full, dc = blk.c(), dims.c()
    L = _lib.lib()
    pl = None
    if placed:  # balance the experts over the ranks by this batch's own load
        load = np.bincount(want_idx.cpu().numpy().ravel(), minlength=dims.num_experts)
        pl = ep.balanced_placement(load.tolist(), G)
    be = ep.CudaBackend(full, full, dc, dc, G, max_tokens=T, max_rows=T, placement=pl)
    _poison(be)
    be.route(x)
    idx = be.topk_idx()
    assert torch.equal(idx, want_idx)
    send_rows, send_meta, counts, pair_pos = be.dispatch(G)
    tok, meta, cnt, pp = ep_plan_ref.dispatch_plan(idx.cpu().numpy(), dims.num_experts, G, pl)
    torch.cuda.synchronize()
    assert counts.cpu().numpy().tolist() == cnt.tolist()
    assert np.array_equal(pair_pos.cpu().numpy(), pp)
    ns = len(tok)
    assert np.array_equal(send_meta[:ns].cpu().numpy(), meta)
    x16 = be._view(_lib.WS_INPUT16, T * d, torch.float16).view(T, d)
    assert torch.equal(send_rows[:ns], x16[torch.from_numpy(tok).cuda()])

    chunks, r0 = [], 0
    total = int((idx >= 0).sum())
    y_direct = torch.full((total, d), float("nan"), dtype=torch.float16, device="cuda")
    for r in range(G):
        nr, npairs = int(cnt[r]), int(cnt[G + r])
        if placed:
            lb, ld, keep = ep.local_block_placed(full, dc, ep.experts_of_rank(pl, G, r))
        else:
            lb, ld = ep.local_block(full, dc, r, G)
        rws_bytes = L.qmoe_ep_rows_workspace_size(ctypes.byref(ld), max(nr, 1))
        rws = torch.full((rws_bytes,), 0xA5, dtype=torch.uint8, device="cuda")
        _lib.check(L.qmoe_workspace_init(rws.data_ptr(), rws_bytes, None))
        y = torch.empty((npairs, d), dtype=torch.float16, device="cuda")
        if nr and direct:
            # rank r returns its outputs straight into the home buffer (one source rank here)
            ret = _lib.QmoeEpReturn()
            ret.n_ranks = 1
            ret.pair_start[0], ret.pair_start[1] = 0, npairs
            ret.dst[0] = y_direct.data_ptr()
            ret.dst_row[0] = int(sum(int(cnt[G + q]) for q in range(r)))
            _lib.check(L.qmoe_ep_experts_return(ctypes.byref(lb), ctypes.byref(ld), send_rows[r0:r0 + nr].data_ptr(),
                                                send_meta[r0:r0 + nr].data_ptr(), nr, ctypes.byref(ret),
                                                rws.data_ptr(), rws_bytes, None), "ep_experts_return")
        elif nr:
            _lib.check(L.qmoe_ep_experts(ctypes.byref(lb), ctypes.byref(ld), send_rows[r0:r0 + nr].data_ptr(),
                                         send_meta[r0:r0 + nr].data_ptr(), nr, npairs, y.data_ptr(), rws.data_ptr(),
                                         rws_bytes, None), "ep_experts")
        chunks.append(y)
        r0 += nr
    y_ret = y_direct if direct else torch.cat(chunks)
    assert y_ret.shape[0] == int((idx >= 0).sum())
    got = be.combine(y_ret, pair_pos, residual)
    torch.cuda.synchronize()
    assert_close(got.cpu().numpy(), want.cpu().numpy(), f"ep G={G}")
    assert torch.equal(got, want)


def test_ep_argument_checks(cuda):
    import torch
    dims = synth.Dims(512, 32, 4, 256, 256)
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=3)
    full, dc = blk.c(), dims.c()
    L = _lib.lib()
    lb, ld = ep.local_block(full, dc, 1, 4)
    assert ld.num_experts == 8
    rws_bytes = L.qmoe_ep_rows_workspace_size(ctypes.byref(ld), 16)
    rws = torch.empty(rws_bytes, dtype=torch.uint8, device="cuda")
    rows = torch.zeros((16, 512), dtype=torch.float16, device="cuda")
    y = torch.empty_like(rows)
    meta = torch.zeros((16, 4), dtype=torch.int32, device="cuda")
    # zero rows is a no-op, too small a workspace is refused, decode-sized routing is refused
    assert L.qmoe_ep_experts(ctypes.byref(lb), ctypes.byref(ld), None, None, 0, 0, None, None, 0, None) == _lib.QMOE_OK
    assert L.qmoe_ep_experts(ctypes.byref(lb), ctypes.byref(ld), rows.data_ptr(), meta.data_ptr(), 16, 16,
                             y.data_ptr(), rws.data_ptr(), 1024, None) == _lib.QMOE_ERR_WORKSPACE
    # more pairs than the rows' slots can hold is an argument error
    assert L.qmoe_ep_experts(ctypes.byref(lb), ctypes.byref(ld), rows.data_ptr(), meta.data_ptr(), 16, 65,
                             y.data_ptr(), rws.data_ptr(), rws_bytes, None) == _lib.QMOE_ERR_ARG
    ws_bytes = L.qmoe_workspace_size(ctypes.byref(dc), 64)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    x = torch.zeros((8, 512), dtype=torch.float32, device="cuda")
    assert L.qmoe_ep_route(ctypes.byref(full), ctypes.byref(dc), x.data_ptr(), None, 1e-6, 8, ws.data_ptr(),
                           ws_bytes, None) == _lib.QMOE_ERR_UNSUPPORTED


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, t_local, q, direct):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        dims = synth.Dims()
        blk = synth.Block(dims, synth.Q4K_TYPES, seed=SEED)          # the same bytes on every rank
        T = t_local * world
        sl = slice(rank * t_local, (rank + 1) * t_local)
        full, dc = blk.c(), dims.c()
        lb, ld = ep.local_block(full, dc, rank, world)
        be = ep.CudaBackend(full, lb, dc, ld, world, max_tokens=t_local, max_rows=t_local)
        _poison(be)
        moe = ep.ExpertParallelMoE(be, dims.num_experts, dims.top_k, dims.d_model, direct=direct)
        results = []
        # two calls with different tokens: the second reuses the exchange and
        # return buffers, which are poisoned again before it
        for call, (xs, rs) in enumerate(((23, 24), (31, 32))):
            x_all = synth.inputs(T, dims.d_model, seed=xs, tag=5)
            r_all = synth.inputs(T, dims.d_model, seed=rs, tag=6)
            want, want_idx = _reference(blk, x_all, r_all)
            x, res = x_all[sl].contiguous(), r_all[sl].contiguous()
            _poison_peer(be, dist)
            got = moe.forward(x, res)
            idx = be.topk_idx()
            torch.cuda.synchronize()
            results.append((bool(torch.equal(idx, want_idx[sl])), float((got - want[sl]).abs().max()),
                            bool(torch.equal(got, want[sl]))))
        q.put((rank, results))
        dist.barrier()
        torch.cuda.synchronize()
        be.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _worlds():
    """2 ranks (rows pushed over peer memory when direct) and every GPU of the
    box up to 8 (rows by NCCL all-to-all above two ranks)."""
    try:
        import torch
        n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:  # noqa: BLE001
        n = 0
    return sorted({2, min(n, 8)}) if n >= 2 else [2]


@pytest.mark.parametrize("world", _worlds())
@pytest.mark.parametrize("direct", [False, True], ids=["all_to_all_return", "direct_return"])
def test_ep_nccl(cuda, direct, world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_nccl_worker, args=(r, world, port, 160, q, direct)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    for rank, results in sorted(q.get() for _ in range(world)):
        for call, (ids_equal, max_err, exact) in enumerate(results):
            assert ids_equal, (rank, call)
            assert max_err <= 1e-3, (rank, call, max_err)
            assert exact, (rank, call, max_err)
