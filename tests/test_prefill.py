"""Prefill path (T > 8 tokens per call): exact-order router logits for every
token, per-token top-k, stable permutation, tcgen05 grouped GEMMs for the
routed and shared experts, combine -- against the CPU oracle on the same
seeded bytes: expert ids and permutation bit-exact, outputs within the
north-star tolerance."""
from __future__ import annotations

import ctypes
import zlib

import numpy as np
import pytest

from oracle import oracle as orc
from qmoe import _lib, synth
from qmoe.quant import GgmlType

from gpu_util import assert_close, oracle_run, oracle_threads

pytestmark = pytest.mark.gpu

REAL = synth.Dims()
CASES = [
    ("small_q4k_T40", synth.Dims(1024, 64, 4, 256, 512), synth.Q4K_TYPES, False, 40),
    ("real_q4k_T300", REAL, synth.Q4K_TYPES, False, 300),
    ("real_mixed_bias_T100", REAL, synth.MIXED_TYPES, True, 100),
    ("small_q5k_q8_T129", synth.Dims(512, 32, 6, 256, 256),
     {**synth.Q4K_TYPES, "gate_exps": GgmlType.Q5_K, "up_exps": GgmlType.Q5_K, "down_exps": GgmlType.Q8_0,
      "shared_gate": GgmlType.Q6_K, "shared_up": GgmlType.Q6_K, "shared_down": GgmlType.Q5_K}, True, 129),
]


def _ws(dims, T):
    import torch
    dc = dims.c()
    n = _lib.lib().qmoe_workspace_size(ctypes.byref(dc), T)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().qmoe_workspace_init(ws.data_ptr(), n, None))
    return dc, ws, n


def _view(ws, dc, T, which, count, dtype):
    p = _lib.lib().qmoe_ws_view(ws.data_ptr(), ctypes.byref(dc), T, which)
    off = p - ws.data_ptr()
    return ws[off:off + count * np.dtype(dtype).itemsize].cpu().numpy().view(dtype)


@pytest.mark.parametrize("name,dims,types,bias,T", CASES, ids=[c[0] for c in CASES])
def test_prefill_block_vs_oracle(name, dims, types, bias, T):
    import torch
    oracle_threads()
    blk = synth.Block(dims, types, seed=zlib.crc32(name.encode()) & 0xFFFF, device="cuda", bias=bias)
    x = synth.inputs(T, dims.d_model, seed=91, tag=T)
    dc, ws, n = _ws(dims, T)
    out = torch.full_like(x, float("nan"))
    c = blk.c()
    _lib.check(_lib.lib().qmoe_block_forward(ctypes.byref(c), ctypes.byref(dc), x.data_ptr(), out.data_ptr(), None, T,
                                             ws.data_ptr(), n, None), "block_forward")
    torch.cuda.synchronize()
    err = (ctypes.c_uint32 * 2)()
    assert _lib.lib().qmoe_check_errors(ws.data_ptr(), ctypes.byref(dc), err, None) == 0
    want = oracle_run(blk, x.cpu().numpy())
    assert np.all(want["status"] == 0)
    k, E = dims.top_k, dims.num_experts
    logits = _view(ws, dc, T, _lib.WS_LOGITS, T * (E + 1), np.float32).reshape(T, E + 1)
    assert np.array_equal(logits[:, :E].view(np.uint32), want["logits"].view(np.uint32)), "router logits not bit-exact"
    idx = _view(ws, dc, T, _lib.WS_TOPK_IDX, T * k, np.int32).reshape(T, k)
    assert np.array_equal(idx, want["idx"])
    wts = _view(ws, dc, T, _lib.WS_TOPK_W, T * k, np.float32).reshape(T, k)
    assert np.allclose(wts, want["w"], rtol=2e-6, atol=0)
    offs, perm, _ = orc.dispatch(want["idx"], E)
    assert np.array_equal(_view(ws, dc, T, _lib.WS_OFFSETS, E + 1, np.int32), offs)
    assert np.array_equal(_view(ws, dc, T, _lib.WS_PERM, T * k, np.int32)[: perm.size], perm)
    assert_close(out.cpu().numpy(), want["out"], f"{name} out")


def test_prefill_prenorm_residual_matches_decode_slabs():
    """qmoe_block_forward_prenorm through the prefill path and through the
    decode path (8-token calls) give the same routing and agree within the
    tolerance."""
    import torch
    dims = REAL
    T = 64
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=321, device="cuda")
    r = synth.inputs(T, dims.d_model, seed=5, tag=1)
    gamma = torch.linspace(0.5, 1.5, dims.d_model, device="cuda")
    c = blk.c()
    dc, ws, n = _ws(dims, T)
    out_pf = torch.empty_like(r)
    _lib.check(_lib.lib().qmoe_block_forward_prenorm(ctypes.byref(c), ctypes.byref(dc), r.data_ptr(),
                                                     gamma.data_ptr(), 1e-6, out_pf.data_ptr(), T, ws.data_ptr(), n,
                                                     None))
    idx_pf = _view(ws, dc, T, _lib.WS_TOPK_IDX, T * dims.top_k, np.int32).copy()
    dc8, ws8, n8 = _ws(dims, 8)
    out_dec = torch.empty_like(r)
    idx_dec = []
    for t0 in range(0, T, 8):
        _lib.check(_lib.lib().qmoe_block_forward_prenorm(ctypes.byref(c), ctypes.byref(dc8), r[t0:].data_ptr(),
                                                         gamma.data_ptr(), 1e-6, out_dec[t0:].data_ptr(), 8,
                                                         ws8.data_ptr(), n8, None))
        torch.cuda.synchronize()
        idx_dec.append(_view(ws8, dc8, 8, _lib.WS_TOPK_IDX, 8 * dims.top_k, np.int32).copy())
    torch.cuda.synchronize()
    assert np.array_equal(idx_pf, np.concatenate(idx_dec))
    assert_close(out_pf.cpu().numpy(), out_dec.cpu().numpy(), "prefill vs decode")


@pytest.mark.parametrize("types,want", [(synth.Q4K_TYPES, 14), (synth.MIXED_TYPES, 13)], ids=["q4k", "mixed"])
def test_prefill_kernel_count(types, want):
    """qmoe_block_kernel_count on the prefill path: routing 4, dispatch 4, the
    routed products (gather + two TMA GEMMs for Q4_K, two cp.async GEMMs
    otherwise), the shared expert's two GEMMs and the combine; decode-sized
    calls stay at 2 (fused) or 3 kernels."""
    dims = synth.Dims()
    blk = synth.Block(dims, types, seed=5, device="cuda")
    c, dc = blk.c(), dims.c()
    L = _lib.lib()
    assert L.qmoe_block_kernel_count(ctypes.byref(c), ctypes.byref(dc), 4096) == want
    assert L.qmoe_block_kernel_count(ctypes.byref(c), ctypes.byref(dc), 1) == 2
    assert L.qmoe_block_kernel_count(ctypes.byref(c), ctypes.byref(dc), 8) == 3
