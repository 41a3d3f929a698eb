"""The batched layer loop (qmoe_stack_forward): the MoE halves of several
layers for a batch of T tokens, the multi-token form of the layer loop of
src/model.cpp:193-212 (rmsnorm :208, MoeLayer::forward :209, residual_add
:211), which the reference only runs one token at a time
(src/main.cpp:391-393).  Checked layer by layer against the CPU oracle
(rmsnorm of the layer's input, the MoE block, the residual add) and bit for
bit against the same loop written out with qmoe_block_forward_prenorm."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import oracle as orc
from qmoe import _lib, synth

from gpu_util import assert_close, oracle_run, oracle_threads

pytestmark = pytest.mark.gpu

EPS = 1e-6


@pytest.mark.parametrize("dims,L,T", [(synth.Dims(1024, 64, 4, 256, 512), 3, 24),   # tensor-core path
                                      (synth.Dims(), 2, 5)],                          # decode kernels
                         ids=["small_L3_T24", "real_L2_T5"])
def test_stack_forward_vs_layer_loop_and_oracle(dims, L, T):
    import torch
    oracle_threads()
    blocks = [synth.Block(dims, synth.Q4K_TYPES, seed=700 + l, device="cuda") for l in range(L)]
    norms = [1.0 + 0.1 * synth.inputs(1, dims.d_model, seed=710 + l, tag=1)[0] for l in range(L)]
    x0 = synth.inputs(T, dims.d_model, seed=720, tag=T) * 2.0
    dc = dims.c()
    n = _lib.lib().qmoe_workspace_size(ctypes.byref(dc), T)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().qmoe_workspace_init(ws.data_ptr(), n, None))
    # the stack entry point, in place on `resid`
    resid = x0.clone()
    tmp = torch.empty_like(resid)
    cblocks = (_lib.QmoeBlock * L)(*[b.c() for b in blocks])
    nptr = (ctypes.c_void_p * L)(*[w.data_ptr() for w in norms])
    _lib.check(_lib.lib().qmoe_stack_forward(cblocks, nptr, L, ctypes.byref(dc), EPS, resid.data_ptr(),
                                             tmp.data_ptr(), T, ws.data_ptr(), n, None), "stack_forward")
    torch.cuda.synchronize()
    # the loop written out, keeping every layer's output
    outs, cur = [], x0
    for l in range(L):
        nxt = torch.full_like(x0, float("nan"))
        c = blocks[l].c()
        _lib.check(_lib.lib().qmoe_block_forward_prenorm(ctypes.byref(c), ctypes.byref(dc), cur.data_ptr(),
                                                         norms[l].data_ptr(), EPS, nxt.data_ptr(), T,
                                                         ws.data_ptr(), n, None), "block_forward_prenorm")
        torch.cuda.synchronize()
        outs.append(nxt)
        cur = nxt
    assert torch.equal(resid, outs[-1])
    # every layer against the oracle, from the GPU's input to that layer
    prev = x0.cpu().numpy()
    for l in range(L):
        wh = norms[l].cpu().numpy()
        xin = np.stack([orc.rmsnorm(prev[t], wh, EPS) for t in range(T)])
        want = prev + oracle_run(blocks[l], xin)["out"]
        got = outs[l].cpu().numpy()
        assert_close(got, want, f"layer {l}")
        prev = got


def test_stack_forward_arguments():
    import torch
    dims = synth.Dims(1024, 64, 4, 256, 512)
    dc = dims.c()
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=7, device="cuda")
    buf = torch.zeros(4, dims.d_model, device="cuda")
    w = torch.ones(dims.d_model, device="cuda")
    n = _lib.lib().qmoe_workspace_size(ctypes.byref(dc), 4)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    cb = (_lib.QmoeBlock * 1)(blk.c())
    nptr = (ctypes.c_void_p * 1)(w.data_ptr())
    f = _lib.lib().qmoe_stack_forward
    assert f(cb, nptr, 0, ctypes.byref(dc), EPS, buf.data_ptr(), buf.data_ptr(), 4, ws.data_ptr(), n, None) == \
        _lib.QMOE_ERR_ARG  # no layers
    assert f(cb, nptr, 1, ctypes.byref(dc), EPS, buf.data_ptr(), buf.data_ptr(), 4, ws.data_ptr(), n, None) == \
        _lib.QMOE_ERR_ARG  # tmp aliases resid
    tmp = torch.empty_like(buf)
    assert f(cb, nptr, 1, ctypes.byref(dc), EPS, buf.data_ptr(), tmp.data_ptr(), 4, ws.data_ptr(), 16, None) == \
        _lib.QMOE_ERR_WORKSPACE
