"""The prefill path at the size it is benchmarked at (config 4): T = 4096
tokens of a Qwen3.5-35B-A3B-shaped block (d 2048, 256 Q4_K experts, top-8,
shared expert), router skewed by the calibrated per-expert bias so that the
expert hit histogram follows Zipf(1.1) (one expert holds nearly every token,
the coldest a handful).  Against the CPU oracle on the same seeded bytes:
router logits, expert ids, selection order and the permutation bit-exact on
all 4096 tokens; the outputs of a sample of tokens (every hit expert's first
token, the tokens of the coldest experts and an even spread) within max-abs
1e-3 / rel 1e-2, with both maxima printed.  The routing and outputs the
reference computes per token: src/layer_moe.cpp:95-155."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import oracle as orc
from qmoe import _lib, synth

from gpu_util import ATOL, RTOL, oracle_threads

pytestmark = pytest.mark.gpu

T = 4096
SEED = 1234


def _view(ws, dc, which, count, dtype):
    p = _lib.lib().qmoe_ws_view(ws.data_ptr(), ctypes.byref(dc), T, which)
    off = p - ws.data_ptr()
    return ws[off:off + count * np.dtype(dtype).itemsize].cpu().numpy().view(dtype)


def test_config4_T4096_zipf_vs_oracle():
    import torch
    oracle_threads()
    dims = synth.Dims()
    d, E, k = dims.d_model, dims.num_experts, dims.top_k
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=SEED, layer=0, device="cuda")
    bias_h, _ = synth.zipf_bias(E, k, d)
    bias = torch.tensor(bias_h, device="cuda")
    c = blk.c()
    c.expert_bias = bias.data_ptr()
    x = synth.inputs(T, d, seed=SEED + 5, tag=4)
    dc = dims.c()
    n = _lib.lib().qmoe_workspace_size(ctypes.byref(dc), T)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().qmoe_workspace_init(ws.data_ptr(), n, None))
    out = torch.full_like(x, float("nan"))
    _lib.check(_lib.lib().qmoe_block_forward(ctypes.byref(c), ctypes.byref(dc), x.data_ptr(), out.data_ptr(), None,
                                             T, ws.data_ptr(), n, None), "block_forward")
    torch.cuda.synchronize()
    err = (ctypes.c_uint32 * 2)()
    assert _lib.lib().qmoe_check_errors(ws.data_ptr(), ctypes.byref(dc), err, None) == 0, list(err)
    got = {"logits": _view(ws, dc, _lib.WS_LOGITS, T * (E + 1), np.float32).reshape(T, E + 1)[:, :E],
           "idx": _view(ws, dc, _lib.WS_TOPK_IDX, T * k, np.int32).reshape(T, k),
           "w": _view(ws, dc, _lib.WS_TOPK_W, T * k, np.float32).reshape(T, k),
           "offsets": _view(ws, dc, _lib.WS_OFFSETS, E + 1, np.int32),
           "perm": _view(ws, dc, _lib.WS_PERM, T * k, np.int32),
           "out": out.cpu().numpy()}
    counts = np.diff(got["offsets"])
    # the skew the benchmark claims: heavy head, long tail
    assert counts.max() > T * 3 // 4 and (counts > 0).sum() > 200, (counts.max(), (counts > 0).sum())
    tensors = {nm: blk.host_bytes(nm) for nm in synth.TENSORS}
    res = orc.check_batch(tensors, blk.types, dims, x.cpu().numpy(), got, bias_h, atol=ATOL, rtol=RTOL)
    print(f"config4 parity: hottest expert {counts.max()} pairs, coldest hit {counts[counts > 0].min()}, "
          f"{res['out']['sample_tokens']} tokens checked: max abs err {res['out']['max_abs_err']:.3e}, "
          f"max rel err {res['out']['max_rel_err']:.3e}")
    assert res["logits_bit_exact"], "router logits not bit-exact"
    assert res["ids_bit_exact"], "expert ids / selection order differ"
    assert res["weights_max_rel_err"] <= 2e-6, res["weights_max_rel_err"]
    assert res["offsets_bit_exact"] and res["perm_bit_exact"], "permutation differs"
    assert res["out"]["oracle_status_ok"]
    assert res["out"]["within_tol"], res["out"]
