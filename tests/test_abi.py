"""The C-ABI library loads on a CPU-only machine, exports every symbol that
include/qmoe.h declares, and its host-side argument checks behave like the
reference's exceptions.  No kernel is launched."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from qmoe import _lib, quant
from qmoe.synth import Dims

HEADER = Path(__file__).resolve().parent.parent / "include" / "qmoe.h"


def declared_symbols():
    return sorted(set(re.findall(r"QMOE_API\s+[\w\s\*]+?\b(qmoe_\w+)\s*\(", HEADER.read_text())))


def test_every_declared_symbol_is_exported_and_bound():
    L = _lib.lib()
    decl = declared_symbols()
    assert len(decl) >= 17
    for name in decl:
        assert hasattr(L, name), name
    assert sorted(n for n, _, _ in _lib.SIGNATURES) == decl


def test_version_and_status_strings():
    L = _lib.lib()
    assert L.qmoe_abi_version() == 1
    assert _lib.status_string(_lib.QMOE_ERR_ROUTING) == "invalid/non-finite MoE routing result"
    assert _lib.status_string(_lib.QMOE_ERR_NOT_NORMALIZED) == "MoE routing weights are not normalized"


def test_type_table_matches_reference():
    # matmul_q4.cu:179-183
    supported = {0, 1, 30, 2, 6, 8, 12, 13, 14}
    for t in quant.GgmlType:
        assert bool(_lib.lib().qmoe_type_supported(int(t))) == (int(t) in supported)
    # quantized.hpp:49-105
    assert quant.ggml_type_size(quant.GgmlType.Q4_K) == 144
    assert quant.ggml_type_size(quant.GgmlType.Q6_K) == 210
    assert quant.ggml_type_size(quant.GgmlType.Q8_0) == 34
    for t in (0, 1, 2, 6, 8, 12, 13, 14, 30):
        for n in (256, 4096, 2048 * 512):
            assert _lib.lib().qmoe_tensor_bytes(t, n) == quant.calculate_tensor_bytes(t, n)
    assert quant.calculate_tensor_bytes(quant.GgmlType.Q4_K, 100) == 0


def test_workspace_size():
    L = _lib.lib()
    d = Dims().c()
    n1 = L.qmoe_workspace_size(ctypes.byref(d), 1)
    n8 = L.qmoe_workspace_size(ctypes.byref(d), 8)
    assert 0 < n1 < n8
    # more than 8 tokens: the prefill path's buffers (fp16 hidden vectors and
    # expert outputs of every (token, expert) pair) dominate
    n1000 = L.qmoe_workspace_size(ctypes.byref(d), 1000)
    k, F, dm = d.top_k, d.expert_dim, d.d_model
    assert n1000 > n8 and n1000 >= 1000 * k * (F + dm) * 2
    bad = Dims(d_model=3000).c()
    assert L.qmoe_workspace_size(ctypes.byref(bad), 1) == 0


def _block_with(dims, **over):
    def t(n, ty):
        return _lib.QmoeTensor(0x10000, ty, 0, n)
    d, E, F, Fs = dims.d_model, dims.num_experts, dims.expert_dim, dims.shared_dim
    f = dict(router=t(E * d, 0), gate_exps=t(E * F * d, 12), up_exps=t(E * F * d, 12), down_exps=t(E * d * F, 12),
             shared_gate_inp=t(d, 0), shared_gate=t(Fs * d, 12), shared_up=t(Fs * d, 12),
             shared_down=t(d * Fs, 12))
    f.update(over)
    return _lib.QmoeBlock(*(f[n] for n in ["router", "gate_exps", "up_exps", "down_exps", "shared_gate_inp",
                                           "shared_gate", "shared_up", "shared_down"]), None)


def test_block_argument_checks_without_gpu():
    L = _lib.lib()
    dims = Dims()
    dc = dims.c()
    ws = 0x20000
    big = 1 << 40

    def fwd(blk, T=1, wsb=big, x=0x30000):
        return L.qmoe_block_forward(ctypes.byref(blk), ctypes.byref(dc), x, 0x40000, None, T, ws, wsb, None)

    d, E, F = dims.d_model, dims.num_experts, dims.expert_dim
    assert fwd(_block_with(dims, router=_lib.QmoeTensor(0, 0, 0, E * d))) == _lib.QMOE_ERR_ARG
    assert fwd(_block_with(dims, gate_exps=_lib.QmoeTensor(0x10000, 3, 0, E * F * d))) == _lib.QMOE_ERR_TYPE
    assert fwd(_block_with(dims, down_exps=_lib.QmoeTensor(0x10000, 12, 0, E * F * d - 256))) == _lib.QMOE_ERR_SHAPE
    assert fwd(_block_with(dims, up_exps=_lib.QmoeTensor(0x10008, 12, 0, E * F * d))) == _lib.QMOE_ERR_ALIGN
    assert fwd(_block_with(dims), T=0) == _lib.QMOE_ERR_ARG
    assert fwd(_block_with(dims), wsb=1024) == _lib.QMOE_ERR_WORKSPACE
    assert fwd(_block_with(dims), x=0x30004) == _lib.QMOE_ERR_ALIGN
    bad = Dims(num_experts=512).c()
    assert L.qmoe_block_forward(ctypes.byref(_block_with(dims)), ctypes.byref(bad), 0x30000, 0x40000, None, 1, ws,
                                big, None) == _lib.QMOE_ERR_UNSUPPORTED
    # the launch count reports argument errors as negative statuses before
    # it looks at the device
    cnt = L.qmoe_block_kernel_count
    assert cnt(ctypes.byref(_block_with(dims)), ctypes.byref(dc), 0) == -_lib.QMOE_ERR_ARG
    assert cnt(ctypes.byref(_block_with(dims, gate_exps=_lib.QmoeTensor(0x10000, 3, 0, E * F * d))), ctypes.byref(dc),
               1) == -_lib.QMOE_ERR_TYPE
    assert cnt(ctypes.byref(_block_with(dims)), ctypes.byref(bad), 1) == -_lib.QMOE_ERR_UNSUPPORTED


def test_gemv_argument_checks_without_gpu():
    L = _lib.lib()
    w = _lib.QmoeTensor(0x10000, 12, 0, 512 * 2048)
    assert L.qmoe_gemv(ctypes.byref(w), 0x1000, 0x2000, 512, 2048, 256, None) == _lib.QMOE_ERR_SHAPE
    w0 = _lib.QmoeTensor(0, 12, 0, 512 * 2048)
    assert L.qmoe_gemv(ctypes.byref(w0), 0x1000, 0x2000, 512, 2048, 0, None) == _lib.QMOE_ERR_ARG
    w3 = _lib.QmoeTensor(0x10000, 3, 0, 512 * 2048)
    assert L.qmoe_gemv(ctypes.byref(w3), 0x1000, 0x2000, 512, 2048, 0, None) == _lib.QMOE_ERR_TYPE
    assert L.qmoe_dequant_row(ctypes.byref(w), 0x1000, 512, 2048, None) == _lib.QMOE_ERR_SHAPE


def test_python_mirror_errors_match_reference_messages():
    from qmoe import matmul
    t = quant.QuantTensor("blk.0.ffn_gate_exps.weight", quant.GgmlType.Q4_K, [2048, 512], 2048 * 512, 0, 0, 0)
    with pytest.raises(RuntimeError, match="is not loaded"):
        matmul.matmul_dispatch(t, 0, 0, 512, 2048)
    t.device_ptr = 0x10000
    with pytest.raises(RuntimeError, match="GEMV shape exceeds tensor"):
        matmul.matmul_dispatch(t, 0x1000, 0x2000, 513, 2048)
    t.type = quant.GgmlType.Q4_1
    with pytest.raises(RuntimeError, match="unsupported GGML type"):
        matmul.matmul_dispatch(t, 0x1000, 0x2000, 512, 2048)
    with pytest.raises(RuntimeError, match="cannot dequantize"):
        matmul.dequantize_row(t, 0x1000, 0, 2048)


def test_repack_sizes_and_argument_checks_without_gpu():
    L = _lib.lib()
    A16 = _lib.QMOE_LAYOUT_Q6K_A16
    assert L.qmoe_repack_bytes(14, 2048 * 512, A16) == 2048 * 512 // 256 * 224
    assert L.qmoe_repack_bytes(14, 2048 * 512, 0) == 2048 * 512 // 256 * 210
    assert L.qmoe_repack_bytes(12, 2048 * 512, A16) == 0      # Q6_K only
    assert L.qmoe_repack_bytes(14, 2048 * 512, 7) == 0        # unknown layout
    q6 = _lib.QmoeTensor(0x10000, 14, 0, 256 * 64)
    q4 = _lib.QmoeTensor(0x10000, 12, 0, 256 * 64)
    assert L.qmoe_repack(ctypes.byref(q4), A16, 0x20000, 1 << 20, None) == _lib.QMOE_ERR_TYPE
    assert L.qmoe_repack(ctypes.byref(q6), 7, 0x20000, 1 << 20, None) == _lib.QMOE_ERR_UNSUPPORTED
    assert L.qmoe_repack(ctypes.byref(q6), A16, 0x20000, 100, None) == _lib.QMOE_ERR_SHAPE
    assert L.qmoe_repack(ctypes.byref(q6), A16, 0x20008, 1 << 20, None) == _lib.QMOE_ERR_ALIGN
    # the block entry points read GGUF layouts only
    dims = Dims()
    dc = dims.c()
    blk = _block_with(dims)
    blk.gate_exps.layout = A16
    assert L.qmoe_block_forward(ctypes.byref(blk), ctypes.byref(dc), 0x30000, 0x40000, None, 1, 0x20000, 1 << 40,
                                None) == _lib.QMOE_ERR_UNSUPPORTED
    # a repacked view of a type that has no repacked layout: rejected before any launch
    q4r = _lib.QmoeTensor(0x10000, 12, A16, 512 * 2048)
    assert L.qmoe_gemv(ctypes.byref(q4r), 0x1000, 0x2000, 512, 2048, 0, None) == _lib.QMOE_ERR_UNSUPPORTED

