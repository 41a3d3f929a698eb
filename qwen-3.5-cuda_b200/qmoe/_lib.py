"""ctypes bindings of libqmoe.so (include/qmoe.h).

The library is loaded from this directory.  There is no fallback: if the
shared library is missing the import fails loudly (build it with
``python qwen-3.5-cuda_b200/qmoe/build.py`` or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int32, c_size_t, c_uint32, c_uint64, c_void_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqmoe.so"

QMOE_OK = 0
QMOE_ERR_ARG = 1
QMOE_ERR_TYPE = 2
QMOE_ERR_SHAPE = 3
QMOE_ERR_ALIGN = 4
QMOE_ERR_WORKSPACE = 5
QMOE_ERR_UNSUPPORTED = 6
QMOE_ERR_CUDA = 7
QMOE_ERR_ROUTING = 10
QMOE_ERR_NOT_NORMALIZED = 11
QMOE_ERR_TIMEOUT = 12
QMOE_ERR_COMM = 13
QMOE_LAYOUT_GGUF, QMOE_LAYOUT_Q6K_A16 = 0, 1

WS_LOGITS, WS_TOPK_IDX, WS_TOPK_W, WS_OFFSETS, WS_PERM, WS_INV_PERM, WS_HIDDEN, WS_ERROR, WS_INPUT, WS_INPUT16 = range(10)


class QmoeTensor(ctypes.Structure):
    _fields_ = [("data", c_void_p), ("ggml_type", c_uint32), ("layout", c_uint32), ("num_elements", c_uint64)]


class QmoeDims(ctypes.Structure):
    _fields_ = [("d_model", c_int32), ("num_experts", c_int32), ("top_k", c_int32), ("expert_dim", c_int32),
                ("shared_dim", c_int32)]


class QmoeBlock(ctypes.Structure):
    _fields_ = [("router", QmoeTensor), ("gate_exps", QmoeTensor), ("up_exps", QmoeTensor),
                ("down_exps", QmoeTensor), ("shared_gate_inp", QmoeTensor), ("shared_gate", QmoeTensor),
                ("shared_up", QmoeTensor), ("shared_down", QmoeTensor), ("expert_bias", c_void_p)]


class QmoeEpReturn(ctypes.Structure):
    _fields_ = [("n_ranks", c_int32), ("pair_start", c_int32 * 33), ("dst", c_void_p * 32),
                ("dst_row", ctypes.c_int64 * 32)]


# (name, restype, argtypes) for every symbol declared in include/qmoe.h
SIGNATURES = [
    ("qmoe_abi_version", c_int, []),
    ("qmoe_status_string", ctypes.c_char_p, [c_int]),
    ("qmoe_type_supported", c_int, [c_uint32]),
    ("qmoe_gemv", c_int, [POINTER(QmoeTensor), c_void_p, c_void_p, c_int, c_int, c_uint64, c_void_p]),
    ("qmoe_gemv_exact", c_int, [POINTER(QmoeTensor), c_void_p, c_void_p, c_int, c_int, c_uint64, c_void_p]),
    ("qmoe_dequant_row", c_int, [POINTER(QmoeTensor), c_void_p, c_int, c_int, c_void_p]),
    ("qmoe_repack_bytes", c_uint64, [c_uint32, c_uint64, c_uint32]),
    ("qmoe_repack", c_int, [POINTER(QmoeTensor), c_uint32, c_void_p, c_size_t, c_void_p]),
    ("qmoe_workspace_size", c_size_t, [POINTER(QmoeDims), c_int]),
    ("qmoe_ws_view", c_void_p, [c_void_p, POINTER(QmoeDims), c_int, c_int]),
    ("qmoe_router_topk", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_void_p, c_int, c_void_p, c_void_p,
                                 c_void_p, c_size_t, c_void_p]),
    ("qmoe_dispatch", c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                              c_void_p]),
    ("qmoe_dispatch_noalloc", c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("qmoe_expert_gateup", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_void_p, c_int, c_void_p, c_size_t,
                                   c_void_p]),
    ("qmoe_down_combine", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_int, c_void_p, c_void_p, c_void_p,
                                  c_size_t, c_void_p]),
    ("qmoe_expert_block", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_int, c_void_p, c_void_p, c_void_p,
                                  c_size_t, c_void_p]),
    ("qmoe_ep_route", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_void_p, c_void_p, c_float, c_int, c_void_p,
                              c_size_t, c_void_p]),
    ("qmoe_ep_dispatch_scratch_size", c_size_t, [c_int, c_int]),
    ("qmoe_ep_dispatch", c_int, [POINTER(QmoeDims), c_int, c_int, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("qmoe_ep_rows_workspace_size", c_size_t, [POINTER(QmoeDims), c_int]),
    ("qmoe_ep_experts", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_void_p, c_void_p, c_int, c_int, c_void_p,
                                c_void_p, c_size_t, c_void_p]),
    ("qmoe_ep_experts_return", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_void_p, c_void_p, c_int,
                                       POINTER(QmoeEpReturn), c_void_p, c_size_t, c_void_p]),
    ("qmoe_peer_alloc", c_int, [c_size_t, POINTER(c_void_p), c_void_p]),
    ("qmoe_peer_open", c_int, [c_void_p, POINTER(c_void_p)]),
    ("qmoe_peer_close", c_int, [c_void_p]),
    ("qmoe_peer_free", c_int, [c_void_p]),
    ("qmoe_copy_async", c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    ("qmoe_ep_shared", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_int, c_void_p, c_size_t, c_void_p]),
    ("qmoe_ep_combine_routed", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_void_p, c_void_p, c_int, c_void_p,
                                       c_void_p, c_void_p, c_size_t, c_void_p]),
    ("qmoe_ep_combine", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                                c_void_p, c_size_t, c_void_p]),
    ("qmoe_block_kernel_count", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_int]),
    ("qmoe_block_forward", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_void_p, c_void_p, c_void_p, c_int,
                                   c_void_p, c_size_t, c_void_p]),
    ("qmoe_block_forward_prenorm", c_int, [POINTER(QmoeBlock), POINTER(QmoeDims), c_void_p, c_void_p, c_float,
                                           c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    ("qmoe_stack_forward", c_int, [POINTER(QmoeBlock), POINTER(c_void_p), c_int, POINTER(QmoeDims), c_float,
                                   c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    ("qmoe_check_errors", c_int, [c_void_p, POINTER(QmoeDims), POINTER(c_uint32), c_void_p]),
    ("qmoe_trace_enable", c_int, [c_void_p, c_size_t]),
    ("qmoe_trace_bytes", c_size_t, []),
    ("qmoe_workspace_init", c_int, [c_void_p, c_size_t, c_void_p]),
    ("qmoe_workspace_set_error_sink", c_int, [c_void_p, c_void_p, c_void_p]),
    ("qmoe_debug_grid_barrier", c_int, [c_uint64, c_int]),
    ("qmoe_synth_fill", c_int, [c_void_p, c_uint32, c_uint64, c_uint64, c_uint64, c_float, c_void_p]),
    ("qmoe_synth_fill_host", c_int, [c_void_p, c_uint32, c_uint64, c_uint64, c_uint64, c_float]),
    ("qmoe_synth_fill_host_range", c_int, [c_void_p, c_uint32, c_uint64, c_uint64, c_uint64, c_uint64, c_float]),
    ("qmoe_tensor_bytes", c_uint64, [c_uint32, c_uint64]),
]

# include/qmoe_ep.h, exported by libqmoe_ep.so (the expert-parallel host layer over NCCL)
EP_LIB_PATH = Path(__file__).resolve().parent / "libqmoe_ep.so"
QMOE_EP_DIRECT = 1
EP_SIGNATURES = [
    ("qmoe_ep_unique_id", c_int, [c_void_p]),
    ("qmoe_ep_comm_init", c_int, [c_void_p, c_int, c_int, POINTER(c_void_p)]),
    ("qmoe_ep_comm_destroy", c_int, [c_void_p]),
    ("qmoe_ep_init", c_int, [c_void_p, POINTER(QmoeDims), c_int, c_int, POINTER(c_void_p)]),
    ("qmoe_ep_is_direct", c_int, [c_void_p]),
    ("qmoe_ep_forward", c_int, [c_void_p, POINTER(QmoeBlock), POINTER(QmoeBlock), c_void_p, c_void_p, c_void_p,
                                c_float, c_void_p, c_void_p, c_int, c_void_p]),
    ("qmoe_ep_finalize", c_int, [c_void_p]),
]

_lib = None
_ep_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"qmoe CUDA library not built: {LIB_PATH} is missing")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ep_lib() -> ctypes.CDLL:
    """libqmoe_ep.so (loads libqmoe.so and NCCL; raises if it has not been built)."""
    global _ep_lib
    if _ep_lib is None:
        lib()  # the C-ABI it calls into, from this directory
        if not EP_LIB_PATH.exists():
            raise ImportError(f"qmoe expert-parallel library not built: {EP_LIB_PATH} is missing")
        L = ctypes.CDLL(str(EP_LIB_PATH))
        for name, res, args in EP_SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _ep_lib = L
    return _ep_lib


def status_string(st: int) -> str:
    return lib().qmoe_status_string(st).decode()


def check(st: int, what: str = "qmoe") -> None:
    if st != QMOE_OK:
        raise RuntimeError(f"{what}: {status_string(st)} (status {st})")
