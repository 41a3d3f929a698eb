"""ctypes wrapper of the CPU oracle (oracle/qmoe_oracle.c) and of the
reference's own CUDA MoE path built into oracle/_ref/ (oracle/build_ref.sh).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product.
"""
from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_float, c_int, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libqwenref.so"

TENSORS = ["router", "gate_exps", "up_exps", "down_exps", "shared_gate_inp", "shared_gate", "shared_up",
           "shared_down"]


class OrTensor(ctypes.Structure):
    _fields_ = [("data", c_void_p), ("type", c_int), ("num_elements", c_uint64)]


class OrBlock(ctypes.Structure):
    _fields_ = [(n, OrTensor) for n in TENSORS] + [("expert_bias", c_void_p)]


_lib = None


def build() -> None:
    subprocess.run(["bash", str(HERE / "build_oracle.sh")], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        L.or_dequant.restype = c_float
        L.or_dequant.argtypes = [c_void_p, c_int, c_uint64]
        L.or_gemv.restype = c_int
        L.or_gemv.argtypes = [c_void_p, c_int, c_uint64, c_void_p, c_void_p, c_int, c_int, c_uint64]
        L.or_dequantize_row.restype = c_int
        L.or_dequantize_row.argtypes = [c_void_p, c_int, c_uint64, c_void_p, c_int, c_int]
        L.or_topk.restype = None
        L.or_topk.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int]
        L.or_moe_forward_batch.restype = c_int
        L.or_moe_forward_batch.argtypes = [POINTER(OrBlock), c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                           c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                           c_void_p]
        L.or_dispatch.restype = c_int
        L.or_dispatch.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]
        L.or_rmsnorm.restype = None
        L.or_rmsnorm.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_float]
        L.or_set_threads.restype = None
        L.or_set_threads.argtypes = [c_int]
        L.or_max_threads.restype = c_int
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().or_set_threads(n)


def max_threads() -> int:
    return lib().or_max_threads()


def dequant_row(data: np.ndarray, ggml_type: int, n: int, row: int, cols: int) -> np.ndarray:
    out = np.empty(cols, dtype=np.float32)
    st = lib().or_dequantize_row(_p(data), ggml_type, n, _p(out), row, cols)
    if st:
        raise RuntimeError(f"oracle dequantize_row status {st}")
    return out


def gemv(data: np.ndarray, ggml_type: int, n: int, x: np.ndarray, M: int, K: int, off: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(M, dtype=np.float32)
    st = lib().or_gemv(_p(data), ggml_type, n, _p(x), _p(y), M, K, off)
    if st:
        raise RuntimeError(f"oracle gemv status {st}")
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().or_rmsnorm(_p(x), _p(w), _p(out), x.size, eps)
    return out


def topk(logits: np.ndarray, k: int):
    x = np.ascontiguousarray(logits, dtype=np.float32)
    idx = np.zeros(k, dtype=np.int32)
    w = np.zeros(k, dtype=np.float32)
    lib().or_topk(_p(x), _p(idx), _p(w), x.size, k)
    return idx, w


def moe_forward(tensors: dict, types: dict, dims, x: np.ndarray, bias: np.ndarray | None = None):
    """tensors: name -> uint8 numpy payload; dims: object with d_model,
    num_experts, top_k, expert_dim, shared_dim.  Returns a dict."""
    d, E, k, F, Fs = dims.d_model, dims.num_experts, dims.top_k, dims.expert_dim, dims.shared_dim
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, d)
    T = x.shape[0]
    elems = {"router": E * d, "gate_exps": E * F * d, "up_exps": E * F * d, "down_exps": E * d * F,
             "shared_gate_inp": d, "shared_gate": Fs * d, "shared_up": Fs * d, "shared_down": d * Fs}
    keep = []
    fields = []
    for n in TENSORS:
        a = np.ascontiguousarray(tensors[n])
        keep.append(a)
        fields.append(OrTensor(_p(a), int(types[n]), elems[n]))
    bp = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32)
        keep.append(bias)
        bp = _p(bias)
    blk = OrBlock(*fields, bp)
    out = np.zeros((T, d), dtype=np.float32)
    idx = np.zeros((T, k), dtype=np.int32)
    w = np.zeros((T, k), dtype=np.float32)
    status = np.zeros(T, dtype=np.int32)
    logits = np.zeros((T, E), dtype=np.float32)
    h = np.zeros((T, k, F), dtype=np.float32)
    hs = np.zeros((T, Fs), dtype=np.float32)
    sg = np.zeros(T, dtype=np.float32)
    lib().or_moe_forward_batch(ctypes.byref(blk), d, E, k, F, Fs, T, _p(x), _p(out), _p(idx), _p(w), _p(status),
                               _p(logits), _p(h), _p(hs), _p(sg))
    return {"out": out, "idx": idx, "w": w, "status": status, "logits": logits, "h": h, "hs": hs, "sgate": sg}


def dispatch(idx: np.ndarray, E: int):
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    T, k = idx.shape
    offsets = np.zeros(E + 1, dtype=np.int32)
    perm = np.full(T * k, -1, dtype=np.int32)
    inv = np.zeros(T * k, dtype=np.int32)
    n = lib().or_dispatch(_p(idx), T, k, E, _p(offsets), _p(perm), _p(inv))
    return offsets, perm[:n], inv


# ---------------------------------------------------------------------------
# The reference's own CUDA path (oracle/_ref/libqwenref.so), GPU box only.
# ---------------------------------------------------------------------------
_ref = None


def ref_available() -> bool:
    return REF_LIB.exists()


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        L = ctypes.CDLL(str(REF_LIB))
        L.ref_last_error.restype = ctypes.c_char_p
        L.ref_gemv.restype = c_int
        L.ref_gemv.argtypes = [c_void_p, c_int, c_uint64, c_void_p, c_void_p, c_int, c_int, c_uint64, c_void_p]
        L.ref_dequantize_row.restype = c_int
        L.ref_dequantize_row.argtypes = [c_void_p, c_int, c_uint64, c_void_p, c_int, c_int, c_void_p]
        L.ref_rmsnorm.restype = c_int
        L.ref_rmsnorm.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_float, c_void_p]
        L.ref_topk.restype = c_int
        L.ref_topk.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]
        L.ref_moe_forward.restype = c_int
        L.ref_moe_forward.argtypes = [c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                      POINTER(c_void_p), POINTER(c_int), POINTER(c_uint64), c_void_p]
        _ref = L
    return _ref


def ref_moe_forward(dims, ptrs: list, types: list, nelem: list, x_ptr: int, out_ptr: int, T: int, stream=None):
    """Runs the reference MoeLayer::forward on device buffers (one call per token)."""
    P = (c_void_p * 8)(*ptrs)
    Ty = (c_int * 8)(*[int(t) for t in types])
    N = (c_uint64 * 8)(*nelem)
    st = ref_lib().ref_moe_forward(dims.d_model, dims.num_experts, dims.top_k, dims.expert_dim, dims.shared_dim, T,
                                   x_ptr, out_ptr, P, Ty, N, stream)
    if st:
        raise RuntimeError("reference MoE path failed: " + ref_lib().ref_last_error().decode())
