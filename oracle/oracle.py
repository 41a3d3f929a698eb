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
SYNTH_LIB = HERE / "libsynth_host.so"

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
        L.or_route_batch.restype = None
        L.or_route_batch.argtypes = [c_void_p, c_int, c_uint64, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                     c_void_p, c_void_p, c_void_p]
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


def route(router: np.ndarray, ggml_type: int, x: np.ndarray, E: int, k: int, bias: np.ndarray | None = None):
    """Router logits (+ bias) and top-k of every row of x: (logits[T][E], idx[T][k], w[T][k])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, d = x.shape
    router = np.ascontiguousarray(router)
    logits = np.zeros((T, E), dtype=np.float32)
    idx = np.zeros((T, k), dtype=np.int32)
    w = np.zeros((T, k), dtype=np.float32)
    bp = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32)
        bp = _p(bias)
    lib().or_route_batch(_p(router), int(ggml_type), E * d, bp, d, E, k, T, _p(x), _p(logits), _p(idx), _p(w))
    return logits, idx, w


def tolerance_report(got: np.ndarray, want: np.ndarray, atol: float = 1e-3, rtol: float = 1e-2) -> dict:
    """Output error against the oracle under the two bounds "max-abs atol /
    rel rtol": an element passes when its absolute error is at most atol or
    its relative error at most rtol.  Reports the largest absolute error,
    the largest relative error among elements with |want| >= atol / rtol
    (where the relative bound is the binding one), and the element count
    outside both bounds."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    diff = np.abs(got - want)
    mag = np.abs(want)
    big = mag >= atol / rtol
    bad = ~((diff <= atol) | (diff <= rtol * mag))
    bad |= ~np.isfinite(got)
    return {"max_abs_err": float(diff.max()) if diff.size else 0.0,
            "max_rel_err": float((diff[big] / mag[big]).max()) if big.any() else 0.0,
            "n_outside": int(bad.sum()), "n": int(diff.size), "within_tol": not bool(bad.any()),
            "tol": f"per element |err| <= {atol:g} or |err|/|want| <= {rtol:g}"}


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
# Seeded synthetic bytes on the host (oracle/libsynth_host.so: the product's
# host generator compiled on its own), for CPU legs that must not load the
# product library.
# ---------------------------------------------------------------------------
_synth = None


def synth_lib() -> ctypes.CDLL:
    global _synth
    if _synth is None:
        if not SYNTH_LIB.exists():
            build()
        L = ctypes.CDLL(str(SYNTH_LIB))
        L.qmoe_synth_fill_host_range.restype = c_int
        L.qmoe_synth_fill_host_range.argtypes = [c_void_p, ctypes.c_uint32, c_uint64, c_uint64, c_uint64, c_uint64,
                                                 c_float]
        _synth = L
    return _synth


def synth_fill(dst: np.ndarray, ggml_type: int, first: int, n: int, seed: int, stream_id: int, sigma: float) -> None:
    """Elements [first, first + n) of the seeded stream, encoded as ggml_type, into dst (uint8)."""
    st = synth_lib().qmoe_synth_fill_host_range(_p(dst), int(ggml_type), first, n, seed, stream_id, sigma)
    if st:
        raise RuntimeError(f"synth_fill status {st}")


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


# ---------------------------------------------------------------------------
# Parity of a large batch (prefill sizes): routing of every token, outputs of
# a sample of tokens.
# ---------------------------------------------------------------------------
def pick_sample(idx: np.ndarray, E: int, n_spread: int = 128, n_cold: int = 8, per_cold: int = 4,
                every_expert: bool = True) -> np.ndarray:
    """Token rows for the output check of a large batch: up to `per_cold`
    tokens of each of the `n_cold` least-hit experts that are hit, the first
    token of every hit expert (with `every_expert`), `n_spread` evenly spaced
    tokens, and the first and last token.  The most-hit experts are in the sample through the
    spread (under Zipf routing nearly every token holds the hottest one)."""
    T = idx.shape[0]
    valid = (idx >= 0) & (idx < E)
    counts = np.bincount(idx[valid].ravel(), minlength=E)
    hit = np.nonzero(counts)[0]
    rows = set([0, T - 1])
    rows.update(np.linspace(0, T - 1, num=min(n_spread, T), dtype=np.int64).tolist())
    for e in hit[np.argsort(counts[hit], kind="stable")][:n_cold]:
        rows.update(np.nonzero((idx == e).any(axis=1))[0][:per_cold].tolist())
    if every_expert:
        for e in hit:
            rows.add(int(np.nonzero((idx == e).any(axis=1))[0][0]))
    return np.array(sorted(rows), dtype=np.int64)


def check_batch(tensors: dict, types: dict, dims, x: np.ndarray, got: dict, bias: np.ndarray | None = None,
                sample: np.ndarray | None = None, atol: float = 1e-3, rtol: float = 1e-2) -> dict:
    """Checks one block call of T tokens against the oracle.  got: device
    results as numpy -- "logits" [T][E], "idx"/"w" [T][k], "offsets" [E+1],
    "perm" [valid pairs], "out" [T][d] (out may be None).  Routing (logits
    bit-exact, ids and selection order, permutation) is checked on every
    token; outputs on `sample` (default: pick_sample of the oracle's ids)."""
    E, k = dims.num_experts, dims.top_k
    x = np.ascontiguousarray(x, dtype=np.float32)
    logits, idx, w = route(tensors["router"], types["router"], x, E, k, bias)
    offs, perm, _ = dispatch(idx, E)
    res = {"tokens": int(x.shape[0]),
           "logits_bit_exact": bool(np.array_equal(np.asarray(got["logits"], np.float32).view(np.uint32),
                                                   logits.view(np.uint32))),
           "ids_bit_exact": bool(np.array_equal(got["idx"], idx)),
           "weights_max_rel_err": float(np.max(np.abs(got["w"] - w) / np.maximum(np.abs(w), 1e-30))),
           "offsets_bit_exact": bool(np.array_equal(got["offsets"], offs)),
           "perm_bit_exact": bool(np.array_equal(np.asarray(got["perm"])[:perm.size], perm))}
    if got.get("out") is not None:
        if sample is None:
            sample = pick_sample(idx, E)
        want = moe_forward(tensors, types, dims, x[sample], bias)
        rep = tolerance_report(np.asarray(got["out"])[sample], want["out"], atol, rtol)
        rep["sample_tokens"] = int(sample.size)
        rep["oracle_status_ok"] = bool(np.all(want["status"] == 0))
        res["out"] = rep
    res["routing_ok"] = (res["logits_bit_exact"] and res["ids_bit_exact"] and res["offsets_bit_exact"]
                         and res["perm_bit_exact"] and res["weights_max_rel_err"] <= 2e-6)
    res["within_tol"] = res["routing_ok"] and (res.get("out") is None or res["out"]["within_tol"])
    return res
