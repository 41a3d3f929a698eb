"""Pins the CPU oracle (oracle/qmoe_oracle.c) before it is trusted:
  * against the reference's own known-answer tests (tests/golden, from
    tests/kernel_tests.cu:116-223 and :424-453 of the reference);
  * against independent restatements (gguf-py decoders + numpy float64 math,
    pure-Python evaluation of the reference's GEMV reduction tree).
CPU only."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as orc

GOLD = json.loads((Path(__file__).parent / "golden" / "quant_kat.json").read_text())


@pytest.mark.parametrize("name", sorted(GOLD["quant"]))
def test_quant_kat(name):
    fx = GOLD["quant"][name]
    raw = np.frombuffer(bytes.fromhex(fx["bytes"]), dtype=np.uint8).copy()
    exp = np.array(fx["expected"], dtype=np.float32)
    got = orc.dequant_row(raw, fx["ggml_type"], exp.size, 0, exp.size)
    assert np.all(np.isfinite(got))
    assert np.max(np.abs(got - exp)) < GOLD["routing"]["abs_tol_quant"]


def test_routing_kat():
    r = GOLD["routing"]
    idx, w = orc.topk(np.array(r["logits"], dtype=np.float32), r["k"])
    assert idx.tolist() == r["ids"]
    assert np.all(np.isfinite(w)) and np.all(w > 0)
    assert abs(float(w.sum()) - 1.0) < r["sum_tol"]
    assert w[0] > w[1] > w[2]


def test_topk_ties_lowest_index_first():
    x = np.array([1.0, 3.0, 3.0, -0.0, 0.0, 3.0, 2.0], dtype=np.float32)
    idx, _ = orc.topk(x, 5)
    assert idx.tolist() == [1, 2, 5, 6, 0]
    idx, _ = orc.topk(np.array([0.0, -0.0, 0.0], dtype=np.float32), 3)
    assert idx.tolist() == [0, 1, 2]


def test_topk_nonfinite_sentinel():
    idx, w = orc.topk(np.array([1.0, np.nan, 2.0], dtype=np.float32), 2)
    assert idx[0] == -1 and np.isnan(w[0])
    idx, w = orc.topk(np.array([1.0, np.inf, 2.0], dtype=np.float32), 2)
    assert idx[0] == -1 and np.isnan(w[0])


def _py_gemv_row(wrow, x):
    """Pure-Python evaluation of matmul_q4.cu:140-167 for one F32 row
    (256 threads; fmaf chain k = t, t+256, ...; shuffle trees)."""
    f = np.float32
    K = len(x)
    part = []
    for t in range(256):
        s = f(0.0)
        for k in range(t, K, 256):
            s = f(np.float64(wrow[k]) * np.float64(x[k]) + np.float64(s))  # fmaf: exact product, one rounding
        part.append(s)

    def tree(v):
        v = list(v)
        off = 16
        while off:
            for i in range(off):
                v[i] = f(v[i] + v[i + off])
            off >>= 1
        return v[0]
    warps = [tree(part[32 * w: 32 * w + 32]) for w in range(8)] + [f(0.0)] * 24
    return tree(warps)


def test_gemv_reduction_order_bit_exact():
    rng = np.random.default_rng(5)
    M, K = 6, 768
    w = rng.standard_normal((M, K)).astype(np.float32) * 0.02
    x = rng.standard_normal(K).astype(np.float32)
    y = orc.gemv(w.view(np.uint8).ravel(), 0, M * K, x, M, K)
    for r in range(M):
        assert y[r] == _py_gemv_row(w[r], x), r


def test_gemv_shape_checks():
    w = np.zeros(64 * 4, dtype=np.uint8)
    with pytest.raises(RuntimeError):
        orc.gemv(w, 0, 64, np.zeros(32, np.float32), 3, 32)  # 96 > 64 elements


def test_dispatch_stable():
    rng = np.random.default_rng(1)
    T, k, E = 97, 8, 40
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    idx[5, :] = -1  # an errored token is excluded
    offsets, perm, inv = orc.dispatch(idx, E)
    pairs = sorted(((int(idx[t, j]), t, j) for t in range(T) for j in range(k) if idx[t, j] >= 0))
    assert perm.tolist() == [t * k + j for (_, t, j) in pairs]
    cnt = np.bincount(idx[idx >= 0], minlength=E)
    assert offsets.tolist() == [0] + np.cumsum(cnt).tolist()
    for pos, p in enumerate(perm):
        assert inv[p] == pos
    assert np.all(inv[5 * k: 6 * k] == -1)


def _gguf_matrix(raw, ggml_type, rows, cols):
    from gguf import GGMLQuantizationType, quants
    if ggml_type == 0:
        return raw.view(np.float32).reshape(rows, cols).astype(np.float64)
    name = {8: "Q8_0", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}[ggml_type]
    return quants.dequantize(raw, getattr(GGMLQuantizationType, name)).reshape(rows, cols).astype(np.float64)


@pytest.mark.parametrize("mixed", [False, True])
def test_moe_forward_vs_float64_restatement(mixed):
    """The oracle's expert compute against numpy float64 with gguf-py
    decoders (independent of both the oracle and the reference code)."""
    from qmoe import synth
    dims = synth.Dims(d_model=256, num_experts=16, top_k=4, expert_dim=256, shared_dim=256)
    blk = synth.Block(dims, synth.MIXED_TYPES if mixed else synth.Q4K_TYPES, seed=11, device="cpu", bias=mixed)
    x = synth.inputs(3, dims.d_model, seed=11, device="cpu")
    res = orc.moe_forward({n: blk.host_bytes(n) for n in synth.TENSORS}, blk.types, dims, x, blk.host_bias())
    d, E, k, F, Fs = 256, 16, 4, 256, 256
    W = {n: _gguf_matrix(blk.host_bytes(n), int(blk.types[n]),
                         *{"router": (E, d), "gate_exps": (E * F, d), "up_exps": (E * F, d),
                           "down_exps": (E * d, F), "shared_gate_inp": (1, d), "shared_gate": (Fs, d),
                           "shared_up": (Fs, d), "shared_down": (d, Fs)}[n]) for n in synth.TENSORS}
    bias = blk.host_bias()
    for t in range(3):
        xt = x[t].astype(np.float64)
        logits = W["router"] @ xt + (bias if bias is not None else 0)
        idx = res["idx"][t]
        # ids/order: the oracle's choice is the float64 top-k unless a near-tie
        order = np.argsort(-logits, kind="stable")[:k]
        gaps = np.diff(np.sort(logits)[::-1][: k + 1])
        if np.min(np.abs(gaps)) > 1e-5:
            assert idx.tolist() == order.tolist()
        sel = logits[idx]
        wt = np.exp(sel - sel.max()); wt /= wt.sum()
        assert np.allclose(res["w"][t], wt, rtol=1e-5, atol=1e-6)
        acc = np.zeros(d)
        for j, e in enumerate(idx):
            g = W["gate_exps"][e * F:(e + 1) * F] @ xt
            u = W["up_exps"][e * F:(e + 1) * F] @ xt
            h = g / (1 + np.exp(-g)) * u
            assert np.allclose(res["h"][t, j], h, rtol=1e-4, atol=1e-5)
            acc += wt[j] * (W["down_exps"][e * d:(e + 1) * d] @ h)
        s = (W["shared_gate_inp"] @ xt)[0]
        g = W["shared_gate"] @ xt
        u = W["shared_up"] @ xt
        acc += (W["shared_down"] @ (g / (1 + np.exp(-g)) * u)) / (1 + np.exp(-s))
        assert np.allclose(res["out"][t], acc, rtol=1e-4, atol=1e-5)
        assert res["status"][t] == 0


def test_moe_forward_nonfinite_input_is_routing_error():
    from qmoe import synth
    dims = synth.Dims(d_model=256, num_experts=16, top_k=4, expert_dim=256, shared_dim=256)
    blk = synth.Block(dims, seed=3, device="cpu")
    x = synth.inputs(2, dims.d_model, seed=3, device="cpu").copy()
    x[1, 7] = np.nan
    res = orc.moe_forward({n: blk.host_bytes(n) for n in synth.TENSORS}, blk.types, dims, x)
    assert res["status"].tolist() == [0, 10]
