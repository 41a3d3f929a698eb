"""GPU parity tests: every kernel through the C-ABI against the CPU oracle
(and, where it adds a pin, against the reference's own CUDA path in
oracle/_ref).  Routing ids, selection order and the permutation must be
bit-exact; outputs within max-abs 1e-3 / rel 1e-2."""
import ctypes
import json
import zlib
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as orc
from qmoe import _lib, synth
from qmoe.quant import GgmlType, calculate_tensor_bytes

from gpu_util import Run, assert_close, oracle_run, oracle_threads

pytestmark = pytest.mark.gpu
GOLD = json.loads((Path(__file__).parent / "golden" / "quant_kat.json").read_text())
REAL = synth.Dims()  # 2048 / 256 / 8 / 512 / 512


@pytest.fixture(scope="module", autouse=True)
def _setup(cuda):
    oracle_threads()


def _tensor(buf, ty, n):
    return _lib.QmoeTensor(buf.data_ptr(), int(ty), 0, n)


@pytest.mark.parametrize("ty", [GgmlType.F32, GgmlType.F16, GgmlType.BF16, GgmlType.Q4_0, GgmlType.Q5_0,
                                GgmlType.Q8_0, GgmlType.Q4_K, GgmlType.Q5_K, GgmlType.Q6_K])
def test_synth_device_matches_host(ty):
    import torch
    n = 256 * 64
    h = np.empty(calculate_tensor_bytes(ty, n), dtype=np.uint8)
    synth.fill(h, ty, n, 99, 5, 0.02)
    d = torch.empty(h.size, dtype=torch.uint8, device="cuda")
    synth.fill(d, ty, n, 99, 5, 0.02)
    assert np.array_equal(d.cpu().numpy(), h)


@pytest.mark.parametrize("name", sorted(GOLD["quant"]))
def test_dequant_row_kat(name):
    import torch
    fx = GOLD["quant"][name]
    raw = torch.tensor(list(bytes.fromhex(fx["bytes"])), dtype=torch.uint8, device="cuda")
    exp = np.array(fx["expected"], dtype=np.float32)
    out = torch.empty(exp.size, dtype=torch.float32, device="cuda")
    t = _tensor(raw, fx["ggml_type"], exp.size)
    _lib.check(_lib.lib().qmoe_dequant_row(ctypes.byref(t), out.data_ptr(), 0, exp.size, None))
    torch.cuda.synchronize()
    assert np.max(np.abs(out.cpu().numpy() - exp)) < 1e-6


@pytest.mark.parametrize("ty", [GgmlType.F32, GgmlType.F16, GgmlType.BF16, GgmlType.Q4_0, GgmlType.Q5_0,
                                GgmlType.Q8_0, GgmlType.Q4_K, GgmlType.Q5_K, GgmlType.Q6_K])
@pytest.mark.parametrize("K", [2048, 768])
def test_gemv_vs_oracle(ty, K):
    import torch
    if K % 256 and ty in (GgmlType.Q4_K, GgmlType.Q5_K, GgmlType.Q6_K):
        pytest.skip("K-quant rows need K % 256 == 0")
    rows, M, row0 = 96, 37, 11
    n = rows * K
    h = np.empty(calculate_tensor_bytes(ty, n), dtype=np.uint8)
    synth.fill(h, ty, n, 5, 17, 0.02)
    xh = np.random.default_rng(2).standard_normal(K).astype(np.float32)
    w = torch.from_numpy(h).cuda()
    x = torch.from_numpy(xh).cuda()
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    t = _tensor(w, ty, n)
    # the reference-order kernel (bit-level checks below) ...
    _lib.check(_lib.lib().qmoe_gemv_exact(ctypes.byref(t), x.data_ptr(), y.data_ptr(), M, K, row0 * K, None))
    torch.cuda.synchronize()
    want = orc.gemv(h, int(ty), n, xh, M, K, row0 * K)
    got = y.cpu().numpy()
    # ... and the default path (the streaming unit decoder where it applies)
    yd = torch.empty(M, dtype=torch.float32, device="cuda")
    _lib.check(_lib.lib().qmoe_gemv(ctypes.byref(t), x.data_ptr(), yd.data_ptr(), M, K, row0 * K, None))
    torch.cuda.synchronize()
    assert np.allclose(yd.cpu().numpy(), want, rtol=1e-5, atol=1e-5)
    if ty == GgmlType.F32:
        assert np.array_equal(got, want)  # same reduction order, bit for bit
    else:
        assert np.allclose(got, want, rtol=1e-5, atol=1e-6)
    if orc.ref_available():
        yr = torch.empty(M, dtype=torch.float32, device="cuda")
        st = orc.ref_lib().ref_gemv(w.data_ptr(), int(ty), n, x.data_ptr(), yr.data_ptr(), M, K, row0 * K, None)
        assert st == 0
        torch.cuda.synchronize()
        ref = yr.cpu().numpy()
        if ty in (GgmlType.F32, GgmlType.F16, GgmlType.BF16):
            assert np.array_equal(got, ref)
            assert np.array_equal(want, ref)
        else:
            assert np.allclose(got, ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("ty", [GgmlType.Q4_K, GgmlType.Q5_K, GgmlType.Q6_K, GgmlType.Q8_0])
@pytest.mark.parametrize("K,M,row0", [(256, 1000, 3), (1024, 777, 0), (2048, 1203, 5), (4096, 301, 2)])
def test_gemv_stream_vs_oracle(ty, K, M, row0):
    """The streaming GEMV (bulk-copied row chunks, unit decoders against the
    24-bit planes of x) over many chunks and CTAs, a ragged last chunk and a
    row offset: within 1e-5 of the oracle's F32 products."""
    import torch
    rows = M + row0 + 1
    n = rows * K
    h = np.empty(calculate_tensor_bytes(ty, n), dtype=np.uint8)
    synth.fill(h, ty, n, 7, 19, 0.02)
    xh = np.random.default_rng(K + M).standard_normal(K).astype(np.float32)
    w = torch.from_numpy(h).cuda()
    x = torch.from_numpy(xh).cuda()
    y = torch.full((M + 1,), float("nan"), dtype=torch.float32, device="cuda")
    t = _tensor(w, ty, n)
    _lib.check(_lib.lib().qmoe_gemv(ctypes.byref(t), x.data_ptr(), y.data_ptr(), M, K, row0 * K, None))
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    want = orc.gemv(h, int(ty), n, xh, M, K, row0 * K)
    assert np.isnan(got[M])  # nothing written past row M-1
    assert np.allclose(got[:M], want, rtol=1e-5, atol=1e-5), np.max(np.abs(got[:M] - want))


@pytest.mark.parametrize("K,M,row0", [(2048, 1203, 5), (256, 777, 3), (4096, 301, 2)])
def test_gemv_on_repacked_q6k(K, M, row0):
    """qmoe_repack to QMOE_LAYOUT_Q6K_A16 (each 210-byte super-block in a
    224-byte slot) and qmoe_gemv on the repacked copy: the bytes match the
    padded GGUF blocks and the products are bit-identical to the GEMV on the
    GGUF layout (same unit decoder, aligned reads)."""
    import torch
    ty = GgmlType.Q6_K
    rows = M + row0 + 1
    n = rows * K
    h = np.empty(calculate_tensor_bytes(ty, n), dtype=np.uint8)
    synth.fill(h, ty, n, 9, 23, 0.02)
    w = torch.from_numpy(h).cuda()
    t = _tensor(w, ty, n)
    nb = _lib.lib().qmoe_repack_bytes(int(ty), n, _lib.QMOE_LAYOUT_Q6K_A16)
    assert nb == n // 256 * 224
    wr = torch.full((nb,), 0x5A, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().qmoe_repack(ctypes.byref(t), _lib.QMOE_LAYOUT_Q6K_A16, wr.data_ptr(), nb, None))
    torch.cuda.synchronize()
    want_bytes = np.zeros((n // 256, 224), dtype=np.uint8)
    want_bytes[:, :210] = h.reshape(-1, 210)
    assert np.array_equal(wr.cpu().numpy().reshape(-1, 224), want_bytes)
    tr = _lib.QmoeTensor(wr.data_ptr(), int(ty), _lib.QMOE_LAYOUT_Q6K_A16, n)
    x = torch.from_numpy(np.random.default_rng(K).standard_normal(K).astype(np.float32)).cuda()
    y0 = torch.empty(M, device="cuda")
    y1 = torch.full((M,), float("nan"), device="cuda")
    _lib.check(_lib.lib().qmoe_gemv(ctypes.byref(t), x.data_ptr(), y0.data_ptr(), M, K, row0 * K, None))
    _lib.check(_lib.lib().qmoe_gemv(ctypes.byref(tr), x.data_ptr(), y1.data_ptr(), M, K, row0 * K, None))
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
    # the repacked layout is read by the streaming GEMV only
    assert _lib.lib().qmoe_gemv_exact(ctypes.byref(tr), x.data_ptr(), y1.data_ptr(), M, K, 0, None) == \
        _lib.QMOE_ERR_UNSUPPORTED
    assert _lib.lib().qmoe_dequant_row(ctypes.byref(tr), y1.data_ptr(), 0, K, None) == _lib.QMOE_ERR_UNSUPPORTED


def _router_block(dims, bias, seed):
    return synth.Block(dims, synth.Q4K_TYPES, seed=seed, device="cuda", bias=bias)


@pytest.mark.parametrize("T,bias,seed", [(1, False, 1), (3, False, 2), (8, False, 3), (8, True, 4), (5, True, 5)])
def test_router_topk_bit_exact(T, bias, seed):
    import torch
    blk = _router_block(REAL, bias, seed)
    r = Run(blk)
    x = synth.inputs(T, REAL.d_model, seed=seed, tag=7)
    idx = torch.empty((T, REAL.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, REAL.top_k), dtype=torch.float32, device="cuda")
    c = blk.c()
    _lib.check(_lib.lib().qmoe_router_topk(ctypes.byref(c), ctypes.byref(r.dims), x.data_ptr(), T, idx.data_ptr(),
                                           w.data_ptr(), r.ws.data_ptr(), r.ws_bytes, None))
    torch.cuda.synchronize()
    E, k = REAL.num_experts, REAL.top_k
    logits = r.view(_lib.WS_LOGITS, T, T * (E + 1), np.float32).reshape(T, E + 1)
    xh = x.cpu().numpy()
    router = blk.host_bytes("router")
    bh = blk.host_bias()
    for t in range(T):
        want = orc.gemv(router, 0, E * REAL.d_model, xh[t], E, REAL.d_model)
        if bh is not None:
            want = (want + bh).astype(np.float32)
        assert np.array_equal(logits[t, :E], want), t  # bit-exact logits
        oi, ow = orc.topk(want, k)
        assert idx[t].cpu().numpy().tolist() == oi.tolist()
        assert np.allclose(w[t].cpu().numpy(), ow, rtol=2e-6, atol=0)
        sg = orc.gemv(blk.host_bytes("shared_gate_inp"), 0, REAL.d_model, xh[t], 1, REAL.d_model)
        assert logits[t, E] == sg[0]
        if orc.ref_available():  # the reference's own top-k kernel on the same logits
            lt = torch.from_numpy(np.ascontiguousarray(logits[t, :E])).cuda()
            ri = torch.empty(k, dtype=torch.int32, device="cuda")
            rw = torch.empty(k, dtype=torch.float32, device="cuda")
            assert orc.ref_lib().ref_topk(lt.data_ptr(), ri.data_ptr(), rw.data_ptr(), E, k, None) == 0
            torch.cuda.synchronize()
            assert ri.cpu().numpy().tolist() == idx[t].cpu().numpy().tolist()
            assert np.array_equal(rw.cpu().numpy(), w[t].cpu().numpy())  # same expf, same order
    st, flags, tok = r.check_errors()
    assert st == 0 and flags == 0


def test_routing_kat_through_router_kernel():
    """tests/kernel_tests.cu:424-453: logits {-2,.4,3,1.2,-.7,2.1}, K=3 -> {2,5,3}."""
    import torch
    g = GOLD["routing"]
    dims = synth.Dims(d_model=256, num_experts=6, top_k=3, expert_dim=256, shared_dim=256)
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=1, device="cuda")
    W = np.zeros((6, 256), dtype=np.float32)
    W[:, 0] = g["logits"]
    blk.buf["router"].copy_(torch.from_numpy(W.view(np.uint8).ravel()))
    x = torch.zeros((1, 256), dtype=torch.float32, device="cuda")
    x[0, 0] = 1.0
    r = Run(blk)
    idx = torch.empty(3, dtype=torch.int32, device="cuda")
    w = torch.empty(3, dtype=torch.float32, device="cuda")
    c = blk.c()
    _lib.check(_lib.lib().qmoe_router_topk(ctypes.byref(c), ctypes.byref(r.dims), x.data_ptr(), 1, idx.data_ptr(),
                                           w.data_ptr(), r.ws.data_ptr(), r.ws_bytes, None))
    torch.cuda.synchronize()
    assert idx.cpu().numpy().tolist() == g["ids"]
    wh = w.cpu().numpy()
    assert np.all(wh > 0) and abs(float(wh.sum()) - 1) < g["sum_tol"] and wh[0] > wh[1] > wh[2]


CASES = [
    ("config1_q4k_T4", REAL, synth.Q4K_TYPES, False, 4),
    ("q4k_T1", REAL, synth.Q4K_TYPES, False, 1),
    ("mixed_bias_T1", REAL, synth.MIXED_TYPES, True, 1),
    ("mixed_bias_T2", REAL, synth.MIXED_TYPES, True, 2),
    # fused kernel with several items per CTA and several down rounds
    ("mixed_bias_T3", REAL, synth.MIXED_TYPES, True, 3),
    # gate/up and down as two kernels (batches of more than 4 tokens)
    ("mixed_bias_T8", REAL, synth.MIXED_TYPES, True, 8),
    ("small_q5k_q80", synth.Dims(512, 64, 6, 256, 512),
     {**synth.Q4K_TYPES, "gate_exps": GgmlType.Q5_K, "up_exps": GgmlType.Q5_K, "down_exps": GgmlType.Q8_0,
      "shared_gate": GgmlType.Q6_K, "shared_up": GgmlType.Q6_K, "shared_down": GgmlType.Q5_K}, False, 3),
    ("small_q6k_F1024", synth.Dims(1024, 32, 4, 1024, 256),
     {**synth.Q4K_TYPES, "down_exps": GgmlType.Q6_K, "shared_down": GgmlType.Q6_K}, True, 5),
]


@pytest.mark.parametrize("name,dims,types,bias,T", CASES, ids=[c[0] for c in CASES])
def test_block_forward_vs_oracle(name, dims, types, bias, T):
    blk = synth.Block(dims, types, seed=zlib.crc32(name.encode()) & 0xFFFF, device="cuda", bias=bias)
    r = Run(blk)
    x = synth.inputs(T, dims.d_model, seed=77, tag=T)
    out = r.forward(x).cpu().numpy()
    want = oracle_run(blk, x.cpu().numpy())
    assert np.all(want["status"] == 0)
    k = dims.top_k
    idx = r.view(_lib.WS_TOPK_IDX, T, T * k, np.int32).reshape(T, k)
    assert np.array_equal(idx, want["idx"])
    wts = r.view(_lib.WS_TOPK_W, T, T * k, np.float32).reshape(T, k)
    assert np.allclose(wts, want["w"], rtol=2e-6, atol=0)
    H = max(dims.expert_dim, dims.shared_dim)
    hid = r.view(_lib.WS_HIDDEN, T, (T * k + T) * H, np.float32).reshape(T * k + T, H)
    F, Fs = dims.expert_dim, dims.shared_dim
    assert_close(hid[: T * k, :F].reshape(T, k, F), want["h"], f"{name} hidden")
    assert_close(hid[T * k:, :Fs], want["hs"], f"{name} shared hidden")
    assert_close(out, want["out"], f"{name} out")
    # permutation = stable order by (expert, token, slot)
    offs, perm, _ = orc.dispatch(want["idx"], dims.num_experts)
    assert np.array_equal(r.view(_lib.WS_OFFSETS, T, dims.num_experts + 1, np.int32), offs)
    assert np.array_equal(r.view(_lib.WS_PERM, T, T * k, np.int32)[: perm.size], perm)
    st, flags, _ = r.check_errors()
    assert st == 0 and flags == 0


@pytest.mark.parametrize("name,dims,types,bias,T", [CASES[i] for i in (1, 3, 4, 6)],
                         ids=[CASES[i][0] for i in (1, 3, 4, 6)])
def test_stage_entry_points_vs_block_forward(name, dims, types, bias, T):
    """router_topk -> expert_gateup -> down_combine (two expert kernels) and
    block_forward (fused expert kernel where an instance exists) agree with
    the oracle and with each other."""
    blk = synth.Block(dims, types, seed=zlib.crc32(name.encode()) & 0xFFFF, device="cuda", bias=bias)
    r = Run(blk)
    x = synth.inputs(T, dims.d_model, seed=78, tag=T)
    res = synth.inputs(T, dims.d_model, seed=79, tag=T)
    want = oracle_run(blk, x.cpu().numpy())
    a = r.staged(x, res).cpu().numpy()
    ida = r.view(_lib.WS_TOPK_IDX, T, T * dims.top_k, np.int32).copy()
    b = r.forward(x, res).cpu().numpy()
    idb = r.view(_lib.WS_TOPK_IDX, T, T * dims.top_k, np.int32).copy()
    assert np.array_equal(ida, idb) and np.array_equal(ida.reshape(T, -1), want["idx"])
    base = want["out"] + res.cpu().numpy()
    # router_topk followed by the one-step expert entry point
    import torch
    c = blk.c()
    L = _lib.lib()
    out3 = torch.full_like(x, float("nan"))
    _lib.check(L.qmoe_router_topk(ctypes.byref(c), ctypes.byref(r.dims), x.data_ptr(), T, None, None,
                                  r.ws.data_ptr(), r.ws_bytes, None))
    _lib.check(L.qmoe_expert_block(ctypes.byref(c), ctypes.byref(r.dims), T, out3.data_ptr(), res.data_ptr(),
                                   r.ws.data_ptr(), r.ws_bytes, None))
    torch.cuda.synchronize()
    assert_close(out3.cpu().numpy(), base, f"{name} expert_block")
    assert L.qmoe_block_kernel_count(ctypes.byref(c), ctypes.byref(r.dims), T) in (2, 3)
    assert_close(a, base, f"{name} staged")
    assert_close(b, base, f"{name} block_forward")
    assert_close(a, b, f"{name} staged vs block_forward")
    st, flags, _ = r.check_errors()
    assert st == 0 and flags == 0


def test_block_forward_vs_reference_cuda_path():
    """Config 1 through the reference's own MoeLayer::forward (oracle/_ref):
    pins the oracle to the reference and the product to both."""
    import torch
    if not orc.ref_available():
        pytest.skip("oracle/_ref not built")
    dims, T = REAL, 4
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=4242, device="cuda")
    x = synth.inputs(T, dims.d_model, seed=4242, tag=1)
    ref_out = torch.full_like(x, float("nan"))
    names = synth.TENSORS
    orc.ref_moe_forward(dims, [blk.buf[n].data_ptr() for n in names], [blk.types[n] for n in names],
                        [dims.elements(n) for n in names], x.data_ptr(), ref_out.data_ptr(), T)
    torch.cuda.synchronize()
    ref = ref_out.cpu().numpy()
    want = oracle_run(blk, x.cpu().numpy())
    # oracle vs reference: same formulas and reduction order; only expf/contraction may differ
    assert np.allclose(want["out"], ref, rtol=1e-5, atol=1e-6)
    got = Run(blk).forward(x).cpu().numpy()
    assert_close(got, ref, "product vs reference CUDA path")


def test_slabs_residual_and_nonfinite_token():
    import torch
    dims, T = REAL, 12  # two decode slabs (8 + 4)
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=9, device="cuda")
    r = Run(blk)
    x = synth.inputs(T, dims.d_model, seed=9, tag=12).clone()
    x[10, 5] = float("nan")
    resid = synth.inputs(T, dims.d_model, seed=10, tag=13)
    out = r.forward(x, residual=resid).cpu().numpy()
    xh = x.cpu().numpy()
    want = oracle_run(blk, xh)
    assert want["status"].tolist() == [0] * 10 + [10, 0]
    good = [t for t in range(T) if t != 10]
    assert_close(out[good], want["out"][good] + resid.cpu().numpy()[good], "residual")
    assert np.all(np.isnan(out[10]))
    st, flags, tok = r.check_errors()
    assert st == _lib.QMOE_ERR_ROUTING and flags & 1 and tok == 2  # token 2 of the second slab
    st, flags, tok = r.check_errors()  # cleared
    assert st == 0 and flags == 0


def test_dispatch_vs_oracle():
    import torch
    rng = np.random.default_rng(3)
    T, k, E = 4096, 8, 256
    p = 1.0 / np.arange(1, E + 1) ** 1.1
    p /= p.sum()
    idx = np.stack([rng.choice(E, k, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    offs, perm, inv = orc.dispatch(idx, E)
    d_idx = torch.from_numpy(idx).cuda()
    o = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    pm = torch.empty(T * k, dtype=torch.int32, device="cuda")
    iv = torch.empty(T * k, dtype=torch.int32, device="cuda")
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().qmoe_dispatch(d_idx.data_ptr(), T, k, E, o.data_ptr(), pm.data_ptr(), iv.data_ptr(),
                                        ws.data_ptr(), ws.numel(), None))
    torch.cuda.synchronize()
    assert np.array_equal(o.cpu().numpy(), offs)
    assert np.array_equal(pm.cpu().numpy(), perm)
    assert np.array_equal(iv.cpu().numpy(), inv)


@pytest.mark.parametrize("T", [1, 3])
def test_fused_prenorm_block(T):
    """model.cpp:208-211 fused: out = resid + MoE(rmsnorm(resid) * w).  The
    normalised input must be bit-identical to the reference's own rmsnorm
    kernel (oracle/_ref); the rest is checked against the oracle."""
    import torch
    dims = REAL
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=31, device="cuda")
    r = Run(blk)
    resid = synth.inputs(T, dims.d_model, seed=31, tag=40) * 3.0
    nw = 1.0 + 0.1 * synth.inputs(1, dims.d_model, seed=31, tag=41)[0]
    out = torch.full_like(resid, float("nan"))
    c = blk.c()
    eps = 1e-6
    _lib.check(_lib.lib().qmoe_block_forward_prenorm(ctypes.byref(c), ctypes.byref(r.dims), resid.data_ptr(),
                                                     nw.data_ptr(), eps, out.data_ptr(), T, r.ws.data_ptr(),
                                                     r.ws_bytes, None))
    torch.cuda.synchronize()
    xin = r.view(_lib.WS_INPUT, T, T * dims.d_model, np.float32).reshape(T, dims.d_model)
    rh, wh = resid.cpu().numpy(), nw.cpu().numpy()
    for t in range(T):
        assert np.allclose(xin[t], orc.rmsnorm(rh[t], wh, eps), rtol=5e-7, atol=0)
        if orc.ref_available():
            ref = torch.empty(dims.d_model, dtype=torch.float32, device="cuda")
            assert orc.ref_lib().ref_rmsnorm(resid[t].data_ptr(), nw.data_ptr(), ref.data_ptr(), dims.d_model, eps,
                                             None) == 0
            torch.cuda.synchronize()
            assert np.array_equal(xin[t], ref.cpu().numpy())
    want = oracle_run(blk, xin)
    idx = r.view(_lib.WS_TOPK_IDX, T, T * dims.top_k, np.int32).reshape(T, dims.top_k)
    assert np.array_equal(idx, want["idx"])
    assert_close(out.cpu().numpy(), rh + want["out"], "prenorm block")
