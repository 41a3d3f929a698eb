#!/usr/bin/env python
"""MoE-block benchmark on B200.

Workload: decode, batch 1, through the 40 MoE blocks of a
Qwen3.5-35B-A3B-shaped stack (hidden 2048, 256 experts, top-8 + 1 shared,
expert FFN 512), random Q4_K expert weights per layer (N(0,0.02), seeded),
F32 router and shared-gate vector, token vectors ~N(0,1) from a 128-token
seeded pool.  One step = one token through all 40 blocks; each block is the
MoE half of a decoder layer as model.cpp:208-211 runs it -- RMSNorm of the
residual stream, MoE block, residual add -- with the norm and the add fused
into the block's kernels, so block l+1 reads block l's output and the 40
blocks run in sequence like in the model.  Metric: microseconds per token per MoE block
(lower is better); ``value`` = device time / (steps * 40) on each GPU, max
over ranks; the ``aggregate`` object gives the whole job's throughput.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (torchrun, one rank per GPU): the headline decode line runs
independent replicas of the same decode stream (decode does not shard:
replicas only); max-over-ranks device time per GPU, aggregate tokens/s over
all GPUs.  The path that shards is prefill: the
``ep_prefill`` object runs T=16384 tokens through one
block with the experts split over the N GPUs and NCCL all-to-all between
them; at N = 1 it is the same block on one GPU.
--impl reference: the reference's CPU path for the same op (the C
restatement in oracle/, all host threads), rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "qwen-3.5-cuda_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "MoE-block µs/token decode (HBM GB/s) & prefill tokens/s at 1/2/4/8 B200"
UNIT = "us/token"
N_LAYERS = 40
POOL = 128
SEED = 1234
EPS = 1e-6
# algorithmic bytes of one Q4_K MoE block for one token (router F32 + 8 experts
# x (gate+up+down) + shared gate/up/down + shared gate vector + x in/out)
BLOCK_BYTES = 2_097_152 + 8 * 1_769_472 + 1_769_472 + 8_192 + 16_384
# the dominant kernel (fused expert launch) for one token: 8 routed experts and
# the shared expert (gate+up+down rows), the block input x_in and the residual
# it reads, the output it writes
EXPERT_BYTES = 9 * 1_769_472 + 3 * 8_192
WORKLOAD = ("config2: decode batch 1, 40 MoE blocks of a Qwen3.5-35B-A3B-shaped stack "
            "(d=2048, E=256, top-8, F=512, shared 512), Q4_K experts, F32 router/shared gate")


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# DRAM bytes (read + write) of one k_experts launch, from an ncu capture of the
# same kernel on the same workload shape (dram__bytes_read.sum +
# dram__bytes_write.sum; the capture command is in
# profiles/k_experts_decode_q4k.md).  Imported, not measured by this run.
EXPERT_TRAFFIC_BYTES = 16_035_840


class ClockSampler(threading.Thread):
    """NVML clocks/throttle reasons sampled during the timed region."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, dev_index: int):
        super().__init__(daemon=True)
        self.samples, self.reasons, self.max_mhz, self.ok = [], set(), None, False
        self._halt = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(dev_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 - NVML is optional
            self.ok = False

    def run(self):
        if not self.ok:
            return
        nv = self.nv
        get_r = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._halt.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = get_r(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.002)

    def stop(self):
        self._halt.set()
        self.join(timeout=2)
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------
def run_ours(args):
    import datetime

    import torch
    import torch.distributed as dist

    from qmoe import _lib, synth

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    L = args.layers
    dims = synth.Dims()
    dc = dims.c()
    blocks = [synth.Block(dims, synth.Q4K_TYPES, seed=SEED, layer=l, device="cuda") for l in range(L)]
    cblocks = [b.c() for b in blocks]
    inputs = synth.inputs(POOL, dims.d_model, seed=SEED, tag=2)
    gamma = torch.ones(dims.d_model, dtype=torch.float32, device="cuda")  # pre-MoE RMSNorm weight
    nws = _lib.lib().qmoe_workspace_size(ctypes.byref(dc), 1)
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().qmoe_workspace_init(ws.data_ptr(), nws, None))
    xbuf = torch.empty((1, dims.d_model), dtype=torch.float32, device="cuda")
    bufs = [torch.empty_like(xbuf), torch.empty_like(xbuf)]
    fwd = _lib.lib().qmoe_block_forward_prenorm

    def step(stream_ptr):
        # residual stream r: r <- r + MoE_l(rmsnorm(r) * gamma), layer by layer
        x = xbuf
        for l in range(L):
            out = bufs[l % 2]
            st = fwd(ctypes.byref(cblocks[l]), ctypes.byref(dc), x.data_ptr(), gamma.data_ptr(), EPS, out.data_ptr(),
                     1, ws.data_ptr(), nws, stream_ptr)
            if st:
                raise RuntimeError(f"block_forward layer {l}: {_lib.status_string(st)}")
            x = out
        return x

    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(3):
            xbuf.copy_(inputs[i:i + 1])
            final = step(s.cuda_stream)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        final = step(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()

    # warm-up
    for i in range(args.warmup):
        xbuf.copy_(inputs[i % POOL:i % POOL + 1], non_blocking=True)
        g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        xbuf.copy_(inputs[i % POOL:i % POOL + 1], non_blocking=True)
        g.replay()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    if world > 1:
        dist.barrier()

    # end to end through the C-ABI: pinned host input -> device, 40 blocks,
    # result -> pinned host, synchronised every token like a decode loop
    h_in = inputs.cpu().pin_memory()
    h_out = torch.empty((POOL, dims.d_model), dtype=torch.float32).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        xbuf.copy_(h_in[i % POOL:i % POOL + 1], non_blocking=True)
        g.replay()
        h_out[i % POOL:i % POOL + 1].copy_(final, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e1.record()
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)

    # the dominant kernel alone: one fused expert launch per layer (each layer's
    # own expert rows, so consecutive launches stream new weights from HBM),
    # on the routing the workspace holds; average launch duration from CUDA
    # events on the launching stream around graph replays of L launches
    expert_block = _lib.lib().qmoe_expert_block
    g.replay()
    torch.cuda.synchronize()
    gk = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gk, stream=s):
        sp = torch.cuda.current_stream().cuda_stream
        for l in range(L):
            st = expert_block(ctypes.byref(cblocks[l]), ctypes.byref(dc), 1, bufs[0].data_ptr(), xbuf.data_ptr(),
                              ws.data_ptr(), nws, sp)
            if st:
                raise RuntimeError(f"expert_block layer {l}: {_lib.status_string(st)}")
    kreps = max(3, min(20, args.steps))
    for _ in range(2):
        gk.replay()
    torch.cuda.synchronize()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record()
    for _ in range(kreps):
        gk.replay()
    k1.record()
    torch.cuda.synchronize()
    kernel_us = k0.elapsed_time(k1) * 1e3 / (kreps * L)
    del gk

    st, flags, _ = _check_errors(_lib, ws, dc)
    if st:
        raise RuntimeError(f"device error word after the run: flags {flags:#x}")
    kernels_per_block = _lib.lib().qmoe_block_kernel_count(ctypes.byref(cblocks[0]), ctypes.byref(dc), 1)

    if world > 1:
        t = torch.tensor([ms, ems, kernel_us], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ems, kernel_us = float(t[0]), float(t[1]), float(t[2])
    del g

    # decode does not shard: N GPUs run N independent replicas of the decode
    # stream, so the time per block and token is per GPU (max over ranks) and
    # the job's throughput is N times one replica's
    per_block_us = ms * 1e3 / (args.steps * L)
    value = per_block_us
    e2e = ems * 1e3 / (args.steps * L)
    peak, peak_kind = _peaks()
    achieved = EXPERT_BYTES / (kernel_us * 1e-6) / 1e9
    block_achieved = BLOCK_BYTES / (per_block_us * 1e-6) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights quantised to Q4_K; x ~ N(0,1))",
        "aggregate": {"tokens_per_s": round(world * args.steps / (ms * 1e-3), 1),
                      "block_tokens_per_s": round(world * args.steps * L / (ms * 1e-3), 1),
                      "note": "all replicas together; value is the per-GPU time per block and token"},
        "config": {"workload": WORKLOAD, "tokens_per_step": 1, "layers": L, "parallelism": f"replicas{world}",
                   "l2": "inputs larger than L2: ~722 MB of distinct weights touched per step vs 126 MB L2",
                   "launch": f"one CUDA graph per step ({kernels_per_block} kernels per block)"},
        "clocks": clk,
        "e2e": {"value": round(e2e, 4), "unit": UNIT, "h2d_bytes_per_step": 4 * dims.d_model,
                "d2h_bytes_per_step": 4 * dims.d_model,
                "note": "pinned host token in, 40 blocks via the C-ABI (graph replay), result to host, sync per token"},
        "gpu_launches": args.steps * L * kernels_per_block,
        "roofline": {"kernel": "k_experts (fused routing + gate/up + down + combine)", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": EXPERT_BYTES,
                     "avg_launch_us": round(kernel_us, 3),
                     "traffic": EXPERT_TRAFFIC_BYTES,
                     "traffic_source": "imported: ncu capture of k_experts (profiles/k_experts_decode_q4k.md)",
                     "block": {"algorithmic_bytes": BLOCK_BYTES, "us": round(per_block_us, 3),
                               "achieved": round(block_achieved, 1), "frac": round(block_achieved / peak, 4)}},
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        line["parity"] = decode_parity(blocks, inputs, dims, dc, ws, nws, 3)
        line["cpu_baseline"] = cpu_baseline(args)
        line["ref_gpu"] = ref_gpu_baseline(blocks, inputs, dims, steps=4)
    if world == 1 and not args.no_extra:
        line["prefill"] = measure_prefill(blocks[0], dims)
        line["prefill_stack"] = measure_prefill_stack(blocks, dims)
        line["prefill_stack"]["token_by_token_tokens_per_s"] = round(1e6 / (value * L), 1)
        line["config3"] = measure_config3(dims)
        line["gemv"] = measure_gemv(dims)
    if not args.no_extra:
        del blocks, cblocks
        line["ep_prefill"] = measure_ep(world, rank, dims)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


PREFILL_T = 4096
ZIPF_S = 1.1  # expert popularity: Zipf(s) over a seeded ranking of the experts


def measure_prefill(blk, dims):
    """one MoE block over T=4096 tokens (prefill), Q4_K
    experts, router skewed by a seeded per-expert logit bias so expert
    popularity is heavy-tailed; grouped expert GEMMs on the tensor cores.
    Timed with CUDA events over repeated calls (inputs: 32 MB of tokens and
    ~460 MB of weights per call, larger than L2)."""
    import numpy as np
    import torch

    from qmoe import _lib

    from qmoe import synth

    T = PREFILL_T
    dc = dims.c()
    bias, bias_h, _ = _zipf_bias(dims)
    c = blk.c()
    c.expert_bias = bias.data_ptr()
    x = synth.inputs(T, dims.d_model, seed=SEED + 5, tag=4)
    n = _lib.lib().qmoe_workspace_size(ctypes.byref(dc), T)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().qmoe_workspace_init(ws.data_ptr(), n, None))
    out = torch.empty_like(x)

    def run():
        _lib.check(_lib.lib().qmoe_block_forward(ctypes.byref(c), ctypes.byref(dc), x.data_ptr(), out.data_ptr(),
                                                 None, T, ws.data_ptr(), n, None), "prefill block_forward")

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    reps = 10
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    st, flags, _ = _check_errors(_lib, ws, dc)
    E, k = dims.num_experts, dims.top_k
    got = {"logits": _ws_view(_lib, ws, dc, T, _lib.WS_LOGITS, T * (E + 1), np.float32).reshape(T, E + 1)[:, :E],
           "idx": _ws_view(_lib, ws, dc, T, _lib.WS_TOPK_IDX, T * k, np.int32).reshape(T, k),
           "w": _ws_view(_lib, ws, dc, T, _lib.WS_TOPK_W, T * k, np.float32).reshape(T, k),
           "offsets": _ws_view(_lib, ws, dc, T, _lib.WS_OFFSETS, E + 1, np.int32),
           "perm": _ws_view(_lib, ws, dc, T, _lib.WS_PERM, T * k, np.int32),
           "out": out.cpu().numpy()}
    counts = np.diff(got["offsets"])
    parity = _oracle_parity(blk, dims, x.cpu().numpy(), got, bias_h)
    k, F, d = dims.top_k, dims.expert_dim, dims.d_model
    flop = 2.0 * T * k * 3 * F * d + 2.0 * T * 3 * dims.shared_dim * d  # routed + shared expert products
    tflops = flop / (us * 1e-6) / 1e12
    peak = _bf16_peak()
    return {"config": "config4: T=4096 tokens x d=2048, 256 Q4_K experts, top-8, Zipf(1.1)-like routing "
                      "(per-expert logit bias calibrated to a Zipf(%.1f) hit histogram)" % ZIPF_S,
            "us_per_block": round(us, 1), "tokens_per_s": round(T / (us * 1e-6), 0),
            "expert_gflop": round(flop / 1e9, 1),
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak[0], "unit": "TFLOP/s",
                         "frac": round(tflops / peak[0], 4), "peak_kind": peak[1],
                         "note": "whole block (router, top-k, dispatch, GEMMs, combine) against dense bf16 peak"},
            "routing": {"experts_hit": int((counts > 0).sum()), "max_per_expert": int(counts.max()),
                        "mean_per_hit_expert": round(float(counts[counts > 0].mean()), 1)},
            "parity": parity,
            "error_flags": flags}


EP_T = 16384


def _zipf_bias(dims):
    """The calibrated Zipf(1.1) router bias on the device, and the expected
    pairs per token of each expert (the placement's load model)."""
    import torch

    from qmoe import synth
    b, target = synth.zipf_bias(dims.num_experts, dims.top_k, dims.d_model, s=ZIPF_S, seed=SEED + 4)
    return torch.tensor(b, dtype=torch.float32, device="cuda"), b, target


def measure_ep(world, rank, dims):
    """T=16384 tokens of prefill through one Q4_K MoE block,
    uniform and Zipf-skewed routing.  world == 1: the whole block on one GPU
    (qmoe_block_forward).  world > 1: expert parallelism -- E/world experts
    per rank, T/world tokens per rank, NCCL all-to-all of the (token, expert)
    rows and of their outputs (qmoe/ep.py).  Every rank also runs the 1-GPU
    block on all T tokens once and checks that its routing is bit-identical
    and its output equal.  Time: CUDA events around repeated calls, max over
    ranks; tokens/s counts all T tokens (total work fixed: strong scaling)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from qmoe import _lib, ep, synth

    T, d, E, k = EP_T, dims.d_model, dims.num_experts, dims.top_k
    Tl = T // world
    dc = dims.c()
    blk = synth.Block(dims, synth.Q4K_TYPES, seed=SEED + 7, device="cuda")  # the same bytes on every rank
    g = torch.Generator(device="cuda").manual_seed(SEED + 8)
    x_all = torch.randn(T, d, generator=g, device="cuda", dtype=torch.float32)
    x = x_all[rank * Tl:(rank + 1) * Tl].contiguous()
    zipf, zipf_h, zipf_target = _zipf_bias(dims)
    n = _lib.lib().qmoe_workspace_size(ctypes.byref(dc), T)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().qmoe_workspace_init(ws.data_ptr(), n, None))
    out_all = torch.empty_like(x_all)
    flop = 2.0 * T * k * 3 * dims.expert_dim * d + 2.0 * T * 3 * dims.shared_dim * d
    peak = _bf16_peak()
    reps = 10
    res = {"config": f"config5: T={T} tokens x d={d}, {E} Q4_K experts ({E // world} per GPU), top-{k}, "
                     f"{world} GPU(s), one fp16 row per (token, rank) over NCCL all-to-all, outputs back by copy-engine "
                     f"writes into the owning rank's buffer over NVLink (CUDA IPC)" if world > 1 else
                     f"config5 at 1 GPU: T={T} tokens x d={d}, {E} Q4_K experts, top-{k}, one block_forward",
           "n_gpus": world, "scaling": "strong", "routings": {}}
    backends = []
    for routing in ("uniform", "zipf"):
        c = blk.c()
        if routing == "zipf":
            c.expert_bias = zipf.data_ptr()

        def one_gpu():
            _lib.check(_lib.lib().qmoe_block_forward(ctypes.byref(c), ctypes.byref(dc), x_all.data_ptr(),
                                                     out_all.data_ptr(), None, T, ws.data_ptr(), n, None),
                       "block_forward")

        one_gpu()
        torch.cuda.synchronize()
        entry = {}
        bias_h = zipf_h if routing == "zipf" else None
        if world == 1:
            run = one_gpu
            got = {"logits": _ws_view(_lib, ws, dc, T, _lib.WS_LOGITS, T * (E + 1), np.float32).reshape(T, E + 1)[:, :E],
                   "idx": _ws_view(_lib, ws, dc, T, _lib.WS_TOPK_IDX, T * k, np.int32).reshape(T, k),
                   "w": _ws_view(_lib, ws, dc, T, _lib.WS_TOPK_W, T * k, np.float32).reshape(T, k),
                   "offsets": _ws_view(_lib, ws, dc, T, _lib.WS_OFFSETS, E + 1, np.int32),
                   "perm": _ws_view(_lib, ws, dc, T, _lib.WS_PERM, T * k, np.int32),
                   "out": out_all.cpu().numpy()}
            entry["parity"] = _oracle_parity(blk, dims, x_all.cpu().numpy(), got, bias_h, n_spread=48, n_cold=4,
                                             per_cold=2, every_expert=False)
        else:
            p = _lib.lib().qmoe_ws_view(ws.data_ptr(), ctypes.byref(dc), T, _lib.WS_TOPK_IDX)
            off = p - ws.data_ptr()
            want_idx = ws[off:off + T * k * 4].view(torch.int32).view(T, k)[rank * Tl:(rank + 1) * Tl].clone()
            pl = None
            if routing == "zipf":  # experts placed to balance the expected (calibrated) per-rank load
                pl = ep.balanced_placement(zipf_target.tolist(), world)
                lb, ld, keep = ep.local_block_placed(c, dc, ep.experts_of_rank(pl, world, rank))
                entry["placement"] = "balanced by the calibrated Zipf(1.1) expert load"
            else:
                lb, ld = ep.local_block(c, dc, rank, world)
                entry["placement"] = "contiguous"
            be = ep.CudaBackend(c, lb, dc, ld, world, max_tokens=Tl, max_rows=2 * Tl, placement=pl)
            if EP_IMPL == "abi":
                # the C-ABI host layer (include/qmoe_ep.h): exchange and ordering in
                # C++ over the library's own NCCL communicator; `be` only routes
                # once more below to read the top-k ids for the parity check
                abi = _ep_abi_context(dc, Tl, rank, world)
                backends.append(abi)
                pl_dev = be.placement
                got = torch.empty_like(x)

                def fwd_abi():
                    _lib.check(_lib.ep_lib().qmoe_ep_forward(
                        abi.ctx, ctypes.byref(c), ctypes.byref(lb), None if pl_dev is None else pl_dev.data_ptr(),
                        x.data_ptr(), None, 1e-6, None, got.data_ptr(), Tl, None), "ep_forward")
                fwd_abi()
                be.route(x)
                moe = None
                entry["exchange"] = "C-ABI (qmoe_ep_forward, libqmoe_ep.so): NCCL from C++"
            else:
                moe = ep.ExpertParallelMoE(be, E, k, d, direct=True)
                backends.append(be)
                got = moe.forward(x)
                entry["exchange"] = "Python (qmoe/ep.py over torch.distributed)"
            idx = be.topk_idx()
            want = out_all[rank * Tl:(rank + 1) * Tl]
            chk = torch.tensor([0.0 if torch.equal(idx, want_idx) else 1.0, float((got - want).abs().max())],
                               dtype=torch.float64, device="cuda")
            dist.all_reduce(chk, op=dist.ReduceOp.MAX)
            orc_rep = _ep_oracle_parity(blk, dims, x.cpu().numpy(), idx.cpu().numpy(), got.cpu().numpy(), bias_h,
                                        world)
            ok = torch.tensor([orc_rep["max_abs_err"], orc_rep["max_rel_err"], float(orc_rep["n_outside"]),
                               0.0 if orc_rep["ids_bit_exact"] else 1.0], dtype=torch.float64, device="cuda")
            dist.all_reduce(ok, op=dist.ReduceOp.MAX)
            entry["parity"] = {"ids_bit_identical_to_1gpu": chk[0].item() == 0.0, "max_abs_diff_vs_1gpu": chk[1].item(),
                               "oracle": {"ids_bit_exact": ok[3].item() == 0.0, "max_abs_err": ok[0].item(),
                                          "max_rel_err": ok[1].item(), "max_n_outside_per_rank": int(ok[2].item()),
                                          "within_tol": ok[3].item() == 0.0 and ok[2].item() == 0.0,
                                          "sample": "every rank: routing of its T/N tokens, outputs of a sample "
                                                    f"of ~{orc_rep['sample_tokens']} of them"}}

            def run():
                if moe is None:
                    fwd_abi()
                else:
                    moe.forward(x)
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            run()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        if world > 1:
            t = torch.tensor([us], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t[0])
        tflops = flop / (us * 1e-6) / 1e12
        entry.update({"us_per_block": round(us, 1), "tokens_per_s": round(T / (us * 1e-6), 0),
                      "tflops_per_gpu": round(tflops / world, 1),
                      "frac_of_peak_per_gpu": round(tflops / world / peak[0], 4)})
        res["routings"][routing] = entry
    res["peak"] = {"bf16_tflops": peak[0], "kind": peak[1]}
    res["expert_gflop"] = round(flop / 1e9, 1)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        for be in backends:
            be.close()
        dist.barrier()
    return res


EP_IMPL = "abi"


class _EpAbi:
    """A qmoe_ep context (include/qmoe_ep.h) over its own NCCL communicator."""

    def __init__(self, ctx, comm):
        self.ctx, self.comm = ctx, comm

    def close(self):
        from qmoe import _lib
        _lib.check(_lib.ep_lib().qmoe_ep_finalize(self.ctx), "ep_finalize")
        _lib.check(_lib.ep_lib().qmoe_ep_comm_destroy(self.comm), "ep_comm_destroy")


def _ep_abi_context(dc, max_tokens, rank, world):
    """Rank 0 makes the NCCL id, torch.distributed hands it to every rank, each
    rank builds its communicator and an expert-parallel context with the
    peer-memory return."""
    import torch.distributed as dist

    from qmoe import _lib
    L = _lib.ep_lib()
    obj = [None]
    if rank == 0:
        uid = (ctypes.c_uint8 * 128)()
        _lib.check(L.qmoe_ep_unique_id(uid), "ep_unique_id")
        obj[0] = bytes(uid)
    dist.broadcast_object_list(obj, src=0)
    comm, ctx = ctypes.c_void_p(), ctypes.c_void_p()
    _lib.check(L.qmoe_ep_comm_init((ctypes.c_uint8 * 128).from_buffer_copy(obj[0]), world, rank, ctypes.byref(comm)),
               "ep_comm_init")
    _lib.check(L.qmoe_ep_init(comm, ctypes.byref(dc), max_tokens, _lib.QMOE_EP_DIRECT, ctypes.byref(ctx)), "ep_init")
    return _EpAbi(ctx, comm)


def _ep_oracle_parity(blk, dims, x_local, idx_local, out_local, bias_h, world):
    """One rank's share of the expert-parallel parity: its tokens' expert ids
    against the oracle's routing, and the outputs of a sample of them."""
    import numpy as np

    from oracle import oracle as orc
    from qmoe import synth
    orc.set_threads(max(1, (os.cpu_count() or 1) // world))
    _, idx, _ = orc.route(blk.host_bytes("router"), blk.types["router"], x_local, dims.num_experts, dims.top_k,
                          bias_h)
    sample = orc.pick_sample(idx, dims.num_experts, n_spread=16, n_cold=2, per_cold=1, every_expert=False)
    want = orc.moe_forward({n: blk.host_bytes(n) for n in synth.TENSORS}, blk.types, dims, x_local[sample], bias_h)
    rep = orc.tolerance_report(out_local[sample], want["out"])
    rep["ids_bit_exact"] = bool(np.array_equal(idx, idx_local))
    rep["sample_tokens"] = int(sample.size)
    return rep


def measure_config3(dims):
    """mixed-quant decode (gate/up Q4_K, down Q6_K, shared
    Q8_0, per-expert router bias ~N(0,1)) at B = 1, 2, 4, 8 tokens per call,
    through 8 layers (~4 GB of weights, larger than L2)."""
    import numpy as np
    import torch

    from qmoe import _lib, synth

    L = 8
    blocks = [synth.Block(dims, synth.MIXED_TYPES, seed=SEED + 3, layer=l, device="cuda", bias=True) for l in range(L)]
    cbs = [b.c() for b in blocks]
    dc = dims.c()
    res = []
    for B in (1, 2, 4, 8):
        n = _lib.lib().qmoe_workspace_size(ctypes.byref(dc), B)
        ws = torch.empty(n, dtype=torch.uint8, device="cuda")
        _lib.check(_lib.lib().qmoe_workspace_init(ws.data_ptr(), n, None))
        x = synth.inputs(B, dims.d_model, seed=SEED + B, tag=3)
        bufs = [torch.empty_like(x), torch.empty_like(x)]
        gamma = torch.ones(dims.d_model, dtype=torch.float32, device="cuda")

        def step(sp):
            cur = x
            for l in range(L):
                o = bufs[l % 2]
                _lib.check(_lib.lib().qmoe_block_forward_prenorm(ctypes.byref(cbs[l]), ctypes.byref(dc),
                                                                 cur.data_ptr(), gamma.data_ptr(), EPS,
                                                                 o.data_ptr(), B, ws.data_ptr(), n, sp))
                cur = o

        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            for _ in range(3):
                step(s.cuda_stream)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step(torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        reps = 20
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * L)
        st, flags, _ = _check_errors(_lib, ws, dc)
        # distinct experts hit by the B tokens of the last layer's call (its offsets)
        offs = _ws_view(_lib, ws, dc, B, _lib.WS_OFFSETS, dims.num_experts + 1, np.int32)
        U = int((np.diff(offs) > 0).sum())
        nbytes = 2_097_152 + U * 2_039_808 + 3_342_336 + 8_192 + B * 16_384
        gbs = nbytes / (us * 1e-6) / 1e9
        res.append({"B": B, "us_per_block": round(us, 2), "us_per_token_block": round(us / B, 2),
                    "distinct_experts": U, "algorithmic_bytes": nbytes, "achieved_gbs": round(gbs, 1),
                    "frac_of_hbm": round(gbs / _peaks()[0], 4), "error_flags": flags})
        del g
    return {"config": "config3: mixed-quant decode (gate/up Q4_K, down Q6_K, shared Q8_0, router bias N(0,1)), "
                      "8 layers, one CUDA graph per step; bytes = router + U x (Q4_K gate/up + Q6_K down) + "
                      "Q8_0 shared + gate vector + B x (x, out), U = distinct experts hit", "results": res}


LM_HEAD_ROWS = 248_320  # vocabulary rows of the LM head (src/model.cpp:216)


def measure_gemv(dims):
    """The matmul_dispatch path at the LM head's shape (248,320 x 2048,
    src/model.cpp:216): the streaming unit-decode GEMV (qmoe_gemv) and the
    reference-order kernel (qmoe_gemv_exact) for Q4_K, Q6_K and Q8_0 weights,
    HBM roofline on the weight bytes; outputs of a row sample checked against
    the oracle's F32 products."""
    import numpy as np
    import torch

    from oracle import oracle as orc
    from qmoe import _lib
    M, K = LM_HEAD_ROWS, dims.d_model
    out = {"shape": [M, K], "what": "y = W x, one token (LM head of src/model.cpp:216 and the other "
                                    "matmul_dispatch callers)", "types": {}}
    peak = _peaks()
    for ty, name in ((12, "Q4_K"), (14, "Q6_K"), (8, "Q8_0")):
        n = M * K
        nb = _lib.lib().qmoe_tensor_bytes(ty, n)
        w = torch.empty(nb, dtype=torch.uint8, device="cuda")
        _lib.check(_lib.lib().qmoe_synth_fill(w.data_ptr(), ty, n, SEED + 21, ty, 0.02, None))
        x = synth_inputs_1(K)
        t = _lib.QmoeTensor(w.data_ptr(), ty, 0, n)
        ent = {}
        ys = {}
        for impl, fn in (("stream", _lib.lib().qmoe_gemv), ("exact", _lib.lib().qmoe_gemv_exact)):
            y = torch.empty(M, device="cuda")
            for _ in range(3):
                _lib.check(fn(ctypes.byref(t), x.data_ptr(), y.data_ptr(), M, K, 0, None))
            torch.cuda.synchronize()
            reps = 10 if impl == "stream" else 3
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn(ctypes.byref(t), x.data_ptr(), y.data_ptr(), M, K, 0, None)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / reps
            gbs = (nb + 4 * K + 4 * M) / (us * 1e-6) / 1e9
            ent[impl] = {"us": round(us, 1), "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / peak[0], 4)}
            ys[impl] = y
        # parity: 4 blocks of 64 rows against the oracle (F32 products), stream vs exact over all rows
        wh = w.cpu().numpy()
        xh = x.cpu().numpy()
        worst = 0.0
        for r0 in (0, 77_777, 160_000, M - 64):
            want = orc.gemv(wh, ty, n, xh, 64, K, r0 * K)
            worst = max(worst, float(np.max(np.abs(ys["stream"][r0:r0 + 64].cpu().numpy() - want))))
        ent["parity"] = {"stream_vs_oracle_max_abs": worst, "rows_checked": 256,
                         "stream_vs_exact_max_abs_all_rows": float((ys["stream"] - ys["exact"]).abs().max()),
                         "within_1e-5": worst <= 1e-5}
        ent["bytes"] = nb
        ent["speedup_vs_exact"] = round(ent["exact"]["us"] / ent["stream"]["us"], 1)
        if ty == 14:  # the load-time repack into 16-byte-aligned super-blocks (qmoe_repack)
            nr = _lib.lib().qmoe_repack_bytes(ty, n, _lib.QMOE_LAYOUT_Q6K_A16)
            wr = torch.empty(nr, dtype=torch.uint8, device="cuda")
            _lib.check(_lib.lib().qmoe_repack(ctypes.byref(t), _lib.QMOE_LAYOUT_Q6K_A16, wr.data_ptr(), nr, None))
            tr = _lib.QmoeTensor(wr.data_ptr(), ty, _lib.QMOE_LAYOUT_Q6K_A16, n)
            yr = torch.empty(M, device="cuda")
            for _ in range(3):
                _lib.check(_lib.lib().qmoe_gemv(ctypes.byref(tr), x.data_ptr(), yr.data_ptr(), M, K, 0, None))
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                _lib.lib().qmoe_gemv(ctypes.byref(tr), x.data_ptr(), yr.data_ptr(), M, K, 0, None)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / 10
            gbs = (nr + 4 * K + 4 * M) / (us * 1e-6) / 1e9
            ent["repacked_a16"] = {"us": round(us, 1), "bytes": nr, "gbs": round(gbs, 1),
                                   "frac_of_hbm": round(gbs / peak[0], 4),
                                   "bit_identical_to_gguf_layout": bool(torch.equal(yr, ys["stream"]))}
            del wr
        out["types"][name] = ent
        del w
    out["peak"] = {"hbm_gbs": peak[0], "kind": peak[1]}
    return out


def synth_inputs_1(K):
    from qmoe import synth
    return synth.inputs(1, K, seed=SEED + 22, tag=9)[0].contiguous()


def measure_prefill_stack(blocks, dims, T=4096):
    """The batched layer loop (qmoe_stack_forward): T=4096 tokens through the
    MoE halves of all 40 layers of the decode stack (pre-norm and residual
    fused), the multi-token loop the reference does not have -- it feeds a
    prompt token by token (src/main.cpp:391-393), i.e. at the decode rate."""
    import torch

    from qmoe import _lib, synth
    L = len(blocks)
    dc = dims.c()
    n = _lib.lib().qmoe_workspace_size(ctypes.byref(dc), T)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    _lib.check(_lib.lib().qmoe_workspace_init(ws.data_ptr(), n, None))
    x0 = synth.inputs(T, dims.d_model, seed=SEED + 9, tag=11)
    resid, tmp = x0.clone(), torch.empty_like(x0)
    norms = torch.ones(dims.d_model, device="cuda")
    cb = (_lib.QmoeBlock * L)(*[b.c() for b in blocks])
    nptr = (ctypes.c_void_p * L)(*([norms.data_ptr()] * L))

    def run():
        _lib.check(_lib.lib().qmoe_stack_forward(cb, nptr, L, ctypes.byref(dc), EPS, resid.data_ptr(),
                                                 tmp.data_ptr(), T, ws.data_ptr(), n, None), "stack_forward")

    resid.copy_(x0)
    run()
    torch.cuda.synchronize()
    reps = 3
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    st, flags, _ = _check_errors(_lib, ws, dc)
    finite = bool(torch.isfinite(resid).all())
    return {"config": f"T={T} tokens through the MoE halves of {L} layers (qmoe_stack_forward, tensor-core path), "
                      "random-routing Q4_K stack of the decode line",
            "us_per_pass": round(us, 1), "tokens_per_s": round(T / (us * 1e-6), 0),
            "us_per_block": round(us / L, 1), "finite": finite, "error_flags": flags}


def _bf16_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def _check_errors(_lib, ws, dc):
    err = (ctypes.c_uint32 * 2)()
    st = _lib.lib().qmoe_check_errors(ws.data_ptr(), ctypes.byref(dc), err, None)
    return st, int(err[0]), int(err[1])


def _ws_view(_lib, ws, dc, T, which, count, dtype):
    import numpy as np
    p = _lib.lib().qmoe_ws_view(ws.data_ptr(), ctypes.byref(dc), T, which)
    off = p - ws.data_ptr()
    return ws[off:off + count * np.dtype(dtype).itemsize].cpu().numpy().view(dtype)


def _oracle_parity(blk, dims, x_host, got, bias_h, threads=None, **sample_kw):
    """orc.check_batch on the host cores: routing of every token bit-exact,
    outputs of a sample of tokens within tolerance (not timed)."""
    from oracle import oracle as orc
    from qmoe import synth
    orc.set_threads(threads or os.cpu_count() or 1)
    sample = None
    if sample_kw:
        logits, idx, _ = orc.route(blk.host_bytes("router"), blk.types["router"], x_host, dims.num_experts,
                                   dims.top_k, bias_h)
        sample = orc.pick_sample(idx, dims.num_experts, **sample_kw)
    t0 = time.perf_counter()
    res = orc.check_batch({n: blk.host_bytes(n) for n in synth.TENSORS}, blk.types, dims, x_host, got, bias_h,
                          sample=sample)
    res["check_s"] = round(time.perf_counter() - t0, 1)
    return res


def _ws_array(_lib, ws, dc, which, count, dtype):
    import numpy as np
    p = _lib.lib().qmoe_ws_view(ws.data_ptr(), ctypes.byref(dc), 1, which)
    off = p - ws.data_ptr()
    return ws[off:off + count * np.dtype(dtype).itemsize].cpu().numpy().view(dtype)


def cpu_info() -> dict:
    model = None
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"model": model, "nproc": os.cpu_count()}


class CpuStack:
    """The config-2 stack's weights on the host for the CPU legs, generated
    lazily (router and shared expert per layer, a routed expert's three
    matrices when a token first selects it) by the oracle's copy of the host
    generator -- the same bytes the GPU arm generates on the device."""

    def __init__(self):
        import numpy as np

        from qmoe import synth
        from qmoe.quant import calculate_tensor_bytes
        self.np, self.synth = np, synth
        self.dims = synth.Dims()
        self.types = synth.Q4K_TYPES
        self.tb = calculate_tensor_bytes
        self.cache = {}
        self.pool = self._inputs()

    def _inputs(self):
        from oracle import oracle as orc
        d = self.dims.d_model
        b = self.np.empty(POOL * d * 4, dtype=self.np.uint8)
        orc.synth_fill(b, 0, 0, POOL * d, SEED, self.synth.input_stream_id(2), 1.0)
        return b.view(self.np.float32).reshape(POOL, d)

    def _fill(self, name, layer, first, n, dst):
        from oracle import oracle as orc
        sid = self.synth.stream_id(layer, self.synth.TENSORS.index(name) + 1)
        orc.synth_fill(dst, int(self.types[name]), first, n, SEED, sid, self.synth.WEIGHT_SIGMA)

    def layer(self, layer):
        if layer not in self.cache:
            t = {}
            for n in self.synth.TENSORS:
                t[n] = self.np.zeros(self.tb(self.types[n], self.dims.elements(n)), dtype=self.np.uint8)
            for n in ("router", "shared_gate_inp", "shared_gate", "shared_up", "shared_down"):
                self._fill(n, layer, 0, self.dims.elements(n), t[n])
            self.cache[layer] = (t, set())
            if len(self.cache) > 4:
                self.cache.pop(next(iter(self.cache)))
        return self.cache[layer]

    def prepare(self, step):
        """Weights of block (step mod 40) with the experts its token selects, and the token."""
        from oracle import oracle as orc
        d, E, k, F = self.dims.d_model, self.dims.num_experts, self.dims.top_k, self.dims.expert_dim
        layer = step % N_LAYERS
        x = self.pool[(step // N_LAYERS) % POOL]
        t, have = self.layer(layer)
        logits = orc.gemv(t["router"], 0, E * d, x, E, d)
        ids, _ = orc.topk(logits, k)
        bpe = self.tb(self.types["gate_exps"], F * d)
        for e in ids.tolist():
            if e not in have:
                for n in ("gate_exps", "up_exps", "down_exps"):
                    self._fill(n, layer, e * F * d, F * d, t[n][e * bpe:(e + 1) * bpe])
                have.add(e)
        return t, x

    def time_blocks(self, steps, warmup, threads):
        """Microseconds per block and token of the oracle on `threads` host threads."""
        from oracle import oracle as orc
        orc.set_threads(threads)
        for i in range(warmup):
            t, x = self.prepare(i)
            orc.moe_forward(t, self.types, self.dims, x)
        secs = 0.0
        for i in range(steps):
            t, x = self.prepare(warmup + i)
            t0 = time.perf_counter()
            res = orc.moe_forward(t, self.types, self.dims, x)
            secs += time.perf_counter() - t0
            assert res["status"][0] == 0
        return secs / steps * 1e6


def cpu_baseline(args):
    """The oracle (C restatement of the reference MoE path) on the host cores
    over a bounded sample: all host threads and one thread."""
    threads = os.cpu_count() or 1
    st = CpuStack()
    n_all, n_one = max(4, args.cpu_layers), 2
    v_all = st.time_blocks(n_all, 2, threads)
    v_one = st.time_blocks(n_one, 1, 1)
    sample = (f"{n_all} MoE blocks x 1 token after 2 warm-up blocks (layer = step mod 40 of the config-2 stack), "
              "oracle/qmoe_oracle.c, OpenMP over output rows")
    return {"value": round(v_all, 1), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
            "single_thread": {"value": round(v_one, 1), "unit": UNIT, "cores": 1,
                              "sample": f"{n_one} MoE blocks x 1 token after 1 warm-up block"},
            "cpu": cpu_info()}


def decode_parity(blocks, inputs, dims, dc, ws, nws, n_blocks):
    """The product's decode output of the first n_blocks layers of the stack
    (one token, the residual stream as in the timed run) against the oracle:
    expert ids bit-exact, outputs within max-abs 1e-3 / rel 1e-2."""
    import numpy as np
    import torch

    from oracle import oracle as orc
    from qmoe import _lib, synth

    orc.set_threads(os.cpu_count() or 1)
    x = inputs[0:1].clone()
    out = torch.empty_like(x)
    ids_ok, max_abs, max_rel, within = True, 0.0, 0.0, True
    gamma = torch.ones(dims.d_model, dtype=torch.float32, device="cuda")
    for l in range(n_blocks):
        c = blocks[l].c()
        _lib.check(_lib.lib().qmoe_block_forward_prenorm(ctypes.byref(c), ctypes.byref(dc), x.data_ptr(),
                                                         gamma.data_ptr(), EPS, out.data_ptr(), 1, ws.data_ptr(),
                                                         nws, None))
        torch.cuda.synchronize()
        gid = _ws_array(_lib, ws, dc, _lib.WS_TOPK_IDX, dims.top_k, np.int32)
        xin = _ws_array(_lib, ws, dc, _lib.WS_INPUT, dims.d_model, np.float32)  # rmsnorm(r) as the block saw it
        res = orc.moe_forward({n: blocks[l].host_bytes(n) for n in synth.TENSORS}, blocks[l].types, dims, xin)
        rep = orc.tolerance_report(out.cpu().numpy(), x.cpu().numpy() + res["out"])
        ids_ok &= bool(np.array_equal(gid, res["idx"][0]))
        max_abs, max_rel = max(max_abs, rep["max_abs_err"]), max(max_rel, rep["max_rel_err"])
        within &= rep["within_tol"]
        x = out.clone()  # the residual stream, as in the timed run
    return {"blocks": n_blocks, "ids_bit_exact": ids_ok, "max_abs_err": max_abs, "max_rel_err": max_rel,
            "within_tol": within and ids_ok, "tol": "per element |err| <= 1e-3 or |err|/|want| <= 1e-2"}


def ref_gpu_baseline(blocks, inputs, dims, steps):
    """The reference's own GPU path (oracle/_ref: MoeLayer::forward and its
    kernels compiled unmodified for sm_100a, with rmsnorm_forward and
    residual_add around it as model.cpp:207-211 runs them) over the same 40
    layers of weights, one token at a time, CUDA events around the steps.
    MoeLayer::forward synchronises the stream inside every call, as shipped."""
    import torch

    from oracle import oracle as orc
    if not orc.ref_available():
        return {"unavailable": "oracle/_ref/libqwenref.so not built (the reference tree was absent at build time)"}
    from qmoe import synth
    L = orc.ref_lib()
    L.ref_stack_create.restype = ctypes.c_void_p
    L.ref_stack_create.argtypes = [ctypes.c_int] * 6 + [ctypes.c_void_p] * 3
    L.ref_stack_forward.restype = ctypes.c_int
    L.ref_stack_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float,
                                    ctypes.c_void_p]
    L.ref_stack_destroy.argtypes = [ctypes.c_void_p]
    nl = len(blocks)
    ptrs = (ctypes.c_void_p * (8 * nl))(*[b.t[n].device_ptr for b in blocks for n in synth.TENSORS])
    tys = (ctypes.c_int * (8 * nl))(*[int(b.types[n]) for b in blocks for n in synth.TENSORS])
    nel = (ctypes.c_uint64 * (8 * nl))(*[dims.elements(n) for b in blocks for n in synth.TENSORS])
    h = L.ref_stack_create(nl, dims.d_model, dims.num_experts, dims.top_k, dims.expert_dim, dims.shared_dim,
                           ptrs, tys, nel)
    if not h:
        return {"unavailable": "reference stack set-up failed: " + L.ref_last_error().decode()}
    gamma = torch.ones(dims.d_model, dtype=torch.float32, device="cuda")
    x = inputs[0:1].clone()
    s = torch.cuda.current_stream().cuda_stream
    try:
        for i in range(3):
            x.copy_(inputs[i:i + 1])
            if L.ref_stack_forward(h, x.data_ptr(), gamma.data_ptr(), EPS, s):
                raise RuntimeError(L.ref_last_error().decode())
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            x.copy_(inputs[i % POOL:i % POOL + 1])
            if L.ref_stack_forward(h, x.data_ptr(), gamma.data_ptr(), EPS, s):
                raise RuntimeError(L.ref_last_error().decode())
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
    finally:
        L.ref_stack_destroy(h)
    return {"us_per_block": round(ms * 1e3 / (steps * nl), 2), "ms_per_step": round(ms / steps, 4),
            "steps": steps, "layers": nl,
            "what": "reference MoeLayer::forward (+ rmsnorm_forward, residual_add) built from the reference sources "
                    "for sm_100a (oracle/_ref), same weights and tokens, one token per step"}


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU path (oracle port), rank 0 only
# ---------------------------------------------------------------------------
def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    value = CpuStack().time_blocks(args.steps, args.warmup, threads)
    sample = (f"{args.steps} MoE blocks x 1 token after {args.warmup} warm-up blocks (layer = step mod 40) of the "
              "config-2 stack; only the routed experts' bytes are generated; oracle/qmoe_oracle.c, OpenMP over "
              "output rows")
    line = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value / 1e3, 3),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": WORKLOAD, "tokens_per_step": 1, "layers": 1,
                                           "parallelism": "cpu"},
            "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample, "cpu": cpu_info()},
            "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=N_LAYERS)
    ap.add_argument("--cpu-layers", type=int, default=3)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the prefill (config 4) and mixed decode (config 3) lines")
    ap.add_argument("--only", choices=["prefill", "config3", "ep", "gemv"],
                    help="run one extra measurement alone and print its object (profiling runs)")
    ap.add_argument("--ep-impl", choices=["abi", "python"], default="abi",
                    help="expert-parallel exchange at N > 1: the C-ABI host layer (default) or qmoe/ep.py")
    args = ap.parse_args()
    global EP_IMPL
    EP_IMPL = args.ep_impl
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.only:
        run_only(args.only)
    else:
        run_ours(args)


def run_only(what):
    import datetime

    import torch
    import torch.distributed as dist

    from qmoe import synth

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    dims = synth.Dims()
    if what == "prefill":
        res = measure_prefill(synth.Block(dims, synth.Q4K_TYPES, seed=SEED, layer=0, device="cuda"), dims)
    elif what == "config3":
        res = measure_config3(dims)
    elif what == "gemv":
        res = measure_gemv(dims)
    else:
        res = measure_ep(world, rank, dims)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({what: res}), flush=True)


if __name__ == "__main__":
    main()
