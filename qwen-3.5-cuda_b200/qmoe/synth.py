"""Seeded synthetic MoE blocks in GGUF layouts (tests and benchmarks).

Every tensor is sigma*N(0,1) from its own counter-based stream and encoded
with the GGML block type requested.  ``device="cuda"`` generates on the GPU,
``device="cpu"`` on the host; both produce the same bytes, so the CPU oracle
can be fed exactly what the kernels read.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _lib
from .quant import GgmlType, QuantTensor, calculate_tensor_bytes

TENSORS = ["router", "gate_exps", "up_exps", "down_exps", "shared_gate_inp", "shared_gate", "shared_up",
           "shared_down"]
GGUF_NAMES = {"router": "ffn_gate_inp.weight", "gate_exps": "ffn_gate_exps.weight", "up_exps": "ffn_up_exps.weight",
              "down_exps": "ffn_down_exps.weight", "shared_gate_inp": "ffn_gate_inp_shexp.weight",
              "shared_gate": "ffn_gate_shexp.weight", "shared_up": "ffn_up_shexp.weight",
              "shared_down": "ffn_down_shexp.weight"}

# the configurations of the benchmark (BASELINE configs 1/2/4/5 and config 3)
Q4K_TYPES = {"router": GgmlType.F32, "gate_exps": GgmlType.Q4_K, "up_exps": GgmlType.Q4_K,
             "down_exps": GgmlType.Q4_K, "shared_gate_inp": GgmlType.F32, "shared_gate": GgmlType.Q4_K,
             "shared_up": GgmlType.Q4_K, "shared_down": GgmlType.Q4_K}
MIXED_TYPES = {"router": GgmlType.F32, "gate_exps": GgmlType.Q4_K, "up_exps": GgmlType.Q4_K,
               "down_exps": GgmlType.Q6_K, "shared_gate_inp": GgmlType.F32, "shared_gate": GgmlType.Q8_0,
               "shared_up": GgmlType.Q8_0, "shared_down": GgmlType.Q8_0}

WEIGHT_SIGMA = 0.02


@dataclass
class Dims:
    d_model: int = 2048
    num_experts: int = 256
    top_k: int = 8
    expert_dim: int = 512
    shared_dim: int = 512

    def c(self) -> _lib.QmoeDims:
        return _lib.QmoeDims(self.d_model, self.num_experts, self.top_k, self.expert_dim, self.shared_dim)

    def elements(self, name: str) -> int:
        d, E, F, Fs = self.d_model, self.num_experts, self.expert_dim, self.shared_dim
        return {"router": E * d, "gate_exps": E * F * d, "up_exps": E * F * d, "down_exps": E * d * F,
                "shared_gate_inp": d, "shared_gate": Fs * d, "shared_up": Fs * d, "shared_down": d * Fs}[name]

    def shape(self, name: str) -> list:
        d, E, F, Fs = self.d_model, self.num_experts, self.expert_dim, self.shared_dim
        return {"router": [d, E], "gate_exps": [d, F, E], "up_exps": [d, F, E], "down_exps": [F, d, E],
                "shared_gate_inp": [d], "shared_gate": [d, Fs], "shared_up": [d, Fs],
                "shared_down": [Fs, d]}[name]


def stream_id(layer: int, idx: int) -> int:
    return (layer << 8) | idx


def input_stream_id(tag: int, layer: int = 0) -> int:
    return (1 << 40) | (tag << 20) | layer


def fill(buf, ggml_type: int, n: int, seed: int, sid: int, sigma: float, stream=None) -> None:
    """Fill a torch CUDA uint8 tensor or a numpy uint8 array."""
    if isinstance(buf, np.ndarray):
        _lib.check(_lib.lib().qmoe_synth_fill_host(buf.ctypes.data, int(ggml_type), n, seed, sid, sigma),
                   "synth_fill_host")
    else:
        s = None if stream is None else stream.cuda_stream
        _lib.check(_lib.lib().qmoe_synth_fill(buf.data_ptr(), int(ggml_type), n, seed, sid, sigma, s), "synth_fill")


class Block:
    """The eight tensors of one MoE layer (+ optional expert bias)."""

    def __init__(self, dims: Dims, types: dict | None = None, seed: int = 1234, layer: int = 0,
                 device: str = "cuda", bias: bool = False):
        self.dims, self.types, self.seed, self.layer, self.device = dims, dict(types or Q4K_TYPES), seed, layer, device
        self.buf, self.t = {}, {}
        for i, name in enumerate(TENSORS):
            n = dims.elements(name)
            ty = self.types[name]
            nb = calculate_tensor_bytes(ty, n)
            if device == "cpu":
                b = np.empty(nb, dtype=np.uint8)
                ptr = b.ctypes.data
            else:
                import torch
                b = torch.empty(nb, dtype=torch.uint8, device=device)
                ptr = b.data_ptr()
            fill(b, ty, n, seed, stream_id(layer, i + 1), WEIGHT_SIGMA)
            self.buf[name] = b
            self.t[name] = QuantTensor(f"blk.{layer}.{GGUF_NAMES[name]}", ty, dims.shape(name), n, nb, 0, ptr, b)
        self.bias = None
        if bias:
            E = dims.num_experts
            if device == "cpu":
                self.bias = np.empty(E * 4, dtype=np.uint8)
            else:
                import torch
                self.bias = torch.empty(E * 4, dtype=torch.uint8, device=device)
            fill(self.bias, GgmlType.F32, E, seed, stream_id(layer, 9), 1.0)

    def c(self) -> _lib.QmoeBlock:
        def v(name):
            q = self.t[name]
            return _lib.QmoeTensor(q.device_ptr, int(q.type), 0, q.num_elements)
        bp = None
        if self.bias is not None:
            bp = self.bias.ctypes.data if isinstance(self.bias, np.ndarray) else self.bias.data_ptr()
        return _lib.QmoeBlock(*(v(n) for n in TENSORS), bp)

    def host_bytes(self, name: str) -> np.ndarray:
        b = self.buf[name]
        return b if isinstance(b, np.ndarray) else b.cpu().numpy()

    def host_bias(self) -> np.ndarray | None:
        if self.bias is None:
            return None
        b = self.bias if isinstance(self.bias, np.ndarray) else self.bias.cpu().numpy()
        return b.view(np.float32)


def inputs(n_tokens: int, d: int, seed: int, tag: int = 0, device: str = "cuda"):
    """x ~ N(0,1) F32 [n_tokens][d] (torch tensor on `device`, or numpy for "cpu")."""
    n = n_tokens * d
    if device == "cpu":
        b = np.empty(n * 4, dtype=np.uint8)
        fill(b, GgmlType.F32, n, seed, input_stream_id(tag), 1.0)
        return b.view(np.float32).reshape(n_tokens, d)
    import torch
    b = torch.empty(n * 4, dtype=torch.uint8, device=device)
    fill(b, GgmlType.F32, n, seed, input_stream_id(tag), 1.0)
    return b.view(torch.float32).view(n_tokens, d)


def zipf_bias(E: int, k: int, d: int, s: float = 1.1, seed: int = 1238, sigma: float = WEIGHT_SIGMA,
              sample: int = 4096, iters: int = 60):
    """Per-expert router logit bias under which the expert hit histogram
    follows Zipf(s) (benchmark configs 4 and 5): the expert of popularity rank
    r (a seeded permutation) gets a share proportional to r^-s of the T*k
    pairs, capped at one pair per token (the capped head's overflow spread
    over the rest).  Calibrated on a seeded sample of the benchmark's input
    distribution (x ~ N(0,1), router rows ~ N(0, sigma^2)) by a damped
    fixed-point iteration on log(target count) - log(sample count).
    Deterministic; about a second of host time.  Returns (bias F32[E],
    expected pairs per token of each expert)."""
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((E, d)) * sigma).astype(np.float32)
    X = rng.standard_normal((sample, d)).astype(np.float32)
    logits = X @ W.T
    ranks = rng.permutation(E) + 1
    z = np.arange(1, E + 1, dtype=np.float64) ** -s
    z = z / z.sum() * sample * k
    for _ in range(64):
        over = np.clip(z - sample, 0, None).sum()
        z = np.minimum(z, sample)
        free = z < sample
        if over <= 0 or not free.any():
            break
        z[free] += over * z[free] / z[free].sum()
    target = np.minimum(z[ranks - 1], sample - 0.5)
    b = -s * np.log(ranks) * 0.5
    for _ in range(iters):
        idx = np.argpartition(-(logits + b[None, :]), k, axis=1)[:, :k]
        cnt = np.bincount(idx.ravel(), minlength=E).astype(np.float64)
        b += 0.5 * (np.log(target) - np.log(np.maximum(cnt, 0.5)))
        b -= b.max()
    return b.astype(np.float32), target / sample
