"""Python mirror of the reference's MoeLayer (include/layer_moe.hpp:10-56,
src/layer_moe.cpp) over the C-ABI, for T >= 1 tokens per call.

Differences from the reference, by design:
  * no host round trip per layer: routing is checked on the device and the
    error word is read at the caller's sync point (``check_errors``), or right
    away with ``strict=True`` (the reference's behaviour, src/layer_moe.cpp:106);
  * one workspace per layer instead of eleven single-token buffers.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _lib
from .quant import QuantTensor


@dataclass
class ModelConfig:
    """MoE fields of the reference ModelConfig (include/config.hpp:33-37, 51-54)."""
    d_model: int = 2048
    num_experts: int = 256
    num_experts_per_tok: int = 8
    moe_intermediate_dim: int = 512
    shared_expert_dim: int = 512

    def validate(self) -> None:  # include/config.hpp:104-110
        if self.moe_intermediate_dim <= 0 or self.shared_expert_dim <= 0:
            raise RuntimeError("invalid MoE dimensions")
        if self.num_experts <= 0 or self.num_experts_per_tok <= 0 or self.num_experts_per_tok > self.num_experts:
            raise RuntimeError("invalid MoE routing configuration")

    def dims(self) -> _lib.QmoeDims:
        return _lib.QmoeDims(self.d_model, self.num_experts, self.num_experts_per_tok, self.moe_intermediate_dim,
                             self.shared_expert_dim)


def _ptr(a):
    if a is None:
        return None
    return a if isinstance(a, int) else a.data_ptr()


def _stream(stream):
    if stream is None:
        return None
    return stream if isinstance(stream, int) else stream.cuda_stream


def _tv(t: QuantTensor) -> _lib.QmoeTensor:
    return _lib.QmoeTensor(t.device_ptr or None, int(t.type), 0, int(t.num_elements))


class MoeLayer:
    def __init__(self):
        self.cfg = None
        self.layer_idx = -1
        self.ws = None
        self.ws_bytes = 0
        self.strict = False

    def init(self, cfg: ModelConfig, layer_idx: int, max_tokens: int = 8, device: str = "cuda",
             strict: bool = False) -> None:
        import torch
        self.free_buffers()
        cfg.validate()
        self.cfg, self.layer_idx, self.strict = cfg, layer_idx, strict
        dims = cfg.dims()
        n = _lib.lib().qmoe_workspace_size(ctypes.byref(dims), max_tokens)
        if n == 0:
            raise RuntimeError("MoE dimensions not supported by the qmoe kernels")
        self.ws = torch.empty(n, dtype=torch.uint8, device=device)
        self.ws_bytes = n
        _lib.check(_lib.lib().qmoe_workspace_init(self.ws.data_ptr(), n, None), "workspace_init")
        torch.cuda.synchronize()

    def free_buffers(self) -> None:
        self.ws = None
        self.ws_bytes = 0

    def block(self, router, eg, eu, ed, sgate, sg, su, sd, bias=None) -> _lib.QmoeBlock:
        return _lib.QmoeBlock(_tv(router), _tv(eg), _tv(eu), _tv(ed), _tv(sgate), _tv(sg), _tv(su), _tv(sd),
                              _ptr(bias))

    def forward(self, x, out, router, eg, eu, ed, sgate, sg, su, sd, stream=None, n_tokens: int = 1,
                residual=None, bias=None) -> None:
        """x/out: device F32 [n_tokens][d_model] (torch tensors or int addresses)."""
        blk = self.block(router, eg, eu, ed, sgate, sg, su, sd, bias)
        dims = self.cfg.dims()
        st = _lib.lib().qmoe_block_forward(ctypes.byref(blk), ctypes.byref(dims), _ptr(x), _ptr(out), _ptr(residual),
                                           n_tokens, self.ws.data_ptr(), self.ws_bytes, _stream(stream))
        _lib.check(st, f"MoE layer {self.layer_idx}")
        if self.strict:
            self.check_errors(stream)

    def check_errors(self, stream=None) -> None:
        """Synchronises the stream and raises the reference's routing errors."""
        err = (ctypes.c_uint32 * 2)()
        dims = self.cfg.dims()
        st = _lib.lib().qmoe_check_errors(self.ws.data_ptr(), ctypes.byref(dims), err, _stream(stream))
        if st == _lib.QMOE_ERR_ROUTING:
            raise RuntimeError(f"invalid/non-finite MoE routing result in layer {self.layer_idx}")
        if st == _lib.QMOE_ERR_NOT_NORMALIZED:
            raise RuntimeError(f"MoE routing weights are not normalized in layer {self.layer_idx}")
        _lib.check(st, f"MoE layer {self.layer_idx}")

    def view(self, which: int, n_tokens: int = 1) -> int:
        dims = self.cfg.dims()
        return _lib.lib().qmoe_ws_view(self.ws.data_ptr(), ctypes.byref(dims), n_tokens, which)
