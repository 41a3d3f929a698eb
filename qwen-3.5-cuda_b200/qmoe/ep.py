"""Expert-parallel MoE block for prefill: the E experts
are sharded contiguously across the G ranks of a process group (E/G per
rank, one GPU per rank), tokens are split across ranks, and the (token,
expert) pairs travel to the rank that owns the expert and back.

Per rank and call (T local tokens):
  1. route    x_in, its fp16 copy and the top-k of every local token
              (qmoe_ep_route: bit-identical routing to the 1-GPU path, since
              the router and top-k are per-token functions)
  2. send     pairs grouped by destination rank (stable: pair order within a
              rank), one fp16 row of x_in per pair plus the expert id local to
              the destination; counts, rows and ids with all-to-all
  3. experts  the rank's experts on the received rows (qmoe_ep_experts,
              tcgen05 grouped GEMMs)
  4. return   outputs back with the reverse all-to-all, placed at their pair
              index t*k + j
  5. combine  shared expert and the slot-ordered combine of the local tokens
              (qmoe_ep_combine)
The exchange runs on torch.distributed (NCCL on GPUs, gloo in the CPU
tests); the compute goes through a backend object, `CudaBackend` in
production, so the exchange logic can be tested without a GPU.
"""
from __future__ import annotations

import ctypes

from . import _lib


def shard_bounds(E: int, world: int, rank: int) -> tuple[int, int]:
    """Experts [lo, hi) owned by `rank` (contiguous, E divisible by world)."""
    if E % world:
        raise ValueError(f"{E} experts cannot be split evenly over {world} ranks")
    n = E // world
    return rank * n, (rank + 1) * n


def plan_sends(idx, E: int, world: int):
    """Pairs of a [T, k] top-k result grouped by destination rank.

    Returns (pairs, dest_eid, counts): pair ids p = t*k + j in (destination,
    p) order for the valid pairs (expert >= 0), the expert id local to each
    pair's destination, and the number of pairs per destination."""
    import torch
    T, k = idx.shape
    n_loc = E // world
    flat = idx.reshape(-1).to(torch.int64)
    valid = flat >= 0
    dest = torch.where(valid, flat // n_loc, torch.full_like(flat, world))
    # stable sort by destination keeps the pair order inside each destination
    key = dest * (T * k) + torch.arange(T * k, device=idx.device)
    order = torch.argsort(key)
    n_valid = int(valid.sum())
    pairs = order[:n_valid]
    dest_eid = (flat[pairs] - dest[pairs] * n_loc).to(torch.int32)
    counts = torch.bincount(dest[pairs], minlength=world)[:world]
    return pairs, dest_eid, counts


class ExpertParallelMoE:
    """One MoE layer sharded over the ranks of `group` (torch.distributed)."""

    def __init__(self, backend, E: int, k: int, d: int, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.backend = backend
        self.E, self.k, self.d = E, k, d
        self.lo, self.hi = shard_bounds(E, self.world, self.rank)

    def _a2a(self, send, send_counts, recv_counts):
        import torch
        recv = torch.empty((int(sum(recv_counts)),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        self.dist.all_to_all_single(recv, send.contiguous(), [int(c) for c in recv_counts],
                                    [int(c) for c in send_counts], group=self.group)
        return recv

    def forward(self, x, residual=None):
        """x: [T, d] local tokens.  Returns out [T, d] (float32)."""
        import torch
        T = x.shape[0]
        idx, rows = self.backend.route(x)                     # [T, k] int32, [T, d] row payload
        pairs, dest_eid, counts = plan_sends(idx, self.E, self.world)
        recv_counts = torch.empty_like(counts)
        self.dist.all_to_all_single(recv_counts, counts, group=self.group)
        sc, rc = counts.tolist(), recv_counts.tolist()
        send_rows = rows.index_select(0, pairs // self.k)
        recv_rows = self._a2a(send_rows, sc, rc)
        recv_eid = self._a2a(dest_eid, sc, rc)
        y_recv = self.backend.experts(recv_rows, recv_eid)    # [n_recv, d]
        y_back = self._a2a(y_recv, rc, sc)
        y_pairs = torch.zeros((T * self.k, self.d), dtype=y_back.dtype, device=y_back.device)
        y_pairs.index_copy_(0, pairs, y_back)
        return self.backend.combine(y_pairs, residual)


class CudaBackend:
    """The qmoe C-ABI on one GPU: the full layer's router and shared expert,
    this rank's slice of the expert tensors."""

    def __init__(self, blk, local_blk, dims, local_dims, max_tokens: int, max_rows: int, norm_weight=None,
                 eps: float = 1e-6):
        import torch
        self.blk, self.local_blk = blk, local_blk
        self.dims, self.local_dims = dims, local_dims
        self.norm_weight, self.eps = norm_weight, eps
        L = _lib.lib()
        self.ws_bytes = L.qmoe_workspace_size(ctypes.byref(dims), max_tokens)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device="cuda")
        _lib.check(L.qmoe_workspace_init(self.ws.data_ptr(), self.ws_bytes, None))
        self._rows_ws(max_rows)
        self.T = 0

    def _rows_ws(self, rows: int) -> None:
        import torch
        self.max_rows = rows
        self.rws_bytes = _lib.lib().qmoe_ep_rows_workspace_size(ctypes.byref(self.local_dims), rows)
        if not self.rws_bytes:
            raise ValueError("qmoe_ep_rows_workspace_size: bad local dims")
        self.rws = torch.empty(self.rws_bytes, dtype=torch.uint8, device="cuda")

    def _view(self, which, count, dtype):
        import torch
        p = _lib.lib().qmoe_ws_view(self.ws.data_ptr(), ctypes.byref(self.dims), self.T, which)
        off = p - self.ws.data_ptr()
        nbytes = count * torch.empty((), dtype=dtype).element_size()
        return self.ws[off:off + nbytes].view(dtype)

    def route(self, x):
        import torch
        self.T = T = x.shape[0]
        self.x = x
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(_lib.lib().qmoe_ep_route(
            ctypes.byref(self.blk), ctypes.byref(self.dims), x.data_ptr(),
            None if self.norm_weight is None else self.norm_weight.data_ptr(), self.eps, T,
            self.ws.data_ptr(), self.ws_bytes, stream), "ep_route")
        k, d = self.dims.top_k, self.dims.d_model
        idx = self._view(_lib.WS_TOPK_IDX, T * k, torch.int32).view(T, k)
        rows = self._view(_lib.WS_INPUT16, T * d, torch.float16).view(T, d)
        return idx, rows

    def experts(self, rows, eid):
        import torch
        n = rows.shape[0]
        y = torch.empty_like(rows)
        if n:
            if n > self.max_rows:  # a rank received more rows than planned: grow its row workspace
                self._rows_ws(n)
            stream = torch.cuda.current_stream().cuda_stream
            _lib.check(_lib.lib().qmoe_ep_experts(
                ctypes.byref(self.local_blk), ctypes.byref(self.local_dims), rows.data_ptr(), eid.data_ptr(), n,
                y.data_ptr(), self.rws.data_ptr(), self.rws_bytes, stream), "ep_experts")
        return y

    def combine(self, y_pairs, residual=None):
        import torch
        out = torch.empty((self.T, self.dims.d_model), dtype=torch.float32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(_lib.lib().qmoe_ep_combine(
            ctypes.byref(self.blk), ctypes.byref(self.dims), y_pairs.data_ptr(), self.T,
            None if residual is None else residual.data_ptr(), out.data_ptr(), self.ws.data_ptr(), self.ws_bytes,
            stream), "ep_combine")
        return out


def local_block(blk: "_lib.QmoeBlock", dims, rank: int, world: int) -> tuple["_lib.QmoeBlock", "_lib.QmoeDims"]:
    """Views of the rank's expert slice of a full layer (pointer offsets into
    the [E][rows][K] GGUF tensors)."""
    from .quant import calculate_tensor_bytes
    lo, hi = shard_bounds(dims.num_experts, world, rank)
    n = hi - lo
    d, F = dims.d_model, dims.expert_dim

    def sl(t, rows, K):
        per_expert = calculate_tensor_bytes(t.ggml_type, rows * K)
        return _lib.QmoeTensor((t.data or 0) + lo * per_expert, t.ggml_type, 0, n * rows * K)

    lb = _lib.QmoeBlock(blk.router, sl(blk.gate_exps, F, d), sl(blk.up_exps, F, d), sl(blk.down_exps, d, F),
                        blk.shared_gate_inp, blk.shared_gate, blk.shared_up, blk.shared_down, None)
    ld = _lib.QmoeDims(d, n, dims.top_k, F, dims.shared_dim)
    return lb, ld
