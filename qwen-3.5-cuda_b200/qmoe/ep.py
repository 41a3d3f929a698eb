"""Expert-parallel MoE block for prefill: the E experts
are sharded contiguously across the G ranks of a process group (E/G per
rank, one GPU per rank), tokens are split across ranks, and each token's row
travels once to every rank that owns one of its experts; the expert outputs
of its (token, slot) pairs travel back.

Per rank and call (T local tokens):
  1. route     x_in, its fp16 copy and the top-k of every local token
               (qmoe_ep_route: the same kernels as the 1-GPU path, so the
               routing is bit-identical to it -- router and top-k are
               per-token functions)
  2. dispatch  send buffers on the device (qmoe_ep_dispatch): one fp16 row
               per (token, rank) with a meta row of local expert ids per slot,
               grouped by rank; rows and pairs per rank; pair_pos, the place
               of every (token, slot) output in the returned buffer
  3. exchange  the per-rank counts (all-to-all, then the one host
               synchronisation of the call: NCCL needs the split sizes), then
               rows and meta rows (all-to-all with those splits; with
               direct=True copy-engine writes into the peers' receive buffers
               and one barrier)
  4. experts   the rank's experts on the received rows (qmoe_ep_experts,
               tcgen05 grouped GEMMs), outputs in (row, slot) order
  5. return    outputs back with the reverse all-to-all -- or, with
               direct=True, over peer memory (CUDA IPC mappings): the down
               GEMM's epilogue stores this rank's own pairs straight into its
               return buffer and the other ranks' pairs contiguously into a
               local staging buffer (qmoe_ep_experts_return), the copy
               engines push each staged chunk into its owner's return buffer
               (one cudaMemcpyAsync per peer), and a one-element all-reduce
               orders those writes before the combine
  6. combine   shared expert and the slot-ordered combine of the local tokens
               through pair_pos (qmoe_ep_combine)
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


PUSH_ROWS_MAX_RANKS = 2


class PeerMemoryUnavailable(RuntimeError):
    """Raised on every rank alike when some rank could not allocate or map
    the peer buffers of the direct return."""


def balanced_placement(load, world: int) -> list:
    """A placement of the experts on `world` ranks (E/world each) that evens
    out the expected per-rank load: experts by decreasing load, each to the
    least-loaded rank with room (greedy LPT).  Returns placement[e] = the
    expert's slot r*(E/world) + local id."""
    E = len(load)
    n = E // world
    if E % world:
        raise ValueError(f"{E} experts cannot be split evenly over {world} ranks")
    order = sorted(range(E), key=lambda e: (-float(load[e]), e))
    rank_load, used = [0.0] * world, [0] * world
    placement = [0] * E
    for e in order:
        r = min((q for q in range(world) if used[q] < n), key=lambda q: (rank_load[q], q))
        placement[e] = r * n + used[r]
        used[r] += 1
        rank_load[r] += float(load[e])
    return placement


def experts_of_rank(placement, world: int, rank: int) -> list:
    """Global ids of the experts placed on `rank`, in local-id order."""
    n = len(placement) // world
    out = [0] * n
    for e, slot in enumerate(placement):
        if slot // n == rank:
            out[slot - rank * n] = e
    return out


class ExpertParallelMoE:
    """One MoE layer sharded over the ranks of `group` (torch.distributed)."""

    def __init__(self, backend, E: int, k: int, d: int, group=None, direct: bool = False):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.backend = backend
        self.E, self.k, self.d = E, k, d
        self.lo, self.hi = shard_bounds(E, self.world, self.rank)
        self.direct = direct
        if direct:
            try:
                backend.setup_direct(self.dist, group, self.world, self.rank)
            except PeerMemoryUnavailable:
                self.direct = False  # on every rank alike: outputs come back by all-to-all

    def gather_counts(self, counts):
        """counts [2G] of every rank -> host matrix C[s] = rank s's counts."""
        import torch
        G = self.world
        out = torch.empty(G * 2 * G, dtype=counts.dtype, device=counts.device)
        self.dist.all_gather_into_tensor(out, counts.contiguous(), group=self.group)
        flat = out.tolist()
        return [flat[s * 2 * G:(s + 1) * 2 * G] for s in range(G)]

    def _route_dispatch(self, x):
        """route + dispatch, or -- when this rank's batch exceeds the planned
        size -- counts of -1, so that every rank learns of the error from the
        count exchange that follows (no rank raises alone and leaves the
        others waiting in a collective)."""
        import torch
        be, G = self.backend, self.world
        if x.shape[0] > be.max_tokens:
            return None, None, torch.full((2 * G,), -1, dtype=torch.int32, device=x.device), None
        be.route(x)
        return be.dispatch(G)

    @staticmethod
    def _check_counts(rows):
        if any(c < 0 for row in rows for c in row):
            raise ValueError("expert-parallel forward: a rank's batch exceeds the planned max_tokens")

    def _forward_direct(self, x, residual):
        be, G, me = self.backend, self.world, self.rank
        send_rows, send_meta, counts, pair_pos = self._route_dispatch(x)
        C = self.gather_counts(counts)  # the one host synchronisation of the call
        self._check_counts(C)
        s_rows = C[me][:G]
        r_rows = [C[s][me] for s in range(G)]
        r_pairs = [C[s][G + me] for s in range(G)]
        ns = sum(s_rows)
        # rows and meta rows over peer memory as well where that measured
        # faster than NCCL's all-to-all (2 ranks: 1572 vs 1630 us per
        # T=16384 block; at 8 ranks the per-peer copies lose, 1015 vs 944 us)
        if hasattr(be, "push_rows") and self.world <= PUSH_ROWS_MAX_RANKS:
            recv_rows, recv_meta = be.push_rows(send_rows, send_meta, C)
        else:
            recv_rows = self._a2a(send_rows[:ns], s_rows, r_rows)
            recv_meta = self._a2a(send_meta[:ns], s_rows, r_rows)
        pair_start = [0]
        for c in r_pairs:
            pair_start.append(pair_start[-1] + c)
        # rank s's buffer holds its pairs grouped by rank: this rank's chunk
        # starts after the pairs s sends to the ranks before it
        dst_row = [sum(C[s][G + r] for r in range(me)) for s in range(G)]
        be.experts_return(recv_rows, recv_meta, pair_start, dst_row)
        # push the staged outputs, barrier (every rank's outputs for this rank
        # have landed), shared expert meanwhile, combine
        return be.finish(sum(C[me][G:]), pair_pos, residual)

    def _a2a(self, send, send_counts, recv_counts):
        import torch
        recv = torch.empty((int(sum(recv_counts)),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        self.dist.all_to_all_single(recv, send, [int(c) for c in recv_counts], [int(c) for c in send_counts],
                                    group=self.group)
        return recv

    def exchange_counts(self, counts):
        """counts [2G] (rows to each rank, then pairs to each rank) -> host
        lists (rows sent, pairs sent, rows received, pairs received)."""
        import torch
        G = self.world
        mine = counts.view(2, G).t().contiguous()  # [G][2]: (rows, pairs) for rank r
        theirs = torch.empty_like(mine)
        self.dist.all_to_all_single(theirs, mine, group=self.group)
        both = torch.cat([mine.reshape(-1), theirs.reshape(-1)]).tolist()
        return both[0:2 * G:2], both[1:2 * G:2], both[2 * G::2], both[2 * G + 1::2]

    def forward(self, x, residual=None):
        """x: [T, d] local tokens.  Returns out [T, d] (float32)."""
        if self.direct:
            return self._forward_direct(x, residual)
        be = self.backend
        send_rows, send_meta, counts, pair_pos = self._route_dispatch(x)
        s_rows, s_pairs, r_rows, r_pairs = self.exchange_counts(counts)
        self._check_counts([s_rows, s_pairs, r_rows, r_pairs])
        ns = sum(s_rows)
        recv_rows = self._a2a(send_rows[:ns], s_rows, r_rows)
        recv_meta = self._a2a(send_meta[:ns], s_rows, r_rows)
        y = be.experts(recv_rows, recv_meta, sum(r_pairs))
        y_back = self._a2a(y, r_pairs, s_pairs)
        return be.combine(y_back, pair_pos, residual)


class CudaBackend:
    """The qmoe C-ABI on one GPU: the full layer's router and shared expert,
    this rank's slice of the expert tensors."""

    def __init__(self, blk, local_blk, dims, local_dims, world: int, max_tokens: int, max_rows: int,
                 norm_weight=None, eps: float = 1e-6, placement=None):
        import torch
        self.blk, self.local_blk = blk, local_blk
        self.placement = None if placement is None else torch.tensor(placement, dtype=torch.int32, device="cuda")
        self.dims, self.local_dims = dims, local_dims
        self.norm_weight, self.eps = norm_weight, eps
        self.world = world
        self.max_tokens = max_tokens
        L = _lib.lib()
        k, d = dims.top_k, dims.d_model
        self.ws_bytes = L.qmoe_workspace_size(ctypes.byref(dims), max_tokens)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device="cuda")
        _lib.check(L.qmoe_workspace_init(self.ws.data_ptr(), self.ws_bytes, None))
        self.scratch_bytes = L.qmoe_ep_dispatch_scratch_size(max_tokens, world)
        self.scratch = torch.empty(self.scratch_bytes, dtype=torch.uint8, device="cuda")
        cap = max_tokens * min(world, k)
        self.send_rows = torch.empty((cap, d), dtype=torch.float16, device="cuda")
        self.send_meta = torch.empty((cap, k), dtype=torch.int32, device="cuda")
        self.counts = torch.empty(2 * world, dtype=torch.int32, device="cuda")
        self.pair_pos = torch.empty(max_tokens * k, dtype=torch.int32, device="cuda")
        self._rows_ws(max_rows)
        self.T = 0

    def _rows_ws(self, rows: int) -> None:
        import torch
        self.max_rows = rows
        self.rws_bytes = _lib.lib().qmoe_ep_rows_workspace_size(ctypes.byref(self.local_dims), rows)
        if not self.rws_bytes:
            raise ValueError("qmoe_ep_rows_workspace_size: bad local dims")
        self.rws = torch.empty(self.rws_bytes, dtype=torch.uint8, device="cuda")
        _lib.check(_lib.lib().qmoe_workspace_init(self.rws.data_ptr(), self.rws_bytes, None))

    def _view(self, which, count, dtype):
        import torch
        p = _lib.lib().qmoe_ws_view(self.ws.data_ptr(), ctypes.byref(self.dims), self.T, which)
        off = p - self.ws.data_ptr()
        nbytes = count * torch.empty((), dtype=dtype).element_size()
        return self.ws[off:off + nbytes].view(dtype)

    def route(self, x):
        import torch
        self.T = T = x.shape[0]
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(_lib.lib().qmoe_ep_route(
            ctypes.byref(self.blk), ctypes.byref(self.dims), x.data_ptr(),
            None if self.norm_weight is None else self.norm_weight.data_ptr(), self.eps, T,
            self.ws.data_ptr(), self.ws_bytes, stream), "ep_route")

    def topk_idx(self):
        import torch
        k = self.dims.top_k
        return self._view(_lib.WS_TOPK_IDX, self.T * k, torch.int32).view(self.T, k)

    def dispatch(self, world: int):
        import torch
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(_lib.lib().qmoe_ep_dispatch(
            ctypes.byref(self.dims), self.T, world, None if self.placement is None else self.placement.data_ptr(),
            self.ws.data_ptr(), self.ws_bytes, self.send_rows.data_ptr(),
            self.send_meta.data_ptr(), self.counts.data_ptr(), self.pair_pos.data_ptr(), self.scratch.data_ptr(),
            self.scratch_bytes, stream), "ep_dispatch")
        return self.send_rows, self.send_meta, self.counts, self.pair_pos[:self.T * self.dims.top_k]

    def experts(self, rows, meta, n_pairs: int):
        import torch
        n = rows.shape[0]
        y = torch.empty((n_pairs, self.dims.d_model), dtype=torch.float16, device="cuda")
        if n:
            if n > self.max_rows:  # a rank received more rows than planned: grow its row workspace
                self._rows_ws(n)
            stream = torch.cuda.current_stream().cuda_stream
            _lib.check(_lib.lib().qmoe_ep_experts(
                ctypes.byref(self.local_blk), ctypes.byref(self.local_dims), rows.data_ptr(), meta.data_ptr(), n,
                n_pairs, y.data_ptr(), self.rws.data_ptr(), self.rws_bytes, stream), "ep_experts")
        return y

    # ---- direct return over peer memory ----
    def _shared_buffer(self, nbytes: int, world: int, rank: int):
        """IPC-shareable device buffer of this rank and every peer's mapping
        of theirs (index = rank; this rank's own pointer at its index; None
        where an allocation or a mapping failed)."""
        L = _lib.lib()
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        own = ptr.value if L.qmoe_peer_alloc(nbytes, ctypes.byref(ptr), handle) == _lib.QMOE_OK else None
        handles = [None] * world
        self.dist.all_gather_object(handles, None if own is None else bytes(handle), group=self.group)
        ptrs = []
        for s, h in enumerate(handles):
            if s == rank:
                ptrs.append(own)
                continue
            q = ctypes.c_void_p()
            if h is None or L.qmoe_peer_open((ctypes.c_uint8 * 64).from_buffer_copy(h), ctypes.byref(q)) != _lib.QMOE_OK:
                q.value = None
            ptrs.append(q.value)
        if own is not None:
            self._owned.append(own)
        self._mapped += [q for s, q in enumerate(ptrs) if s != rank and q]
        return ptrs

    def setup_direct(self, dist, group, world: int, rank: int) -> None:
        """IPC-shareable buffers mapped by every peer: this rank's return
        buffer (one fp16 row per pair of its tokens) and its receive buffers
        for rows and meta rows (one row per (token, rank) of every rank)."""
        import torch
        self.dist, self.group, self.rank_ = dist, group, rank
        self._owned, self._mapped = [], []
        d, k = self.dims.d_model, self.dims.top_k
        self.peer_ptrs = self._shared_buffer(self.pair_pos.numel() * d * 2, world, rank)
        self.ret_ptr = self.peer_ptrs[rank]
        self.recv_cap = world * self.pair_pos.numel() // k  # rows: every rank's tokens once
        self.peer_rows = self._shared_buffer(self.recv_cap * d * 2, world, rank)
        self.peer_meta = self._shared_buffer(self.recv_cap * k * 4, world, rank)
        failed = any(p is None for p in self.peer_ptrs + self.peer_rows + self.peer_meta)
        # every rank learns whether all mappings exist, so that all of them
        # take the same path (a rank that raised alone would leave the others
        # waiting in the next collective)
        ok = torch.tensor([0 if failed else 1], dtype=torch.int32, device="cuda")
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if int(ok.item()) == 0:
            self.close()
            raise PeerMemoryUnavailable("peer memory between the ranks could not be mapped")
        self.stage = None
        self.side = torch.cuda.Stream()
        self._flag = torch.zeros(1, dtype=torch.int32, device="cuda")

    def push_rows(self, send_rows, send_meta, C):
        """Rows and meta rows to every rank's receive buffers with the copy
        engines (this rank's chunk for rank r lands after the chunks of the
        ranks before it), then a barrier; returns this rank's received rows."""
        import torch
        L = _lib.lib()
        G, me = len(C), self.rank_
        d, k = self.dims.d_model, self.dims.top_k
        stream = torch.cuda.current_stream().cuda_stream
        src = 0
        for r in range(G):
            n = C[me][r]
            if n:
                at = sum(C[s][r] for s in range(me))
                # holds by construction: a rank sends each of its <= max_tokens
                # tokens to a rank at most once, and the buffer has room for
                # every rank's max_tokens rows
                assert at + n <= self.recv_cap, "expert-parallel receive buffer too small"
                _lib.check(L.qmoe_copy_async(self.peer_rows[r] + at * d * 2, send_rows.data_ptr() + src * d * 2,
                                             n * d * 2, stream), "copy_async")
                _lib.check(L.qmoe_copy_async(self.peer_meta[r] + at * k * 4, send_meta.data_ptr() + src * k * 4,
                                             n * k * 4, stream), "copy_async")
            src += n
        self.dist.all_reduce(self._flag, group=self.group)  # every chunk for this rank has landed
        n_recv = sum(C[s][me] for s in range(G))
        rows = torch.as_tensor(_DevicePtr(self.peer_rows[me], max(n_recv, 1) * d * 2), device="cuda")
        meta = torch.as_tensor(_DevicePtr(self.peer_meta[me], max(n_recv, 1) * k * 4), device="cuda")
        return (rows.view(torch.float16).view(-1, d)[:n_recv], meta.view(torch.int32).view(-1, k)[:n_recv])

    def experts_return(self, rows, meta, pair_start, dst_row) -> None:
        """This rank's experts on the received rows; the outputs of rank s's
        pairs land in rank s's return buffer from row dst_row[s] on."""
        import torch
        n = rows.shape[0]
        if n == 0:
            return
        if n > self.max_rows:
            self._rows_ws(n)
        L = _lib.lib()
        row_bytes = self.dims.d_model * 2
        n_pairs = pair_start[-1]
        if self.stage is None or self.stage.shape[0] < n_pairs:
            self.stage = torch.empty((n_pairs, self.dims.d_model), dtype=torch.float16, device="cuda")
        ret = _lib.QmoeEpReturn()
        ret.n_ranks = len(dst_row)
        for i, v in enumerate(pair_start):
            ret.pair_start[i] = v
        for s, r0 in enumerate(dst_row):  # own pairs: final place; the others: staged in received order
            own = s == self.rank_
            ret.dst[s] = self.ret_ptr if own else self.stage.data_ptr()
            ret.dst_row[s] = r0 if own else pair_start[s]
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(L.qmoe_ep_experts_return(
            ctypes.byref(self.local_blk), ctypes.byref(self.local_dims), rows.data_ptr(), meta.data_ptr(), n,
            ctypes.byref(ret), self.rws.data_ptr(), self.rws_bytes, stream), "ep_experts_return")
        self.pushes = [(self.peer_ptrs[s] + r0 * row_bytes, self.stage.data_ptr() + pair_start[s] * row_bytes,
                        (pair_start[s + 1] - pair_start[s]) * row_bytes)
                       for s, r0 in enumerate(dst_row) if s != self.rank_ and pair_start[s + 1] > pair_start[s]]

    def finish(self, n_pairs: int, pair_pos, residual=None):
        """Push the staged outputs to their ranks (copy engines) and barrier on
        a side stream while the shared expert runs on this stream; then the
        combine of this rank's tokens from its return buffer."""
        import torch
        L = _lib.lib()
        main = torch.cuda.current_stream()
        ready = torch.cuda.Event()
        ready.record(main)
        with torch.cuda.stream(self.side):
            self.side.wait_event(ready)
            for dst, src, nb in getattr(self, "pushes", []):
                _lib.check(L.qmoe_copy_async(dst, src, nb, self.side.cuda_stream), "copy_async")
            self.dist.all_reduce(self._flag, group=self.group)
            landed = torch.cuda.Event()
            landed.record(self.side)
        self.pushes = []
        _lib.check(L.qmoe_ep_shared(ctypes.byref(self.blk), ctypes.byref(self.dims), self.T, self.ws.data_ptr(),
                                    self.ws_bytes, main.cuda_stream), "ep_shared")
        main.wait_event(landed)
        out = torch.empty((self.T, self.dims.d_model), dtype=torch.float32, device="cuda")
        y = self.returned(n_pairs)
        _lib.check(L.qmoe_ep_combine_routed(
            ctypes.byref(self.blk), ctypes.byref(self.dims), y.data_ptr(), pair_pos.data_ptr(), self.T,
            None if residual is None else residual.data_ptr(), out.data_ptr(), self.ws.data_ptr(), self.ws_bytes,
            main.cuda_stream), "ep_combine_routed")
        return out

    def returned(self, n_pairs: int):
        """This rank's return buffer as [n_pairs][d] fp16."""
        import torch
        if n_pairs == 0:
            return torch.zeros((1, self.dims.d_model), dtype=torch.float16, device="cuda")
        t = _DevicePtr(self.ret_ptr, n_pairs * self.dims.d_model * 2)
        return torch.as_tensor(t, device="cuda").view(torch.float16).view(n_pairs, self.dims.d_model)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after the last call)."""
        L = _lib.lib()
        for ptr in getattr(self, "_mapped", []):
            L.qmoe_peer_close(ptr)
        for ptr in getattr(self, "_owned", []):
            L.qmoe_peer_free(ptr)
        self._mapped, self._owned, self.peer_ptrs = [], [], []
        self.ret_ptr = None

    def combine(self, y, pair_pos, residual=None):
        import torch
        out = torch.empty((self.T, self.dims.d_model), dtype=torch.float32, device="cuda")
        if y.shape[0] == 0:  # no pair anywhere (every token failed routing): any valid pointer will do
            y = torch.zeros((1, self.dims.d_model), dtype=torch.float16, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(_lib.lib().qmoe_ep_combine(
            ctypes.byref(self.blk), ctypes.byref(self.dims), y.data_ptr(), pair_pos.data_ptr(), self.T,
            None if residual is None else residual.data_ptr(), out.data_ptr(), self.ws.data_ptr(), self.ws_bytes,
            stream), "ep_combine")
        return out


class _DevicePtr:
    """A raw device allocation seen by torch through __cuda_array_interface__
    (bytes, read-write); the memory stays owned by the caller."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def local_block_placed(blk: "_lib.QmoeBlock", dims, experts) -> tuple:
    """The rank's experts (global ids, in local-id order) copied into
    contiguous [E_loc][rows][K] tensors on this GPU, as qmoe_ep_experts
    reads them.  Returns (block, dims, buffers to keep alive)."""
    import torch
    from .quant import calculate_tensor_bytes
    n, d, F = len(experts), dims.d_model, dims.expert_dim
    L = _lib.lib()
    keep = []

    def gather(t, rows, K):
        per_expert = calculate_tensor_bytes(t.ggml_type, rows * K)
        buf = torch.empty(n * per_expert, dtype=torch.uint8, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        for i, e in enumerate(experts):
            _lib.check(L.qmoe_copy_async(buf.data_ptr() + i * per_expert, (t.data or 0) + e * per_expert, per_expert,
                                         stream), "copy_async")
        keep.append(buf)
        return _lib.QmoeTensor(buf.data_ptr(), t.ggml_type, 0, n * rows * K)

    lb = _lib.QmoeBlock(blk.router, gather(blk.gate_exps, F, d), gather(blk.up_exps, F, d),
                        gather(blk.down_exps, d, F), blk.shared_gate_inp, blk.shared_gate, blk.shared_up,
                        blk.shared_down, None)
    return lb, _lib.QmoeDims(d, n, dims.top_k, F, dims.shared_dim), keep


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
    ld = _lib.QmoeDims(d, n, dims.top_k, F, dims.shared_dim)  # top_k: the layer's k (meta row width)
    return lb, ld
