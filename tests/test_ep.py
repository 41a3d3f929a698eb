"""Expert-parallel exchange (qmoe/ep.py) on CPU: gloo ranks and a fake compute
backend whose experts are simple per-expert scalings, checked against the same
block computed without the exchange.  The backend's route / dispatch /
experts / combine are the qmoe_ep_* calls on a GPU; here they are numpy (the
dispatch layout from tests/ep_plan_ref.py, which the CUDA kernels are checked
against on the GPU) so that only the exchange logic (count exchange, row and
meta all-to-all, return of the outputs, pair placement, invalid slots, ragged
and empty ranks) is under test."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import ep_plan_ref
from qmoe import ep

D, K = 16, 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _routing(x: np.ndarray, E: int, seed: int):
    """A deterministic top-k of x @ W (ties impossible at these sizes), with
    every seventh token's last slot marked invalid (-1)."""
    W = np.random.default_rng(seed).standard_normal((D, E)).astype(np.float32)
    logits = x @ W
    idx = np.argsort(-logits, axis=1, kind="stable")[:, :K].astype(np.int32)
    w = np.take_along_axis(logits, idx, 1)
    w = np.exp(w - w.max(1, keepdims=True))
    w /= w.sum(1, keepdims=True)
    idx[::7, K - 1] = -1
    return idx, w.astype(np.float32)


def _scale(E: int) -> np.ndarray:
    return 1.0 + np.arange(E, dtype=np.float32) / 8


def _reference(x: np.ndarray, E: int, seed: int) -> np.ndarray:
    idx, w = _routing(x, E, seed)
    s = _scale(E)
    out = x.copy()
    for t in range(x.shape[0]):
        for j in range(K):
            if idx[t, j] >= 0:
                out[t] += w[t, j] * s[idx[t, j]] * x[t]
    return out


class FakeBackend:
    """route / dispatch / experts / combine with the semantics of the
    qmoe_ep_* calls, on the host."""

    def __init__(self, E: int, lo: int, seed: int, max_tokens: int = 1 << 20):
        self.E, self.lo, self.seed = E, lo, seed
        self.max_tokens = max_tokens
        self.received = 0

    def route(self, x):
        self.x = x.numpy()
        self.idx, self.w = _routing(self.x, self.E, self.seed)

    def dispatch(self, G):
        tok, meta, counts, pair_pos = ep_plan_ref.dispatch_plan(self.idx, self.E, G)
        rows = self.x[tok] if len(tok) else np.zeros((0, D), np.float32)
        return (torch.from_numpy(np.ascontiguousarray(rows)), torch.from_numpy(meta.reshape(-1, K)),
                torch.from_numpy(counts), torch.from_numpy(pair_pos))

    def experts(self, rows, meta, n_pairs):
        m = meta.numpy()
        r, e = ep_plan_ref.pair_rows(m)
        assert len(r) == n_pairs
        self.received += n_pairs
        assert (e < self.E).all()
        y = rows.numpy()[r] * _scale(self.E)[self.lo + e][:, None] if n_pairs else np.zeros((0, D), np.float32)
        return torch.from_numpy(np.ascontiguousarray(y, dtype=np.float32))

    # direct return: every rank's return buffer is a slice of one shared-memory
    # array (standing in for the peer mappings of the GPU path)
    def setup_direct(self, dist, group, world, rank):
        from multiprocessing import shared_memory
        self.dist, self.rank = dist, rank
        self.shm = shared_memory.SharedMemory(name=self.shm_name)
        n_ret, n_rows = world * self.cap * D, world * self.rcap * D
        self.bufs = np.ndarray((world, self.cap, D), dtype=np.float32, buffer=self.shm.buf)
        self.rows_in = np.ndarray((world, self.rcap, D), dtype=np.float32, buffer=self.shm.buf, offset=4 * n_ret)
        self.meta_in = np.ndarray((world, self.rcap, K), dtype=np.int32, buffer=self.shm.buf,
                                  offset=4 * (n_ret + n_rows))

    def push_rows(self, send_rows, send_meta, C):
        G, me = len(C), self.rank
        src = 0
        for r in range(G):
            n = C[me][r]
            at = sum(C[s][r] for s in range(me))
            self.rows_in[r, at:at + n] = send_rows.numpy()[src:src + n]
            self.meta_in[r, at:at + n] = send_meta.numpy()[src:src + n]
            src += n
        self.dist.barrier()
        n_recv = sum(C[s][me] for s in range(G))
        return (torch.from_numpy(self.rows_in[me, :n_recv].copy()), torch.from_numpy(self.meta_in[me, :n_recv].copy()))

    def experts_return(self, rows, meta, pair_start, dst_row):
        self.pending = (self.experts(rows, meta, pair_start[-1]).numpy(), pair_start, dst_row)

    def finish(self, n_pairs, pair_pos, residual=None):
        if getattr(self, "pending", None) is not None:
            y, pair_start, dst_row = self.pending
            for s in range(len(dst_row)):
                q0, q1 = pair_start[s], pair_start[s + 1]
                self.bufs[s, dst_row[s]:dst_row[s] + q1 - q0] = y[q0:q1]
        self.pending = None
        self.dist.barrier()
        return self.combine(torch.from_numpy(self.bufs[self.rank, :n_pairs].copy()), pair_pos, residual)

    def combine(self, y, pair_pos, residual=None):
        T = self.x.shape[0]
        yv, pp = y.numpy(), pair_pos.numpy()
        out = self.x.copy()
        for t in range(T):
            for j in range(K):
                if pp[t * K + j] >= 0:
                    out[t] += self.w[t, j] * yv[pp[t * K + j]]
        return torch.from_numpy(out)


def _worker(rank, world, port, E, token_counts, seed, q, shm_name=None, max_tokens=1 << 20):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = ep.shard_bounds(E, world, rank)
        be = FakeBackend(E, lo, seed, max_tokens)
        be.shm_name, be.cap, be.rcap = shm_name, max(token_counts) * K, sum(token_counts)
        moe = ep.ExpertParallelMoE(be, E, K, D, direct=shm_name is not None)
        x = np.random.default_rng(100 + rank).standard_normal((token_counts[rank], D)).astype(np.float32)
        try:
            out = moe.forward(torch.from_numpy(x)).numpy()
        except ValueError as err:  # every rank must see a batch-size error, none may hang
            q.put((rank, "error", str(err), 0))
            return
        ref = _reference(x, E, seed)
        q.put((rank, float(np.abs(out - ref).max()) if out.size else 0.0, out.shape, be.received))
    finally:
        dist.destroy_process_group()


def _run(world, E, token_counts, seed=5, direct=False, max_tokens=1 << 20):
    from multiprocessing import shared_memory
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    size = world * (max(token_counts) * K * D + sum(token_counts) * (D + K)) * 4
    shm = shared_memory.SharedMemory(create=True, size=size) if direct else None
    try:
        ps = [ctx.Process(target=_worker,
                          args=(r, world, port, E, token_counts, seed, q, shm.name if shm else None, max_tokens))
              for r in range(world)]
        for p in ps:
            p.start()
        for p in ps:
            p.join(120)
        assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
        res = sorted(q.get() for _ in range(world))
    finally:
        if shm is not None:
            shm.close()
            shm.unlink()
    return res


def test_dispatch_plan_layout():
    idx = np.array([[5, 0, 3], [-1, -1, -1], [6, 1, 4]], dtype=np.int32)
    tok, meta, counts, pair_pos = ep_plan_ref.dispatch_plan(idx, 8, 2)
    # rank 0 owns experts 0..3, rank 1 owns 4..7; one row per (token, rank)
    assert tok.tolist() == [0, 2, 0, 2]
    assert meta.tolist() == [[-1, 0, 3], [-1, 1, -1], [1, -1, -1], [2, -1, 0]]
    assert counts.tolist() == [2, 2, 3, 3]
    # returned outputs: rank 0's pairs (0,1) (0,2) (2,1), then rank 1's (0,0) (2,0) (2,2)
    assert pair_pos.tolist() == [3, 0, 1, -1, -1, -1, 4, 2, 5]


def test_dispatch_plan_with_placement():
    # experts 0 and 4 are hot: placement puts them on different ranks
    pl = ep.balanced_placement([10, 1, 1, 1, 9, 1, 1, 1], 2)
    assert pl == [0, 5, 1, 6, 4, 2, 7, 3]
    assert ep.experts_of_rank(pl, 2, 0) == [0, 2, 5, 7] and ep.experts_of_rank(pl, 2, 1) == [4, 1, 3, 6]
    idx = np.array([[0, 4, 2], [7, 1, -1]], dtype=np.int32)
    tok, meta, counts, pair_pos = ep_plan_ref.dispatch_plan(idx, 8, 2, pl)
    # token 0: experts 0 (rank 0 local 0), 4 (rank 1 local 0), 2 (rank 0 local 1); token 1: 7 (rank 0 local 3), 1 (rank 1 local 1)
    assert tok.tolist() == [0, 1, 0, 1]
    assert meta.tolist() == [[0, -1, 1], [3, -1, -1], [-1, 0, -1], [-1, 1, -1]]
    assert counts.tolist() == [2, 2, 3, 2]
    assert pair_pos.tolist() == [0, 3, 1, 2, 4, -1]


def test_shard_bounds():
    assert ep.shard_bounds(256, 8, 3) == (96, 128)
    with pytest.raises(ValueError):
        ep.shard_bounds(256, 3, 0)


@pytest.mark.parametrize("direct", [False, True], ids=["all_to_all_return", "direct_return"])
@pytest.mark.parametrize("world,E,tokens", [(2, 8, [13, 9]), (4, 16, [5, 0, 11, 3])])
def test_exchange_matches_single_process(world, E, tokens, direct):
    res = _run(world, E, tokens, direct=direct)
    for rank, err, shape, _ in res:
        assert shape == (tokens[rank], D)
        assert err < 1e-5, (rank, err)
    # every valid pair is computed exactly once across the ranks
    total_valid = 0
    for r in range(world):
        x = np.random.default_rng(100 + r).standard_normal((tokens[r], D)).astype(np.float32)
        idx, _ = _routing(x, E, 5)
        total_valid += int((idx >= 0).sum())
    assert sum(r[3] for r in res) == total_valid


@pytest.mark.parametrize("direct", [False, True], ids=["all_to_all_return", "direct_return"])
def test_oversized_batch_fails_on_every_rank(direct):
    # rank 1 holds more tokens than the backends were planned for: it must not
    # route, and both ranks must raise together instead of one waiting in a
    # collective for the other
    res = _run(2, 8, [4, 9], direct=direct, max_tokens=8)
    assert [r[1] for r in res] == ["error", "error"], res
    assert all("max_tokens" in r[2] for r in res)
