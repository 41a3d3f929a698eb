// Expert-parallel MoE block over NCCL (include/qmoe_ep.h): the host-side
// exchange around the qmoe expert-parallel entry points of include/qmoe.h.
// Built into libqmoe_ep.so (links libqmoe, NCCL and the CUDA runtime), so the
// single-GPU library carries no NCCL dependency.
#include "qmoe_ep.h"

#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>
#include <vector>

namespace {

constexpr int kMaxRanks = 32;          // qmoe_ep_return holds 32 ranks
constexpr int kPushRowsMaxRanks = 2;   // rows over peer memory only up to here (NCCL measured faster at 8)

struct Ctx {
    ncclComm_t comm = nullptr;
    int G = 1, me = 0;
    qmoe_dims dims{}, ldims{};
    int max_tokens = 0;
    bool direct = false;
    // full-layer workspace (route, dispatch source, shared expert, combine)
    void* ws = nullptr;
    size_t ws_bytes = 0;
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    void* send_rows = nullptr;   // fp16 [max_tokens * min(G, k)][d]
    int32_t* send_meta = nullptr;
    int32_t* counts = nullptr;      // [2G]
    int32_t* counts_all = nullptr;  // [G][2G]
    int32_t* h_counts = nullptr;    // pinned copy
    int32_t* pair_pos = nullptr;    // [max_tokens * k]
    // this rank's experts
    void* rws = nullptr;
    size_t rws_bytes = 0;
    int recv_cap = 0;   // rows: every rank's tokens once
    int pairs_cap = 0;  // received pairs
    void* recv_rows = nullptr;
    int32_t* recv_meta = nullptr;
    void* y = nullptr;       // outputs of received pairs (all-to-all return)
    void* y_back = nullptr;  // this rank's pairs back (all-to-all return)
    // peer memory (QMOE_EP_DIRECT)
    void* own[3] = {nullptr, nullptr, nullptr};  // return, rows, meta
    void* peer[3][kMaxRanks] = {};
    void* stage = nullptr;
    int32_t* flag = nullptr;
    cudaStream_t side = nullptr;
    cudaEvent_t ev_counts = nullptr, ev_ready = nullptr, ev_landed = nullptr;
};

int cu(cudaError_t e) { return e == cudaSuccess ? QMOE_OK : QMOE_ERR_CUDA; }
int nc(ncclResult_t r) { return r == ncclSuccess ? QMOE_OK : QMOE_ERR_COMM; }

#define TRY(expr)                      \
    do {                               \
        const int st_ = (expr);        \
        if (st_ != QMOE_OK) return st_; \
    } while (0)

size_t row_bytes16(const qmoe_dims& d) { return static_cast<size_t>(d.d_model) * 2; }

void release(Ctx* c) {
    cudaDeviceSynchronize();
    for (int b = 0; b < 3; ++b)
        for (int s = 0; s < c->G; ++s)
            if (s != c->me && c->peer[b][s]) qmoe_peer_close(c->peer[b][s]);
    for (void*& p : c->own)
        if (p) {
            qmoe_peer_free(p);
            p = nullptr;
        }
    void* bufs[] = {c->ws, c->scratch, c->send_rows, c->send_meta, c->counts, c->counts_all, c->pair_pos, c->rws,
                    c->recv_rows, c->recv_meta, c->y, c->y_back, c->stage, c->flag};
    for (void* p : bufs)
        if (p) cudaFree(p);
    if (c->h_counts) cudaFreeHost(c->h_counts);
    if (c->side) cudaStreamDestroy(c->side);
    if (c->ev_counts) cudaEventDestroy(c->ev_counts);
    if (c->ev_ready) cudaEventDestroy(c->ev_ready);
    if (c->ev_landed) cudaEventDestroy(c->ev_landed);
}

// IPC buffers of every rank mapped by every peer; returns false on this rank
// if any allocation or mapping failed (the caller agrees with the others).
bool setup_peers(Ctx* c, const size_t bytes[3]) {
    bool ok = true;
    uint8_t mine[3][64] = {};
    for (int b = 0; b < 3; ++b)
        if (qmoe_peer_alloc(bytes[b], &c->own[b], mine[b]) != QMOE_OK) ok = false;
    uint8_t* d_all = nullptr;
    const size_t per = 3 * 64;
    if (cudaMalloc(&d_all, per * (c->G + 1)) != cudaSuccess) return false;
    std::vector<uint8_t> all(per * c->G);
    bool exch = cudaMemcpy(d_all + per * c->G, mine, per, cudaMemcpyHostToDevice) == cudaSuccess &&
                ncclAllGather(d_all + per * c->G, d_all, per, ncclUint8, c->comm, nullptr) == ncclSuccess &&
                cudaMemcpy(all.data(), d_all, per * c->G, cudaMemcpyDeviceToHost) == cudaSuccess;
    cudaFree(d_all);
    if (!exch) return false;
    for (int s = 0; s < c->G; ++s)
        for (int b = 0; b < 3; ++b) {
            if (s == c->me) {
                c->peer[b][s] = c->own[b];
                continue;
            }
            bool zero = true;
            for (int i = 0; i < 64; ++i) zero = zero && all[per * s + 64 * b + i] == 0;
            if (zero || qmoe_peer_open(&all[per * s + 64 * b], &c->peer[b][s]) != QMOE_OK) {
                c->peer[b][s] = nullptr;
                ok = false;
            }
        }
    return ok;
}

void drop_peers(Ctx* c) {
    cudaDeviceSynchronize();
    for (int b = 0; b < 3; ++b)
        for (int s = 0; s < c->G; ++s) {
            if (s != c->me && c->peer[b][s]) qmoe_peer_close(c->peer[b][s]);
            c->peer[b][s] = nullptr;
        }
    for (void*& p : c->own)
        if (p) {
            qmoe_peer_free(p);
            p = nullptr;
        }
}

int init_impl(Ctx* c, void* comm, const qmoe_dims* D, int max_tokens, int flags) {
    c->comm = static_cast<ncclComm_t>(comm);
    TRY(nc(ncclCommCount(c->comm, &c->G)));
    TRY(nc(ncclCommUserRank(c->comm, &c->me)));
    if (c->G < 1 || c->G > kMaxRanks || D->num_experts % c->G) return QMOE_ERR_UNSUPPORTED;
    c->dims = *D;
    c->ldims = *D;
    c->ldims.num_experts = D->num_experts / c->G;
    c->max_tokens = max_tokens;
    const int G = c->G, k = D->top_k;
    const size_t rb = row_bytes16(*D);
    c->ws_bytes = qmoe_workspace_size(D, max_tokens);
    c->scratch_bytes = qmoe_ep_dispatch_scratch_size(max_tokens, G);
    c->recv_cap = G * max_tokens;
    c->pairs_cap = G * max_tokens * std::min(k, c->ldims.num_experts);
    c->rws_bytes = qmoe_ep_rows_workspace_size(&c->ldims, c->recv_cap);
    if (!c->ws_bytes || !c->scratch_bytes || !c->rws_bytes) return QMOE_ERR_UNSUPPORTED;
    const size_t send_cap = static_cast<size_t>(max_tokens) * std::min(G, k);
    TRY(cu(cudaMalloc(&c->ws, c->ws_bytes)));
    TRY(cu(cudaMalloc(&c->scratch, c->scratch_bytes)));
    TRY(cu(cudaMalloc(&c->send_rows, send_cap * rb)));
    TRY(cu(cudaMalloc(reinterpret_cast<void**>(&c->send_meta), send_cap * k * 4)));
    TRY(cu(cudaMalloc(reinterpret_cast<void**>(&c->counts), 2 * G * 4)));
    TRY(cu(cudaMalloc(reinterpret_cast<void**>(&c->counts_all), 2 * G * G * 4)));
    TRY(cu(cudaHostAlloc(reinterpret_cast<void**>(&c->h_counts), 2 * G * G * 4, cudaHostAllocDefault)));
    TRY(cu(cudaMalloc(reinterpret_cast<void**>(&c->pair_pos), static_cast<size_t>(max_tokens) * k * 4)));
    TRY(cu(cudaMalloc(&c->rws, c->rws_bytes)));
    TRY(cu(cudaMalloc(reinterpret_cast<void**>(&c->flag), 256)));
    TRY(cu(cudaMemset(c->flag, 0, 256)));
    TRY(cu(cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking)));
    TRY(cu(cudaEventCreateWithFlags(&c->ev_counts, cudaEventDisableTiming)));
    TRY(cu(cudaEventCreateWithFlags(&c->ev_ready, cudaEventDisableTiming)));
    TRY(cu(cudaEventCreateWithFlags(&c->ev_landed, cudaEventDisableTiming)));
    TRY(qmoe_workspace_init(c->ws, c->ws_bytes, nullptr));
    TRY(qmoe_workspace_init(c->rws, c->rws_bytes, nullptr));
    if ((flags & QMOE_EP_DIRECT) && G > 1) {
        // return buffer: one row per pair of this rank's tokens; receive
        // buffers: one row (and meta row) per token of every rank
        const size_t bytes[3] = {static_cast<size_t>(max_tokens) * k * rb, static_cast<size_t>(c->recv_cap) * rb,
                                 static_cast<size_t>(c->recv_cap) * k * 4};
        int ok = setup_peers(c, bytes) ? 1 : 0;
        int* d_ok = c->flag + 32;
        // every rank learns whether all mappings exist, so all take the same path
        TRY(cu(cudaMemcpy(d_ok, &ok, 4, cudaMemcpyHostToDevice)));
        TRY(nc(ncclAllReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, c->comm, nullptr)));
        TRY(cu(cudaMemcpy(&ok, d_ok, 4, cudaMemcpyDeviceToHost)));
        c->direct = ok == 1;
        if (!c->direct) drop_peers(c);
    }
    if (c->direct) {
        TRY(cu(cudaMalloc(&c->stage, static_cast<size_t>(c->pairs_cap) * rb)));
        if (G > kPushRowsMaxRanks) {
            TRY(cu(cudaMalloc(&c->recv_rows, static_cast<size_t>(c->recv_cap) * rb)));
            TRY(cu(cudaMalloc(reinterpret_cast<void**>(&c->recv_meta), static_cast<size_t>(c->recv_cap) * k * 4)));
        }
    } else {
        TRY(cu(cudaMalloc(&c->recv_rows, static_cast<size_t>(c->recv_cap) * rb)));
        TRY(cu(cudaMalloc(reinterpret_cast<void**>(&c->recv_meta), static_cast<size_t>(c->recv_cap) * k * 4)));
        TRY(cu(cudaMalloc(&c->y, static_cast<size_t>(c->pairs_cap) * rb)));
        TRY(cu(cudaMalloc(&c->y_back, static_cast<size_t>(max_tokens) * k * rb)));
    }
    return cu(cudaDeviceSynchronize());
}

// Grouped send/recv of variable-size chunks: rank r gets send_n[r] items of
// `item` bytes from send + send_off[r]; recv_n[r] items from rank r land at
// recv + recv_off[r].
int exchange(Ctx* c, const void* send, const std::vector<int>& send_n, void* recv, const std::vector<int>& recv_n,
             size_t item, cudaStream_t s) {
    TRY(nc(ncclGroupStart()));
    size_t so = 0, ro = 0;
    for (int r = 0; r < c->G; ++r) {
        if (send_n[r])
            if (ncclSend(static_cast<const uint8_t*>(send) + so, send_n[r] * item, ncclUint8, r, c->comm, s) != ncclSuccess) {
                ncclGroupEnd();
                return QMOE_ERR_COMM;
            }
        if (recv_n[r])
            if (ncclRecv(static_cast<uint8_t*>(recv) + ro, recv_n[r] * item, ncclUint8, r, c->comm, s) != ncclSuccess) {
                ncclGroupEnd();
                return QMOE_ERR_COMM;
            }
        so += send_n[r] * item;
        ro += recv_n[r] * item;
    }
    return nc(ncclGroupEnd());
}

int forward_impl(Ctx* c, const qmoe_block* layer, const qmoe_block* local, const int32_t* placement, const float* x,
                 const float* norm_w, float eps, const float* residual, float* out, int T, cudaStream_t s) {
    const int G = c->G, me = c->me, k = c->dims.top_k;
    const size_t rb = row_bytes16(c->dims);
    // a batch over the planned size becomes counts of -1 (every rank then sees it in the exchange)
    const bool too_big = T > c->max_tokens;
    if (!too_big) {
        TRY(qmoe_ep_route(layer, &c->dims, x, norm_w, eps, T, c->ws, c->ws_bytes, s));
        TRY(qmoe_ep_dispatch(&c->dims, T, G, placement, c->ws, c->ws_bytes, c->send_rows, c->send_meta, c->counts,
                             c->pair_pos, c->scratch, c->scratch_bytes, s));
    } else {
        TRY(cu(cudaMemsetAsync(c->counts, 0xFF, 2 * G * 4, s)));
    }
    TRY(nc(ncclAllGather(c->counts, c->counts_all, 2 * G, ncclInt32, c->comm, s)));
    TRY(cu(cudaMemcpyAsync(c->h_counts, c->counts_all, 2 * G * G * 4, cudaMemcpyDeviceToHost, s)));
    TRY(cu(cudaEventRecord(c->ev_counts, s)));
    TRY(cu(cudaEventSynchronize(c->ev_counts)));  // the one host synchronisation of the call
    const int32_t* C = c->h_counts;               // C[s*2G + r]: rows s -> r; C[s*2G + G + r]: pairs s -> r
    for (int i = 0; i < 2 * G * G; ++i)
        if (C[i] < 0) return QMOE_ERR_ARG;  // some rank's batch exceeds max_tokens: every rank returns this
    std::vector<int> s_rows(G), r_rows(G), s_pairs(G), r_pairs(G);
    int n_recv = 0, n_pairs = 0;
    for (int r = 0; r < G; ++r) {
        s_rows[r] = C[me * 2 * G + r];
        s_pairs[r] = C[me * 2 * G + G + r];
        r_rows[r] = C[r * 2 * G + me];
        r_pairs[r] = C[r * 2 * G + G + me];
        n_recv += r_rows[r];
        n_pairs += r_pairs[r];
    }
    if (n_recv > c->recv_cap || n_pairs > c->pairs_cap) return QMOE_ERR_ARG;  // cannot happen for valid counts
    // rows and meta rows to the ranks that own the experts
    const void* rows = c->recv_rows;
    const int32_t* meta = c->recv_meta;
    if (c->direct && G <= kPushRowsMaxRanks) {
        size_t src = 0;
        for (int r = 0; r < G; ++r) {
            const int n = s_rows[r];
            if (n) {
                int at = 0;  // this rank's chunk lands after the chunks of the ranks before it
                for (int q = 0; q < me; ++q) at += C[q * 2 * G + r];
                TRY(qmoe_copy_async(static_cast<uint8_t*>(c->peer[1][r]) + static_cast<size_t>(at) * rb,
                                    static_cast<const uint8_t*>(c->send_rows) + src * rb, n * rb, s));
                TRY(qmoe_copy_async(static_cast<uint8_t*>(c->peer[2][r]) + static_cast<size_t>(at) * k * 4,
                                    c->send_meta + src * k, static_cast<size_t>(n) * k * 4, s));
            }
            src += n;
        }
        TRY(nc(ncclAllReduce(c->flag, c->flag, 1, ncclInt32, ncclSum, c->comm, s)));  // every chunk has landed
        rows = c->own[1];
        meta = static_cast<const int32_t*>(c->own[2]);
    } else {
        TRY(exchange(c, c->send_rows, s_rows, c->recv_rows, r_rows, rb, s));
        TRY(exchange(c, c->send_meta, s_rows, c->recv_meta, r_rows, static_cast<size_t>(k) * 4, s));
    }
    if (c->direct) {
        // outputs: own pairs in place, the other ranks' pairs staged, then
        // pushed into their return buffers by the copy engines on the side stream
        qmoe_ep_return ret{};
        ret.n_ranks = G;
        ret.pair_start[0] = 0;
        for (int q = 0; q < G; ++q) ret.pair_start[q + 1] = ret.pair_start[q] + r_pairs[q];
        for (int q = 0; q < G; ++q) {
            int before = 0;  // pairs rank q sends to the ranks before this one
            for (int r = 0; r < me; ++r) before += C[q * 2 * G + G + r];
            ret.dst[q] = q == me ? c->own[0] : c->stage;
            ret.dst_row[q] = q == me ? before : ret.pair_start[q];
        }
        if (n_recv) TRY(qmoe_ep_experts_return(local, &c->ldims, rows, meta, n_recv, &ret, c->rws, c->rws_bytes, s));
        TRY(cu(cudaEventRecord(c->ev_ready, s)));
        TRY(cu(cudaStreamWaitEvent(c->side, c->ev_ready, 0)));
        for (int q = 0; q < G; ++q) {
            const int n = r_pairs[q];
            if (q == me || !n) continue;
            int before = 0;
            for (int r = 0; r < me; ++r) before += C[q * 2 * G + G + r];
            TRY(qmoe_copy_async(static_cast<uint8_t*>(c->peer[0][q]) + static_cast<size_t>(before) * rb,
                                static_cast<const uint8_t*>(c->stage) + static_cast<size_t>(ret.pair_start[q]) * rb,
                                static_cast<size_t>(n) * rb, c->side));
        }
        TRY(nc(ncclAllReduce(c->flag, c->flag, 1, ncclInt32, ncclSum, c->comm, c->side)));  // every push landed
        TRY(cu(cudaEventRecord(c->ev_landed, c->side)));
        // the shared expert (it needs only the routing) while the copy engines push
        TRY(qmoe_ep_shared(layer, &c->dims, T, c->ws, c->ws_bytes, s));
        TRY(cu(cudaStreamWaitEvent(s, c->ev_landed, 0)));
        return qmoe_ep_combine_routed(layer, &c->dims, c->own[0], c->pair_pos, T, residual, out, c->ws, c->ws_bytes, s);
    }
    if (n_recv) TRY(qmoe_ep_experts(local, &c->ldims, rows, meta, n_recv, n_pairs, c->y, c->rws, c->rws_bytes, s));
    TRY(qmoe_ep_shared(layer, &c->dims, T, c->ws, c->ws_bytes, s));
    TRY(exchange(c, c->y, r_pairs, c->y_back, s_pairs, rb, s));
    return qmoe_ep_combine_routed(layer, &c->dims, c->y_back, c->pair_pos, T, residual, out, c->ws, c->ws_bytes, s);
}

}  // namespace

struct qmoe_ep {
    Ctx c;
};

extern "C" {

int qmoe_ep_unique_id(uint8_t id[128]) {
    if (!id) return QMOE_ERR_ARG;
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
    ncclUniqueId u;
    TRY(nc(ncclGetUniqueId(&u)));
    std::memcpy(id, &u, 128);
    return QMOE_OK;
}

int qmoe_ep_comm_init(const uint8_t id[128], int world, int rank, void** nccl_comm) {
    if (!id || !nccl_comm || world < 1 || rank < 0 || rank >= world) return QMOE_ERR_ARG;
    ncclUniqueId u;
    std::memcpy(&u, id, 128);
    ncclComm_t comm = nullptr;
    TRY(nc(ncclCommInitRank(&comm, world, u, rank)));
    *nccl_comm = comm;
    return QMOE_OK;
}

int qmoe_ep_comm_destroy(void* nccl_comm) {
    if (!nccl_comm) return QMOE_ERR_ARG;
    return nc(ncclCommDestroy(static_cast<ncclComm_t>(nccl_comm)));
}

int qmoe_ep_init(void* nccl_comm, const qmoe_dims* dims, int max_tokens, int flags, qmoe_ep** ep) {
    if (!nccl_comm || !dims || !ep || max_tokens <= 8) return QMOE_ERR_ARG;
    *ep = nullptr;
    qmoe_ep* e = new (std::nothrow) qmoe_ep;
    if (!e) return QMOE_ERR_CUDA;
    const int st = init_impl(&e->c, nccl_comm, dims, max_tokens, flags);
    if (st != QMOE_OK) {
        release(&e->c);
        delete e;
        return st;
    }
    *ep = e;
    return QMOE_OK;
}

int qmoe_ep_is_direct(const qmoe_ep* ep) { return ep && ep->c.direct ? 1 : 0; }

int qmoe_ep_forward(qmoe_ep* ep, const qmoe_block* layer, const qmoe_block* local, const int32_t* placement,
                    const float* x, const float* norm_weight, float eps, const float* residual, float* out, int T,
                    qmoe_stream_t stream) {
    if (!ep || !layer || !local || !x || !out || T <= 8) return QMOE_ERR_ARG;
    return forward_impl(&ep->c, layer, local, placement, x, norm_weight, eps, residual, out, T,
                        reinterpret_cast<cudaStream_t>(stream));
}

int qmoe_ep_finalize(qmoe_ep* ep) {
    if (!ep) return QMOE_ERR_ARG;
    release(&ep->c);
    delete ep;
    return QMOE_OK;
}

}  // extern "C"
