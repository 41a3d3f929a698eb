/*
 * qmoe_ep.h -- expert-parallel MoE block over an NCCL communicator
 * (libqmoe_ep.so, host code over the qmoe C-ABI of include/qmoe.h).
 *
 * No counterpart in the reference, which runs one GPU (sahan974/qwen-3.5-cuda
 * src/model.cpp:209 calls MoeLayer::forward per token on one device).  This is
 * the host side of expert parallelism that a C++ caller such as model.cpp
 * links: one process per GPU, the E routed experts split over the G ranks of
 * the communicator (E/G per rank), each rank's T local tokens routed on its
 * own GPU (routing bit-identical to one GPU), their rows sent to the ranks
 * that own their experts and the expert outputs returned, then the
 * slot-ordered combine with the shared expert on the home rank.
 *
 * Per qmoe_ep_forward call, on the caller's stream:
 *   qmoe_ep_route, qmoe_ep_dispatch         (include/qmoe.h)
 *   ncclAllGather of the per-rank row/pair counts, copied to pinned host
 *   the one host synchronisation: the counts (NCCL needs the split sizes)
 *   rows + meta rows: grouped ncclSend/ncclRecv, or with QMOE_EP_DIRECT on
 *     <= 2 ranks copy-engine writes into the peers' receive buffers (CUDA IPC)
 *     and a one-element ncclAllReduce as the barrier
 *   the rank's experts on the received rows (tcgen05 grouped GEMMs):
 *     QMOE_EP_DIRECT: outputs stored into the owners' return buffers (own
 *     pairs in place, the others' staged and pushed by the copy engines on a
 *     side stream, then a barrier); else grouped send/recv of the outputs
 *   qmoe_ep_shared (while the copy engines push), qmoe_ep_combine_routed
 *     (slot order j = 0..k-1)
 * Every rank must make the same calls in the same order (NCCL); the counts
 * exchange also carries errors (a batch over max_tokens), so all ranks return
 * the same status.  No TMA or bulk load reads another GPU's memory: peer data
 * moves by copy engine or NCCL only.
 */
#ifndef QMOE_EP_H
#define QMOE_EP_H

#include "qmoe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct qmoe_ep qmoe_ep; /* opaque expert-parallel context */

enum qmoe_ep_flags {
    QMOE_EP_DIRECT = 1 /* return (and on <= 2 ranks, send) rows over CUDA IPC peer memory;
                          the experts' outputs are then stored by the down GEMM's epilogue,
                          which needs Q4_K expert tensors */
};

/* NCCL bootstrap for callers without their own communicator: rank 0 makes a
 * 128-byte id, every rank receives it out of band (e.g. a TCP store) and
 * calls qmoe_ep_comm_init with its device current. */
QMOE_API int qmoe_ep_unique_id(uint8_t id[128]);
QMOE_API int qmoe_ep_comm_init(const uint8_t id[128], int world, int rank, void** nccl_comm);
QMOE_API int qmoe_ep_comm_destroy(void* nccl_comm);

/* Context for layers of `dims` over the communicator `nccl_comm` (an
 * ncclComm_t; not owned), batches of up to max_tokens local tokens per rank.
 * Allocates every buffer the exchange needs (device, pinned host, and with
 * QMOE_EP_DIRECT the IPC buffers mapped by every peer -- if any rank cannot
 * map them, every rank falls back to the all-to-all return together).
 * Collective: all ranks call it. */
QMOE_API int qmoe_ep_init(void* nccl_comm, const qmoe_dims* dims, int max_tokens, int flags, qmoe_ep** ep);

/* 1 if the context moves data over peer memory (QMOE_EP_DIRECT took effect). */
QMOE_API int qmoe_ep_is_direct(const qmoe_ep* ep);

/* One MoE block for this rank's T local tokens (T > 8, T <= max_tokens).
 * layer: the full layer (router, shared expert; its expert tensors are not
 * read); local: this rank's experts only, as qmoe_ep_experts reads them
 * (E/G experts, local ids in placement order); placement: optional device
 * int32[E] (NULL = contiguous shards).  x, residual, out: device F32 [T][d];
 * norm_weight optional (pre-MoE RMSNorm fused into the router); residual
 * optional.  Collective: all ranks call it with their own T. */
QMOE_API int qmoe_ep_forward(qmoe_ep* ep, const qmoe_block* layer, const qmoe_block* local,
                             const int32_t* placement, const float* x, const float* norm_weight, float eps,
                             const float* residual, float* out, int T, qmoe_stream_t stream);

/* Releases the context (unmaps and frees the peer buffers; the caller's
 * communicator stays).  Call after the last forward has completed on every
 * rank (it synchronises the device first). */
QMOE_API int qmoe_ep_finalize(qmoe_ep* ep);

#ifdef __cplusplus
}
#endif

#endif /* QMOE_EP_H */
