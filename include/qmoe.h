/*
 * qmoe.h -- C-ABI of the B200 MoE block (router, dispatch, grouped expert
 * products, shared expert, combine) for Qwen3.5-35B-A3B-shaped layers.
 *
 * Plain pointers and sizes only.  Every tensor/activation pointer is a DEVICE
 * pointer; every call is asynchronous on the given CUDA stream (NULL = legacy
 * default stream) and returns a status code; no C++ exception crosses this
 * boundary.  The C++ headers include/quantized.hpp, include/matmul_q4.hpp and
 * include/layer_moe.hpp wrap these calls with the reference's interfaces and
 * turn status codes back into std::runtime_error.
 *
 * Reference interfaces replaced (sahan974/qwen-3.5-cuda, file:line):
 *   qmoe_type_supported   include/matmul_q4.hpp:10   matmul_type_supported
 *   qmoe_gemv             include/matmul_q4.hpp:13-21 matmul_dispatch
 *   qmoe_gemv_exact       src/cuda/matmul_q4.cu:140-167 gemv_kernel (same
 *                         operation order, bit-identical output)
 *   qmoe_dequant_row      include/matmul_q4.hpp:24-30 dequantize_row
 *   qmoe_repack           src/loader_gguf.cpp:322-381 (an optional repack step
 *                         after a tensor's upload; the reference uploads raw)
 *   qmoe_router_topk      src/layer_moe.cpp:98-99     router GEMV + moe_topk
 *                         (src/cuda/moe.cu:7-57), plus the host checks of
 *                         src/layer_moe.cpp:102-124 moved onto the device
 *   qmoe_dispatch         no counterpart (the reference is single-token)
 *   qmoe_expert_gateup    src/layer_moe.cpp:131-135, 147-149 (gate/up GEMVs,
 *                         moe_silu_mul) for all routed pairs + shared expert
 *   qmoe_expert_block     src/layer_moe.cpp:127-154 (all expert work after routing)
 *   qmoe_ep_*             no counterpart (expert parallelism across GPUs)
 *   qmoe_down_combine     src/layer_moe.cpp:138-141, 150-154 (down GEMVs,
 *                         moe_add, moe_shared_add, final copy)
 *   qmoe_block_forward    src/layer_moe.cpp:82-155   MoeLayer::forward, for
 *                         T >= 1 tokens at once
 *   qmoe_stack_forward    src/model.cpp:193-212 layer loop (MoE halves, rmsnorm
 *                         :208 and residual_add :211 fused), for T tokens at
 *                         once instead of src/main.cpp:391-393's one per call
 *   qmoe_workspace_size   src/layer_moe.cpp:51-78    MoeLayer::init buffers
 */
#ifndef QMOE_H
#define QMOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QMOE_API __attribute__((visibility("default")))
#else
#define QMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; spelled out so this header needs no CUDA header. */
typedef struct CUstream_st* qmoe_stream_t;

/* Status codes.  Host-side argument checks mirror the reference's exceptions. */
enum qmoe_status {
    QMOE_OK = 0,
    QMOE_ERR_ARG = 1,            /* null / not-loaded tensor (matmul_q4.cu:187-189) or bad argument */
    QMOE_ERR_TYPE = 2,           /* unsupported GGML type (matmul_q4.cu:190-192) */
    QMOE_ERR_SHAPE = 3,          /* shape exceeds tensor (matmul_q4.cu:193-195, :215-217) */
    QMOE_ERR_ALIGN = 4,          /* device pointer not 16-byte aligned */
    QMOE_ERR_WORKSPACE = 5,      /* workspace missing or too small */
    QMOE_ERR_UNSUPPORTED = 6,    /* dimensions outside what the kernels support */
    QMOE_ERR_CUDA = 7,           /* CUDA runtime / launch error */
    QMOE_ERR_ROUTING = 10,       /* device error word: invalid or non-finite routing (layer_moe.cpp:116-118) */
    QMOE_ERR_NOT_NORMALIZED = 11,/* device error word: route weights not normalised (layer_moe.cpp:122-124) */
    QMOE_ERR_TIMEOUT = 12,       /* device error word: a bounded device-side wait gave up */
    QMOE_ERR_COMM = 13           /* collective communication (NCCL) error: include/qmoe_ep.h */
};

/* Non-owning view of one GGUF tensor on the device (reference QuantTensor,
 * include/quantized.hpp:38-46: device_ptr, type, num_elements). */
typedef struct qmoe_tensor {
    const void* data;       /* device pointer to the raw GGUF payload, 16-byte aligned */
    uint32_t ggml_type;     /* GgmlType id (include/quantized.hpp:12-36) */
    uint32_t layout;        /* QMOE_LAYOUT_GGUF (0): the GGUF bytes in place; other values:
                               a repacked copy made by qmoe_repack */
    uint64_t num_elements;  /* logical element count */
} qmoe_tensor;

/* Byte layouts of a tensor's payload (qmoe_tensor.layout). */
enum qmoe_layout {
    QMOE_LAYOUT_GGUF = 0,     /* the GGUF blocks as stored in the file, read in place */
    QMOE_LAYOUT_Q6K_A16 = 1   /* Q6_K only: each 210-byte super-block in a 224-byte slot
                                 (14 zero bytes after it), so every block starts on a
                                 16-byte boundary; read by qmoe_gemv */
};

/* MoE dimensions (reference ModelConfig MoE fields, include/config.hpp:33-37). */
typedef struct qmoe_dims {
    int32_t d_model;        /* hidden size (2048) */
    int32_t num_experts;    /* routed experts E (256) */
    int32_t top_k;          /* experts per token k (8) */
    int32_t expert_dim;     /* routed expert FFN dim F (512) */
    int32_t shared_dim;     /* shared expert FFN dim Fs */
} qmoe_dims;

/* The eight tensors of one MoE block, named as in model.cpp:140-147. */
typedef struct qmoe_block {
    qmoe_tensor router;          /* ffn_gate_inp.weight        {d, E}     F32 */
    qmoe_tensor gate_exps;       /* ffn_gate_exps.weight       {d, F, E}       */
    qmoe_tensor up_exps;         /* ffn_up_exps.weight         {d, F, E}       */
    qmoe_tensor down_exps;       /* ffn_down_exps.weight       {F, d, E}       */
    qmoe_tensor shared_gate_inp; /* ffn_gate_inp_shexp.weight  {d}        F32 */
    qmoe_tensor shared_gate;     /* ffn_gate_shexp.weight      {d, Fs}         */
    qmoe_tensor shared_up;       /* ffn_up_shexp.weight        {d, Fs}         */
    qmoe_tensor shared_down;     /* ffn_down_shexp.weight      {Fs, d}         */
    const float* expert_bias;    /* optional device F32[E] added to the router logits before
                                    selection (no counterpart in the reference; used by the
                                    uneven-routing benchmark); NULL = none */
} qmoe_block;

/* Named buffers inside a block workspace (see qmoe_ws_view). */
enum qmoe_ws_buffer {
    QMOE_WS_LOGITS = 0,   /* float [T][E+1]; column E holds the shared-expert gate logit */
    QMOE_WS_TOPK_IDX = 1, /* int32 [T][k], selection order */
    QMOE_WS_TOPK_W = 2,   /* float [T][k] */
    QMOE_WS_OFFSETS = 3,  /* int32 [E+1] first pair of each expert in the permutation */
    QMOE_WS_PERM = 4,     /* int32 [T*k]  pair p = t*k + j at each permuted position */
    QMOE_WS_INV_PERM = 5, /* int32 [T*k]  permuted position of each pair (-1: invalid) */
    QMOE_WS_HIDDEN = 6,   /* float [T*k + T][max(F,Fs)] silu(gate)*up: routed pairs, then shared per token */
    QMOE_WS_ERROR = 7,    /* uint32 [4]: error flags, first failing token, spare */
    QMOE_WS_INPUT = 8,    /* float [T][d] the block input as the router saw it (after the fused norm) */
    QMOE_WS_INPUT16 = 9   /* fp16 [T][d] the same input for the tensor cores (T > 8 only), each
                             8-element chunk stored in the order 0,2,1,3,4,6,5,7 */
};

/* ABI version of this header (bumped on any incompatible change). */
QMOE_API int qmoe_abi_version(void);
/* Static text for a status code. */
QMOE_API const char* qmoe_status_string(int status);

/* 1 if GGML type `ggml_type` is accepted by qmoe_gemv / qmoe_dequant_row
 * (F32, F16, BF16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K), else 0. */
QMOE_API int qmoe_type_supported(uint32_t ggml_type);

/* y[M] = rows [element_offset/K, element_offset/K + M) of W times x[K].
 * Q4_K / Q5_K / Q6_K / Q8_0 rows with K = 256 * 2^j <= 4096 (and x 16-byte
 * aligned) stream through shared memory with bulk copies and are decoded a
 * 64-element unit at a time against 24-bit fixed-point planes of x: F32-level
 * accuracy (~2^-22 relative), but not the reference's summation order.  Other
 * types and shapes take the qmoe_gemv_exact path. */
QMOE_API int qmoe_gemv(const qmoe_tensor* w, const float* x, float* y, int M, int K,
              uint64_t element_offset, qmoe_stream_t stream);

/* The same product in the reference GEMV's exact F32 operation order
 * (src/cuda/matmul_q4.cu:140-167: per-thread FMA chains over k = t + 256 i,
 * then the warp and block shuffle trees), one warp per row: bit-identical to
 * the reference kernel's output. */
QMOE_API int qmoe_gemv_exact(const qmoe_tensor* w, const float* x, float* y, int M, int K,
              uint64_t element_offset, qmoe_stream_t stream);

/* Load-time repack (the GGUF loader's upload, src/loader_gguf.cpp:322-381,
 * may call it once per tensor): bytes of a tensor of `ggml_type` and
 * `num_elements` in `layout` (0 if that layout does not apply to the type),
 * and the copy of src (GGUF layout) into dst in `layout`.  Only
 * QMOE_LAYOUT_Q6K_A16 of Q6_K tensors is defined: +6.7% bytes, and
 * qmoe_gemv's unit decoder reads aligned 16-byte words instead of two reads
 * and a funnel shift per word.  The block entry points take GGUF layouts only
 * (QMOE_ERR_UNSUPPORTED otherwise). */
QMOE_API uint64_t qmoe_repack_bytes(uint32_t ggml_type, uint64_t num_elements, uint32_t layout);
QMOE_API int qmoe_repack(const qmoe_tensor* src, uint32_t layout, void* dst, size_t dst_bytes,
                         qmoe_stream_t stream);

/* out[cols] = elements [row*cols, row*cols + cols) of W, dequantised to F32. */
QMOE_API int qmoe_dequant_row(const qmoe_tensor* w, float* out, int row, int cols, qmoe_stream_t stream);

/* Device workspace bytes needed by the block entry points for up to
 * `max_tokens` tokens per call; 0 if the dimensions are unsupported. */
QMOE_API size_t qmoe_workspace_size(const qmoe_dims* dims, int max_tokens);

/* Device pointer to a named buffer inside `workspace` for a call of T tokens. */
QMOE_API void* qmoe_ws_view(void* workspace, const qmoe_dims* dims, int T, int which);

/* Router logits (reference reduction order, so expert ids are bit-identical),
 * optional expert bias, top-k selection + softmax over the selected logits,
 * on-device validation, and the token->expert permutation.  Results stay in
 * the workspace (QMOE_WS_*); `topk_idx`/`topk_w` (optional, device) receive
 * copies.  Routing errors are recorded in the device error word. */
QMOE_API int qmoe_router_topk(const qmoe_block* blk, const qmoe_dims* dims, const float* x, int T,
                     int32_t* topk_idx, float* topk_w,
                     void* workspace, size_t workspace_bytes, qmoe_stream_t stream);

/* Stable token->expert permutation of a top-k result: pairs p = t*k + j are
 * ordered by (expert, t, j).  offsets[E+1], perm[T*k], inv_perm[T*k] (device). */
QMOE_API int qmoe_dispatch(const int32_t* topk_idx, int T, int k, int E,
                  int32_t* offsets, int32_t* perm, int32_t* inv_perm,
                  void* workspace, size_t workspace_bytes, qmoe_stream_t stream);

/* The permutation of qmoe_dispatch with nothing to allocate and no workspace
 * argument.  No counterpart in the reference.  It is meant for callers that
 * cannot hand the library device memory: a serving engine that reserves all
 * of its device memory in pools at start-up and allows no allocation on the
 * token path, or a binding layer (ctypes, cgo, JNI) with no place to keep a
 * device buffer between calls.
 * Its scratch is a fixed array inside the library, 32 KiB per device, which
 * limits it to num_experts <= 256; larger E returns QMOE_ERR_UNSUPPORTED.
 * Nothing has to start at zero: every call clears the scratch it uses.
 * Every call looks up the scratch's address in the current device context
 * (cudaGetSymbolAddress, a host-side query that allocates nothing); make the
 * first call on a device before capturing a stream, since the library's
 * module is loaded on that device by the first call.  All calls on a device
 * share the scratch, so two calls that
 * overlap in time race: order them on one stream, or synchronise between
 * streams. */
QMOE_API int qmoe_dispatch_noalloc(const int32_t* topk_idx, int T, int k, int E,
                          int32_t* offsets, int32_t* perm, int32_t* inv_perm, qmoe_stream_t stream);

/* Gate/up products of every routed (token, expert) pair and of the shared
 * expert, fused with silu(gate)*up, for the routing in the workspace. */
QMOE_API int qmoe_expert_gateup(const qmoe_block* blk, const qmoe_dims* dims, const float* x, int T,
                       void* workspace, size_t workspace_bytes, qmoe_stream_t stream);

/* Down products of every routed pair and of the shared expert, combined per
 * token in selection order j = 0..k-1, then + sigmoid(shared gate) * shared:
 * out[t] = (residual ? residual[t] : 0) + moe(x[t]). */
QMOE_API int qmoe_down_combine(const qmoe_block* blk, const qmoe_dims* dims, int T,
                      float* out, const float* residual,
                      void* workspace, size_t workspace_bytes, qmoe_stream_t stream);

/* expert_gateup + down_combine in one step for the routing the workspace holds
 * (after qmoe_router_topk, T <= 8): for up to 4 tokens a single fused launch
 * -- gate/up items, a device-wide barrier, down rows, combine -- where the
 * weight types have a fused instance, else (and for 5-8 tokens) the two
 * kernels.  Same result as the two calls. */
QMOE_API int qmoe_expert_block(const qmoe_block* blk, const qmoe_dims* dims, int T,
                      float* out, const float* residual,
                      void* workspace, size_t workspace_bytes, qmoe_stream_t stream);

/* Expert parallelism for prefill (experts sharded contiguously over G ranks,
 * E/G per rank; the caller moves buffers between ranks, e.g. with NCCL
 * all-to-all).  No counterpart in the reference, which runs on one GPU.
 * Per rank, for T > 8 local tokens:
 *   qmoe_ep_route     x_in (optional pre-MoE RMSNorm), its fp16 copy
 *                     (QMOE_WS_INPUT16) and the top-k of every local token
 *                     (QMOE_WS_TOPK_IDX / QMOE_WS_TOPK_W), in `workspace`
 *   qmoe_ep_dispatch  send buffers from that routing: one fp16 row per
 *                     (token, rank) pair that has at least one expert on the
 *                     rank -- grouped by rank, token order inside a rank --
 *                     with a meta row of k ints (slot j: the expert's id local
 *                     to that rank, or -1); counts[r] = rows to rank r,
 *                     counts[G + r] = (token, slot) pairs to rank r; and
 *                     pair_pos[t*k + j] = the position of pair (t, j) in the
 *                     returned outputs (grouped by rank; inside a rank in
 *                     (row, slot) order), -1 for a failed token
 *   qmoe_ep_experts   this rank's experts on n received rows and meta rows
 *                     (any concatenation of the ranks' chunks): y_pairs
 *                     [n_pairs][d] fp16 = down(silu(gate x) * up x) for every
 *                     valid slot, in (row, slot) order -- the order that
 *                     pair_pos on the sending rank refers to; n_pairs = the
 *                     valid slots of the rows (the senders' pair counts)
 *   qmoe_ep_combine   shared expert and combine of the T local tokens:
 *                     out[t] = residual[t] + sum_j w[t][j] y[pair_pos[t*k+j]]
 *                              + sigmoid(shared gate) * shared(x_in[t])
 * placement (device int32 [E], optional): expert e lives on rank
 * placement[e] / (E/G) as local expert placement[e] % (E/G) -- a permutation
 * of 0..E-1 that balances expected load; NULL = contiguous shards (rank r owns
 * experts r*E/G .. (r+1)*E/G - 1).
 * send_rows holds at most T * min(G, k) rows (send_meta the same number of
 * k-int rows); `scratch` comes from qmoe_ep_dispatch_scratch_size.  local_blk
 * holds the rank's slices of the expert tensors (router and shared tensors are
 * not read), local_dims its expert count (top_k = the layer's k); the
 * workspace of qmoe_ep_experts comes from qmoe_ep_rows_workspace_size. */
QMOE_API int qmoe_ep_route(const qmoe_block* blk, const qmoe_dims* dims, const float* x, const float* norm_weight,
                   float eps, int T, void* workspace, size_t workspace_bytes, qmoe_stream_t stream);
QMOE_API size_t qmoe_ep_dispatch_scratch_size(int T, int G);
QMOE_API int qmoe_ep_dispatch(const qmoe_dims* dims, int T, int G, const int32_t* placement, void* workspace,
                      size_t workspace_bytes, void* send_rows, int32_t* send_meta, int32_t* counts,
                      int32_t* pair_pos, void* scratch, size_t scratch_bytes, qmoe_stream_t stream);
QMOE_API size_t qmoe_ep_rows_workspace_size(const qmoe_dims* local_dims, int max_rows);
QMOE_API int qmoe_ep_experts(const qmoe_block* local_blk, const qmoe_dims* local_dims, const void* x16_rows,
                     const int32_t* meta, int n_rows, int n_pairs, void* y_pairs, void* workspace,
                     size_t workspace_bytes, qmoe_stream_t stream);

/* Direct return of the expert outputs (expert parallelism over peer memory,
 * e.g. NVLink): instead of y_pairs, the down GEMM's epilogue stores the output
 * of received pair q (q in [pair_start[s], pair_start[s+1]) came from rank s)
 * into rank s's return buffer dst[s] at row dst_row[s] + q - pair_start[s],
 * i.e. where rank s's pair_pos expects it (dst_row[s] = the pairs rank s sends
 * to the ranks before this one).  dst[s] is a peer pointer (qmoe_peer_open),
 * this rank's own buffer for s = itself.  The caller orders the writes before
 * rank s's qmoe_ep_combine (kernel completion, then any cross-rank barrier on
 * the streams, e.g. a one-element NCCL all-reduce).  Q4_K experts only. */
typedef struct qmoe_ep_return {
    int32_t n_ranks;          /* G <= 32 */
    int32_t pair_start[33];
    void* dst[32];
    int64_t dst_row[32];
} qmoe_ep_return;
QMOE_API int qmoe_ep_experts_return(const qmoe_block* local_blk, const qmoe_dims* local_dims, const void* x16_rows,
                            const int32_t* meta, int n_rows, const qmoe_ep_return* ret, void* workspace,
                            size_t workspace_bytes, qmoe_stream_t stream);

/* Device memory another process on this node can map (CUDA IPC): allocate
 * with a 64-byte handle to hand to the peers, open a peer's handle, close an
 * opened mapping, free an allocation. */
QMOE_API int qmoe_peer_alloc(size_t bytes, void** ptr, void* handle64);
QMOE_API int qmoe_peer_open(const void* handle64, void** ptr);
QMOE_API int qmoe_peer_close(void* ptr);
QMOE_API int qmoe_peer_free(void* ptr);
/* Stream-ordered device copy (one cudaMemcpyAsync; a peer pointer from
 * qmoe_peer_open makes it a copy-engine transfer over NVLink). */
QMOE_API int qmoe_copy_async(void* dst, const void* src, size_t bytes, qmoe_stream_t stream);
QMOE_API int qmoe_ep_combine(const qmoe_block* blk, const qmoe_dims* dims, const void* y_pairs,
                     const int32_t* pair_pos, int T, const float* residual, float* out, void* workspace,
                     size_t workspace_bytes, qmoe_stream_t stream);
/* qmoe_ep_combine in two halves, so that the shared expert can run while the
 * routed outputs are still travelling: qmoe_ep_shared (needs only the
 * qmoe_ep_route workspace), then qmoe_ep_combine_routed (same arguments as
 * qmoe_ep_combine). */
QMOE_API int qmoe_ep_shared(const qmoe_block* blk, const qmoe_dims* dims, int T, void* workspace,
                    size_t workspace_bytes, qmoe_stream_t stream);
QMOE_API int qmoe_ep_combine_routed(const qmoe_block* blk, const qmoe_dims* dims, const void* y_pairs,
                            const int32_t* pair_pos, int T, const float* residual, float* out, void* workspace,
                            size_t workspace_bytes, qmoe_stream_t stream);

/* Number of kernels one qmoe_block_forward call with these arguments launches
 * (for profiling and launch accounting), assuming a workspace of
 * qmoe_workspace_size(dims, T) bytes: T > 8 with that workspace runs the
 * prefill path, a smaller one runs chunks of 8 tokens through the decode
 * kernels.  Negative status on bad arguments. */
QMOE_API int qmoe_block_kernel_count(const qmoe_block* blk, const qmoe_dims* dims, int T);

/* The whole MoE block for T tokens: router_topk, expert_gateup, down_combine.
 * x, out: device F32 [T][d_model]; residual optional (NULL). */
QMOE_API int qmoe_block_forward(const qmoe_block* blk, const qmoe_dims* dims, const float* x, float* out,
                       const float* residual, int T,
                       void* workspace, size_t workspace_bytes, qmoe_stream_t stream);

/* The MoE half of a decoder layer (model.cpp:208-211 of the reference:
 * rmsnorm_forward, MoeLayer::forward, residual_add) in the same three
 * launches: out = resid + MoE(rmsnorm(resid) * norm_weight), with the
 * reference's RMSNorm arithmetic (src/cuda/ops.cu:25-65: sum of squares in
 * the GEMV's reduction order, rsqrtf(mean + eps), (x * scale) * weight). */
QMOE_API int qmoe_block_forward_prenorm(const qmoe_block* blk, const qmoe_dims* dims, const float* resid,
                                        const float* norm_weight, float eps, float* out, int T,
                                        void* workspace, size_t workspace_bytes, qmoe_stream_t stream);

/* The MoE halves of n_layers decoder layers for a batch of T tokens, in
 * layer order (the multi-token form of the layer loop of src/model.cpp:193-212,
 * which the reference runs one token at a time from src/main.cpp:391-393):
 * for l = 0..n_layers-1:  resid <- resid + MoE_l(rmsnorm(resid) * norm_weights[l])
 * (qmoe_block_forward_prenorm per layer; T > 8 takes the tensor-core path).
 * `blocks` and `norm_weights` are host arrays of n_layers entries (device
 * pointers inside); resid [T][d] is updated in place; tmp is device scratch of
 * the same size; one workspace serves every layer (stream-ordered).  The token
 * mixing that model.cpp runs between the MoE halves is the caller's: call this
 * once per layer (n_layers = 1) with the mixer between, or for a run of
 * consecutive MoE halves. */
QMOE_API int qmoe_stack_forward(const qmoe_block* blocks, const float* const* norm_weights, int n_layers,
                                const qmoe_dims* dims, float eps, float* resid, float* tmp, int T,
                                void* workspace, size_t workspace_bytes, qmoe_stream_t stream);

/* Waits for `stream`, reads the device error word of `workspace` into
 * err[0..1] (flags, first failing token) and clears it.  Returns the status
 * the flags map to (QMOE_OK if none). */
QMOE_API int qmoe_check_errors(void* workspace, const qmoe_dims* dims, uint32_t* err, qmoe_stream_t stream);

/* Phase tracer (profiling): while a device buffer of qmoe_trace_bytes() is
 * registered, the decode kernels write %globaltimer stamps (ns) of their
 * phases into it, laid out [kernel 0..2][CTA 0..159][event 0..7] (uint64;
 * kernel 0 router, 1 gate/up, 2 down).  Later launches overwrite earlier
 * ones.  NULL disables it (the default). */
QMOE_API int qmoe_trace_enable(uint64_t* device_buffer, size_t bytes);
QMOE_API size_t qmoe_trace_bytes(void);

/* Clears the workspace control words (call once after allocating it, and
 * again after a call reported QMOE_ERR_TIMEOUT).  It also removes an error
 * sink (below). */
QMOE_API int qmoe_workspace_init(void* workspace, size_t workspace_bytes, qmoe_stream_t stream);

/* Registers a host-mapped 32-bit word (a device-accessible pointer from
 * cudaHostAlloc(..., cudaHostAllocMapped) + cudaHostGetDevicePointer) into
 * which the kernels OR the same error flags they record in the workspace
 * (1 routing, 2 weights not normalised, 4 timed-out wait, 8 misaligned copy).
 * The host can then notice a failed call by reading that word, without
 * synchronising the stream -- the reference throws from MoeLayer::forward
 * after a stream synchronisation (src/layer_moe.cpp:106-124); the shim in
 * this library throws at its next forward instead.  NULL removes the sink.
 * Stream-ordered; qmoe_workspace_init clears it. */
QMOE_API int qmoe_workspace_set_error_sink(void* workspace, uint32_t* sink, qmoe_stream_t stream);

/* Test hook for the bounded grid-barrier wait of the fused decode kernel (no
 * counterpart in the reference): later launches wait at most `wait_ns`
 * nanoseconds (0 restores the default, 200 ms) and wait for
 * `phantom_arrivals` extra CTAs that never arrive (0 = normal operation;
 * > 0 makes the wait run out, so a test can check that the kernel returns
 * and reports QMOE_ERR_TIMEOUT instead of hanging).  Process-wide; not for
 * use while other threads launch. */
QMOE_API int qmoe_debug_grid_barrier(uint64_t wait_ns, int phantom_arrivals);

/* Synthetic tensors for tests and benchmarks: elements sigma*N(0,1) from a
 * counter-based stream (seed, stream_id), encoded as `ggml_type`.  The device
 * and host versions write identical bytes. */
QMOE_API int qmoe_synth_fill(void* dst, uint32_t ggml_type, uint64_t num_elements, uint64_t seed,
                    uint64_t stream_id, float sigma, qmoe_stream_t stream);
QMOE_API int qmoe_synth_fill_host(void* dst, uint32_t ggml_type, uint64_t num_elements, uint64_t seed,
                         uint64_t stream_id, float sigma);
/* Host: elements [first_element, first_element + num_elements) of the same
 * stream (first_element a multiple of the block size), written to dst. */
QMOE_API int qmoe_synth_fill_host_range(void* dst, uint32_t ggml_type, uint64_t first_element,
                                        uint64_t num_elements, uint64_t seed, uint64_t stream_id, float sigma);
/* Bytes of a GGML tensor of `num_elements` elements (quantized.hpp:98-105), 0 if invalid. */
QMOE_API uint64_t qmoe_tensor_bytes(uint32_t ggml_type, uint64_t num_elements);

#ifdef __cplusplus
}
#endif
#endif /* QMOE_H */
