// TMA-fed grouped Q4_K expert GEMM (k_tgemm.cu): parameters and launchers.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace qmoe {

// MODE 1 outputs sent to the ranks that own the rows (expert parallelism):
// row q of the received pairs, q in [start[s], start[s+1]), goes to
// dst[s] + (dst_row[s] + q - start[s]) * N.  n_src = 0: rows go to `out`.
struct TgScatter {
    int n_src;
    int32_t start[33];
    __half* dst[32];
    int64_t dst_row[32];
};

struct TgParams {
    int N, K;                   // output columns (F or d), reduction length
    int groups;                 // experts (1 for the shared expert)
    int group_rows;             // weight rows per group (F for gate/up, d for down)
    const int32_t* grp_start;   // [groups + 1] first A row of each group
    const int32_t* tile_start;  // [groups + 1] prefix of 128-row tiles per group
    __half* out;                // [rows][N] fp16; MODE 0 in the chunk element order
    const int32_t* out_rows;    // output row of each A row (null: the same row)
    int out_cap;                // rows of `out` (rows mapped past it are not written)
    uint32_t* ctrl;             // error word
    TgScatter sc;               // MODE 1 only
};

struct TgArgs {
    int mode;           // 0: gate/up (silu(gate) * up), 1: down
    const __half* a16;  // A rows [a_rows][K] fp16, chunk element order, contiguous per group
    uint64_t a_rows;    // rows of A the tensor map covers
    const void* w0;     // gate (mode 0) or down (mode 1): Q4_K rows of K elements
    const void* w1;     // up (mode 0)
    int K;
    TgParams p;
};

bool tgemm_supported(int wtype, int mode, int N, int K);
cudaError_t launch_tgemm(const TgArgs& a, cudaStream_t s);
cudaError_t launch_gather_rows(const __half* src, const int32_t* idx, const int32_t* n_rows, int cap, int d,
                               __half* dst, cudaStream_t s);

}  // namespace qmoe
