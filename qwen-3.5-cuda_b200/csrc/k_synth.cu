// Device generation of synthetic GGUF tensors (tests and benchmarks).  One
// thread per GGML block; the block encoders of qmoe_synth.h are written so
// that host and device produce identical bytes.
#include "qmoe_synth.h"
#include "qmoe_internal.h"

namespace qmoe {

__global__ void k_synth(uint8_t* dst, int type, uint64_t nblocks, uint64_t key, float sigma) {
    const int bb = qs_block_bytes(type);
    for (uint64_t b = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; b < nblocks;
         b += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        uint8_t tmp[256];
        qs_gen_block(type, key, sigma, b, tmp);
        uint8_t* o = dst + b * bb;
        for (int i = 0; i < bb; ++i) o[i] = tmp[i];
    }
}

cudaError_t launch_synth(void* dst, int type, uint64_t nblocks, uint64_t seed, uint64_t stream_id, float sigma,
                         cudaStream_t s) {
    const uint64_t key = qs_stream_key(seed, stream_id);
    const int threads = 128;
    uint64_t blocks = (nblocks + threads - 1) / threads;
    if (blocks > 148ull * 64) blocks = 148ull * 64;
    if (blocks == 0) return cudaSuccess;
    k_synth<<<static_cast<unsigned>(blocks), threads, 0, s>>>(static_cast<uint8_t*>(dst), type, nblocks, key, sigma);
    return cudaGetLastError();
}

}  // namespace qmoe
