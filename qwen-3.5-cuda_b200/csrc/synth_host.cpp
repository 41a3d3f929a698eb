// Host side of the synthetic tensor generator (compiled with
// -ffp-contract=off so that it matches k_synth.cu byte for byte).
#include <cstdint>
#include "qmoe_synth.h"
#include "../../include/qmoe.h"

extern "C" int qmoe_synth_fill_host_range(void* dst, uint32_t type, uint64_t first, uint64_t n, uint64_t seed,
                                          uint64_t stream_id, float sigma) {
    const int be = qs_block_elems(static_cast<int>(type));
    const int bb = qs_block_bytes(static_cast<int>(type));
    if (!dst || be == 0 || n % static_cast<uint64_t>(be) || first % static_cast<uint64_t>(be)) return QMOE_ERR_ARG;
    const uint64_t b0 = first / static_cast<uint64_t>(be);
    const uint64_t key = qs_stream_key(seed, stream_id);
    const int64_t nb = static_cast<int64_t>(n / be);
    uint8_t* out = static_cast<uint8_t*>(dst);
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; ++b) qs_gen_block(static_cast<int>(type), key, sigma, b0 + static_cast<uint64_t>(b), out + b * bb);
    return QMOE_OK;
}

extern "C" int qmoe_synth_fill_host(void* dst, uint32_t type, uint64_t n, uint64_t seed, uint64_t stream_id,
                                    float sigma) {
    return qmoe_synth_fill_host_range(dst, type, 0, n, seed, stream_id, sigma);
}
