// Quantised GEMV and row dequantisation.  Drop-in for the reference's
// include/matmul_q4.hpp:10-30 (same declarations); the definitions in
// qwen-3.5-cuda_b200/cpp/matmul_q4_shim.cpp call qmoe_gemv /
// qmoe_dequant_row (include/qmoe.h) and throw std::runtime_error with the
// reference's messages (src/cuda/matmul_q4.cu:187-195, 210-217).
#ifndef QWEN_MATMUL_Q4_HPP
#define QWEN_MATMUL_Q4_HPP

#include <cuda_runtime.h>
#include "quantized.hpp"

namespace qwen {

// True for every type the GEMV reads (F32, F16, BF16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K).
bool matmul_type_supported(GgmlType type);

// y[0..M) = rows [element_offset/K, element_offset/K + M) of weight times x[0..K),
// asynchronous on `stream`.
void matmul_dispatch(const QuantTensor& weight, const float* x, float* y, int M, int K,
                     cudaStream_t stream = nullptr, uint64_t element_offset = 0);

// out[0..cols) = row `row` of tensor, dequantised to F32, asynchronous on `stream`.
void dequantize_row(const QuantTensor& tensor, float* out, int row, int cols, cudaStream_t stream = nullptr);

// Optional load-time repack (no counterpart in the reference, whose loader
// uploads every tensor as stored, src/loader_gguf.cpp:322-381): for a Q6_K
// tensor read only by matmul_dispatch (the LM head of Q4_K_M models, for
// example), moves its super-blocks into 16-byte-aligned 224-byte slots
// (qmoe_repack, QMOE_LAYOUT_Q6K_A16): a new cudaMalloc allocation replaces
// device_ptr (the old one is freed; the loader's unload frees the new one),
// size_bytes and layout are updated.  Other types are left as they are.
// Returns true if the tensor was repacked.  Synchronises `stream`.
bool repack_tensor(QuantTensor& tensor, cudaStream_t stream = nullptr);

}  // namespace qwen

#endif  // QWEN_MATMUL_Q4_HPP
