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

}  // namespace qwen

#endif  // QWEN_MATMUL_Q4_HPP
