// Definitions of include/matmul_q4.hpp over the C-ABI (include/qmoe.h).
// Error behaviour follows src/cuda/matmul_q4.cu:185-217 of the reference:
// std::runtime_error with the same messages; CUDA launch failures as the
// reference's CUDA_CHECK reports them ("CUDA Error: ...").
#include "matmul_q4.hpp"

#include <stdexcept>
#include <string>

#include "qmoe.h"

namespace qwen {
namespace {

qmoe_tensor view(const QuantTensor& t) {
    qmoe_tensor v{};
    v.data = t.device_ptr;
    v.ggml_type = static_cast<uint32_t>(t.type);
    v.num_elements = t.num_elements;
    v.layout = t.layout;
    return v;
}

void raise_status(int st, const char* what) {
    if (st == QMOE_ERR_CUDA) throw std::runtime_error(std::string("CUDA Error: ") + qmoe_status_string(st));
    throw std::runtime_error(std::string(what) + ": " + qmoe_status_string(st));
}

}  // namespace

bool matmul_type_supported(GgmlType type) { return qmoe_type_supported(static_cast<int>(type)) != 0; }

void matmul_dispatch(const QuantTensor& w, const float* x, float* y, int M, int K, cudaStream_t stream,
                     uint64_t element_offset) {
    if (!w.device_ptr) throw std::runtime_error("tensor '" + w.name + "' is not loaded");
    if (!matmul_type_supported(w.type)) throw std::runtime_error("unsupported GGML type for tensor '" + w.name + "'");
    const qmoe_tensor v = view(w);
    const int st = qmoe_gemv(&v, x, y, M, K, element_offset, stream);
    if (st == QMOE_ERR_SHAPE) throw std::runtime_error("GEMV shape exceeds tensor '" + w.name + "'");
    if (st != QMOE_OK) raise_status(st, "matmul_dispatch");
}

void dequantize_row(const QuantTensor& t, float* out, int row, int cols, cudaStream_t stream) {
    if (!t.device_ptr || !matmul_type_supported(t.type))
        throw std::runtime_error("cannot dequantize tensor '" + t.name + "'");
    const qmoe_tensor v = view(t);
    const int st = qmoe_dequant_row(&v, out, row, cols, stream);
    if (st == QMOE_ERR_SHAPE) throw std::runtime_error("row is outside tensor '" + t.name + "'");
    if (st != QMOE_OK) raise_status(st, "dequantize_row");
}

bool repack_tensor(QuantTensor& t, cudaStream_t stream) {
    if (!t.device_ptr) throw std::runtime_error("tensor '" + t.name + "' is not loaded");
    if (t.type != GgmlType::Q6_K || t.layout != QMOE_LAYOUT_GGUF) return false;
    const uint64_t n = qmoe_repack_bytes(static_cast<uint32_t>(t.type), t.num_elements, QMOE_LAYOUT_Q6K_A16);
    if (n == 0) return false;
    void* dst = nullptr;
    if (cudaMalloc(&dst, n) != cudaSuccess) throw std::runtime_error("CUDA Error: out of memory repacking '" + t.name + "'");
    const qmoe_tensor v = view(t);
    const int st = qmoe_repack(&v, QMOE_LAYOUT_Q6K_A16, dst, n, stream);
    if (st != QMOE_OK || cudaStreamSynchronize(stream) != cudaSuccess) {
        cudaFree(dst);
        raise_status(st != QMOE_OK ? st : QMOE_ERR_CUDA, "repack_tensor");
    }
    cudaFree(t.device_ptr);
    t.device_ptr = dst;
    t.size_bytes = n;
    t.layout = QMOE_LAYOUT_Q6K_A16;
    return true;
}

}  // namespace qwen
