// Test stand-in for the reference project's include/cuda_utils.hpp: the
// CUDA_CHECK macro and a CudaContext owning one stream (reference
// cuda_utils.hpp:30-38, 51-87, without the cuBLAS handle).  In the reference
// project its own cuda_utils.hpp is used instead.
#pragma once
#include <cuda_runtime.h>
#include <stdexcept>
#include <string>
#define CUDA_CHECK(call)                                                                              \
    do {                                                                                              \
        cudaError_t err_ = (call);                                                                    \
        if (err_ != cudaSuccess) throw std::runtime_error("CUDA Error: " + std::string(cudaGetErrorString(err_))); \
    } while (0)
namespace qwen {
class CudaContext {
public:
    CudaContext() { CUDA_CHECK(cudaStreamCreate(&stream_)); }
    ~CudaContext() { if (stream_) cudaStreamDestroy(stream_); }
    CudaContext(const CudaContext&) = delete;
    CudaContext& operator=(const CudaContext&) = delete;
    cudaStream_t stream() const { return stream_; }
    void synchronize() const { CUDA_CHECK(cudaStreamSynchronize(stream_)); }
private:
    cudaStream_t stream_ = nullptr;
};
}  // namespace qwen
