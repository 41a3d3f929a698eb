// Force-included (-include) ahead of the reference's sources when they are
// compiled into oracle/_ref/.  The reference's include/cuda_utils.hpp does not
// compile as shipped (its multi-line CUDA_CHECK/CUBLAS_CHECK macros lost their
// line continuations, include/cuda_utils.hpp:30-48).  Defining its include
// guard here makes that header a no-op and supplies the three names the MoE
// path uses from it -- CUDA_CHECK, CudaContext::stream() -- with the same
// meaning (throw std::runtime_error on a CUDA error; one stream per context).
// TEST INFRASTRUCTURE ONLY: used to run the reference as a parity oracle.
#ifndef QWEN_CUDA_UTILS_HPP
#define QWEN_CUDA_UTILS_HPP
#include <cuda_runtime.h>
#include <stdexcept>
#include <string>

#define CUDA_CHECK(call)                                                              \
    do {                                                                              \
        cudaError_t qref_err_ = (call);                                               \
        if (qref_err_ != cudaSuccess)                                                 \
            throw std::runtime_error(std::string("CUDA Error: ") +                    \
                                     cudaGetErrorString(qref_err_));                  \
    } while (0)

namespace qwen {
class CudaContext {
public:
    explicit CudaContext(cudaStream_t s) : stream_(s) {}
    CudaContext(const CudaContext&) = delete;
    CudaContext& operator=(const CudaContext&) = delete;
    cudaStream_t stream() const { return stream_; }
    void synchronize() const { CUDA_CHECK(cudaStreamSynchronize(stream_)); }
private:
    cudaStream_t stream_;
};
}  // namespace qwen
#endif
