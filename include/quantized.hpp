// GGUF tensor types and the non-owning tensor view of the MoE boundary.
// Drop-in for the reference's include/quantized.hpp:12-105: the same names,
// enum values and helpers (the values are GGUF format ids and block geometry,
// so they have to match the files the loader reads).
#ifndef QWEN_QUANTIZED_HPP
#define QWEN_QUANTIZED_HPP

#include <cstdint>
#include <limits>
#include <string>
#include <vector>

namespace qwen {

enum class GgmlType : uint32_t {
    F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q8_1 = 9,
    Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, Q8_K = 15,
    IQ2_XXS = 16, IQ2_XS = 17, IQ3_XXS = 18, I8 = 24, I16 = 25, I32 = 26, F64 = 28, BF16 = 30,
    COUNT
};

// A tensor of the loaded model.  device_ptr is owned by the loader; the MoE
// layer and the GEMV only read through it.
struct QuantTensor {
    std::string name;
    GgmlType type;
    std::vector<int64_t> shape;
    uint64_t num_elements;
    uint64_t size_bytes;
    uint64_t offset;              // byte offset in the GGUF payload
    void* device_ptr = nullptr;   // device copy of the payload
    uint32_t layout = 0;          // byte layout of device_ptr (qmoe_layout: 0 = the GGUF blocks as
                                  // uploaded; set by repack_tensor, include/matmul_q4.hpp)
};

namespace detail {
struct TypeGeom { uint32_t elems, bytes; };  // elements and bytes per block
inline TypeGeom type_geom(GgmlType t) {
    switch (t) {
        case GgmlType::F32: return {1, 4};
        case GgmlType::F16: case GgmlType::BF16: return {1, 2};
        case GgmlType::Q4_0: return {32, 18};
        case GgmlType::Q4_1: return {32, 20};
        case GgmlType::Q5_0: return {32, 22};
        case GgmlType::Q5_1: return {32, 24};
        case GgmlType::Q8_0: return {32, 34};
        case GgmlType::Q8_1: return {32, 36};
        case GgmlType::Q2_K: return {256, 82};
        case GgmlType::Q3_K: return {256, 110};
        case GgmlType::Q4_K: return {256, 144};
        case GgmlType::Q5_K: return {256, 176};
        case GgmlType::Q6_K: return {256, 210};
        case GgmlType::Q8_K: return {256, 292};
        case GgmlType::I8: return {1, 1};
        case GgmlType::I16: return {1, 2};
        case GgmlType::I32: return {1, 4};
        default: return {0, 0};
    }
}
}  // namespace detail

// Elements per block (0 for types without a block layout here).
inline uint64_t ggml_type_block_size(GgmlType type) { return detail::type_geom(type).elems; }

// Bytes per block.
inline uint64_t ggml_type_size(GgmlType type) { return detail::type_geom(type).bytes; }

// Payload bytes of num_elements elements; 0 when the count is not a whole
// number of blocks, the type is unknown, or the product overflows.
inline uint64_t calculate_tensor_bytes(GgmlType type, uint64_t num_elements) {
    const uint64_t be = ggml_type_block_size(type), bb = ggml_type_size(type);
    if (be == 0 || bb == 0 || num_elements % be != 0) return 0;
    const uint64_t nb = num_elements / be;
    if (nb > std::numeric_limits<uint64_t>::max() / bb) return 0;
    return nb * bb;
}

}  // namespace qwen

#endif  // QWEN_QUANTIZED_HPP
