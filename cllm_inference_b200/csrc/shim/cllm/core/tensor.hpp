// Tensor descriptor with the reference's layout (cllm_inference
// include/cllm/core/tensor.hpp:10-30): shape in GGUF order, type, a pointer
// into the read-only model mapping and the file offset.  dequantize() and
// dequantize_f16() are defined by libcllm_quant.so and run on the GPU.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include "cllm/core/quant.hpp"

namespace cllm {

struct Tensor {
    std::vector<uint32_t> shape;
    GgmlType type = GgmlType::F32;
    const void* data = nullptr;
    uint64_t offset = 0;

    uint64_t numel() const {
        uint64_t n = 1;
        for (auto d : shape) n *= d;
        return n;
    }

    std::vector<float> dequantize() const;
    std::vector<uint16_t> dequantize_f16() const;
};

}  // namespace cllm
