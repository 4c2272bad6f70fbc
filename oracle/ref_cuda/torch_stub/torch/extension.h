// torch/extension.h stand-in for compiling the reference's sampling and optimizer sources without libtorch
// (TEST INFRASTRUCTURE ONLY). Those files hold the reference's CUDA kernels next to host wrappers that take
// torch::Tensor arguments; oracle/ref_cuda/ref_sampling.cu includes them to launch the kernels directly, so the
// wrappers only have to compile. Every member here is a placeholder that is never executed: the checker's own
// launchers replace the wrappers.
#pragma once

#include <cstdint>
#include <cstddef>
#include <initializer_list>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

namespace torch {

enum ScalarType { kFloat, kHalf, kDouble, kInt, kLong, kByte, kBFloat16 };
enum DeviceType { kCUDA };

struct BFloat16 {
    uint16_t bits;
};

struct TensorOptions {
    TensorOptions dtype(ScalarType) const { return *this; }
    TensorOptions device(DeviceType) const { return *this; }
};

class Tensor {
public:
    bool is_cuda() const { return false; }
    bool is_contiguous() const { return false; }
    ScalarType scalar_type() const { return kFloat; }
    int64_t numel() const { return 0; }
    int64_t size(int64_t) const { return 0; }
    TensorOptions options() const { return {}; }
    void* data_ptr() const { return nullptr; }
    template <typename T>
    T* data_ptr() const { return nullptr; }
};

inline Tensor zeros(std::initializer_list<int64_t>, TensorOptions) { return {}; }
inline Tensor empty(std::initializer_list<int64_t>, TensorOptions) { return {}; }
inline Tensor zeros_like(const Tensor&) { return {}; }
inline Tensor empty_like(const Tensor&) { return {}; }
inline Tensor empty_like(const Tensor&, TensorOptions) { return {}; }

}  // namespace torch
