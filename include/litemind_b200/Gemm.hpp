// Gemm.hpp -- the reference's gemm:: kernels (include/Gemm.hpp:23-72) on device memory.
//
// Same names and argument meaning, with device pointers and a CUDA stream in place
// of the host ThreadPool.  They are not the MoE hot path (MoeLayer is); they give the
// reference's other gemm:: callers device equivalents.  Each returns the lm_status of
// the launch.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include "litemind_moe.h"

namespace litemind::b200::gemm {

/** Which kernels this build runs, for logs (the reference's gemm::kernel_description). */
inline std::string kernel_description() { return lm_kernel_description(); }

/** out = weights * input, weights row-major [out_dim, in_dim] bf16. */
inline lm_status matvec_bf16(const std::uint16_t* weights, const float* input, float* out, std::size_t out_dim,
                             std::size_t in_dim, void* stream = nullptr) {
    return lm_gemm_matvec_bf16(weights, input, out, static_cast<int64_t>(out_dim), static_cast<int64_t>(in_dim),
                               stream);
}

/** out += scale * (weights * input). */
inline lm_status matvec_bf16_accumulate(const std::uint16_t* weights, const float* input, float* out,
                                        std::size_t out_dim, std::size_t in_dim, float scale,
                                        void* stream = nullptr) {
    return lm_gemm_matvec_bf16_accumulate(weights, input, out, static_cast<int64_t>(out_dim),
                                          static_cast<int64_t>(in_dim), scale, stream);
}

/** out = weights * input for a row-major float32 matrix (the router gate). */
inline lm_status matvec_f32(const float* weights, const float* input, float* out, std::size_t out_dim,
                            std::size_t in_dim, void* stream = nullptr) {
    return lm_gemm_matvec_f32(weights, input, out, static_cast<int64_t>(out_dim), static_cast<int64_t>(in_dim),
                              stream);
}

/** destination += scale * source. */
inline lm_status axpy(float scale, const float* source, float* destination, std::size_t count,
                      void* stream = nullptr) {
    return lm_gemm_axpy(scale, source, destination, static_cast<int64_t>(count), stream);
}

/** In-place RMS normalisation, sum of squares in double. */
inline lm_status rms_norm(float* values, const float* weight, std::size_t count, float epsilon,
                          void* stream = nullptr) {
    return lm_gemm_rms_norm(values, weight, 1, static_cast<int64_t>(count), epsilon, stream);
}

/** In-place max-subtracted softmax. */
inline lm_status softmax(float* values, std::size_t count, void* stream = nullptr) {
    return lm_gemm_softmax(values, 1, static_cast<int64_t>(count), stream);
}

/** destination[i] = silu(gate[i]) * up[i]. */
inline lm_status silu_multiply(const float* gate, const float* up, float* destination, std::size_t count,
                               void* stream = nullptr) {
    return lm_gemm_silu_multiply(gate, up, destination, static_cast<int64_t>(count), stream);
}

}  // namespace litemind::b200::gemm
