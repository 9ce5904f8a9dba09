// gemm_ops.cu -- the reference's gemm:: kernels (include/Gemm.hpp:23-72) on device
// memory, plus the row kernels the decoder sub-layer needs around the MoE block.
//
// These are not the MoE hot path (that is router.cu + grouped_gemm.cu); they give
// DeepSeekRunner's other callers of gemm:: (e.g. Attention, src/Attention.cpp:34-58)
// device equivalents with the same argument meaning, and the RMSNorm of the
// feed-forward sub-layer (src/Gemm.cpp:197-207, src/DeepSeekRunner.cpp:265-267).
#include <cuda_bf16.h>

#include "litemind_moe.h"
#include "moe_internal.h"

#include <algorithm>

namespace lm {
namespace {

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

template <typename W>
__device__ __forceinline__ float widen(W v);
template <>
__device__ __forceinline__ float widen<uint16_t>(uint16_t v) { return bf16_bits_to_float(v); }
template <>
__device__ __forceinline__ float widen<float>(float v) { return v; }

// Sixteen bytes of weights widened to f32, multiplied by the matching x values.
__device__ __forceinline__ float dot16(const uint16_t* w, const float* x, float acc) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(w));
    const float4 x0 = __ldg(reinterpret_cast<const float4*>(x));
    const float4 x1 = __ldg(reinterpret_cast<const float4*>(x) + 1);
    const uint32_t p[4] = {v.x, v.y, v.z, v.w};
    const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc = fmaf(__uint_as_float(p[i] << 16), xs[2 * i], acc);
        acc = fmaf(__uint_as_float(p[i] & 0xffff0000u), xs[2 * i + 1], acc);
    }
    return acc;
}
__device__ __forceinline__ float dot16(const float* w, const float* x, float acc) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(w));
    const float4 xv = __ldg(reinterpret_cast<const float4*>(x));
    acc = fmaf(v.x, xv.x, acc);
    acc = fmaf(v.y, xv.y, acc);
    acc = fmaf(v.z, xv.z, acc);
    return fmaf(v.w, xv.w, acc);
}

// One warp per output row; out[r] = (accumulate ? fmaf(scale, dot, out[r]) : dot).
// A row that starts on a 16-byte boundary (with x aligned too) is read 16 bytes per
// lane per load -- 512 contiguous bytes per warp instruction, four loads in flight --
// and its last cols % (16 / sizeof(W)) elements one by one; a row that does not
// (a ragged width such as 253) is read one element per lane per step, still
// contiguous across the warp.
template <typename W>
__global__ void __launch_bounds__(256) matvec_kernel(const W* __restrict__ w, const float* __restrict__ x,
                                                     float* __restrict__ out, int64_t rows, int64_t cols, float scale,
                                                     int accumulate) {
    constexpr int V = 16 / static_cast<int>(sizeof(W));
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const W* wr = w + row * cols;
    float acc = 0.0f;
    const bool vec = ((reinterpret_cast<uintptr_t>(wr) | reinterpret_cast<uintptr_t>(x)) & 15u) == 0;
    int64_t c0 = 0;
    if (vec) {
        const int64_t nv = cols / V;  // whole vectors in the row
        int64_t v = lane;
        float a[4] = {0.f, 0.f, 0.f, 0.f};
        for (; v + 96 < nv; v += 128) {
#pragma unroll
            for (int u = 0; u < 4; ++u) a[u] = dot16(wr + (v + 32 * u) * V, x + (v + 32 * u) * V, a[u]);
        }
        for (; v < nv; v += 32) a[0] = dot16(wr + v * V, x + v * V, a[0]);
        acc = (a[0] + a[1]) + (a[2] + a[3]);
        c0 = nv * V;
    }
    for (int64_t c = c0 + lane; c < cols; c += 32) acc = fmaf(widen(wr[c]), x[c], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) out[row] = accumulate ? fmaf(scale, acc, out[row]) : acc;
}

// Block per row: max-subtracted exponentials, f32 sum, multiply by 1/sum.
__global__ void softmax_rows_kernel(float* __restrict__ v, int64_t count) {
    __shared__ float red[32];
    float* row = v + static_cast<int64_t>(blockIdx.x) * count;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    float m = -3.402823466e38f;
    for (int64_t i = threadIdx.x; i < count; i += blockDim.x) m = fmaxf(m, row[i]);
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int i = 1; i < warps; ++i) m = fmaxf(m, red[i]);
    __syncthreads();
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
        const float e = expf(row[i] - m);
        row[i] = e;
        s += e;
    }
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    s = 0.0f;
    for (int i = 0; i < warps; ++i) s += red[i];
    const float inv = s > 0.0f ? 1.0f / s : 0.0f;
    for (int64_t i = threadIdx.x; i < count; i += blockDim.x) row[i] *= inv;
}

__global__ void silu_multiply_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ d,
                                     int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) {
        const float v = g[i];
        d[i] = v / (1.0f + expf(-v)) * u[i];
    }
}

__global__ void axpy_kernel(float scale, const float* __restrict__ src, float* __restrict__ dst, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = fmaf(scale, src[i], dst[i]);
}

// Block per row: the sum of squares accumulates in double, as the reference's does
// (src/Gemm.cpp:199-202); the result is written in place and/or as a bf16 copy.
__global__ void rms_norm_rows_kernel(const float* __restrict__ in, float* __restrict__ out_f32,
                                     uint16_t* __restrict__ out_bf16, const float* __restrict__ weight,
                                     int64_t count, float eps) {
    __shared__ double red[32];
    const float* row = in + static_cast<int64_t>(blockIdx.x) * count;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < count; i += blockDim.x) s = fma(static_cast<double>(row[i]), static_cast<double>(row[i]), s);
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    s = 0.0;
    for (int i = 0; i < warps; ++i) s += red[i];
    const float inverse = static_cast<float>(1.0 / sqrt(s / static_cast<double>(count) + static_cast<double>(eps)));
    for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
        const float v = row[i] * inverse * weight[i];
        if (out_f32 != nullptr) out_f32[static_cast<int64_t>(blockIdx.x) * count + i] = v;
        if (out_bf16 != nullptr) {
            const __nv_bfloat16 b = __float2bfloat16_rn(v);
            out_bf16[static_cast<int64_t>(blockIdx.x) * count + i] = *reinterpret_cast<const uint16_t*>(&b);
        }
    }
}

__global__ void add_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) dst[i] += src[i];
}

// Weight packing on upload: row-major gate and up [I, H] and down [H, I] into the
// grouped GEMMs' tile-major layout -- 128-row x 64-column tiles, tile (rb, cb) at
// (rb * (cols / 64) + cb) * 8192 elements -- with gate rows on the even rows of w13
// and up rows on the odd ones.  One thread moves 16 bytes; reads run along rows.
__global__ void __launch_bounds__(256) pack_swiglu_kernel(const uint16_t* __restrict__ gate,
                                                          const uint16_t* __restrict__ up,
                                                          const uint16_t* __restrict__ down, int I, int H,
                                                          uint16_t* __restrict__ w13, uint16_t* __restrict__ w2) {
    const int64_t n13 = int64_t(2) * I * H / 8, n2 = int64_t(H) * I / 8;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < n13 + n2; v += stride) {
        const bool first = v < n13;
        const int cols = first ? H : I;
        const int64_t q = first ? v : v - n13;
        const int64_t r = q / (cols / 8);
        const int c = static_cast<int>(q - r * (cols / 8)) * 8;
        const uint16_t* src = first ? ((r & 1) ? up : gate) + (r >> 1) * int64_t(H) + c : down + r * int64_t(I) + c;
        const int64_t dst = ((r / 128 * (cols / 64) + c / 64) * 128 + r % 128) * 64 + c % 64;
        *reinterpret_cast<uint4*>((first ? w13 : w2) + dst) = *reinterpret_cast<const uint4*>(src);
    }
}

thread_local std::string g_last_error;

lm_status finish(cudaError_t e) {
    if (e != cudaSuccess) {
        g_last_error = cudaGetErrorString(e);
        return LM_ERR_CUDA;
    }
    return LM_OK;
}

unsigned blocks_for(int64_t n, int per) { return static_cast<unsigned>((n + per - 1) / per); }

}  // namespace

const std::string& context_free_error() { return g_last_error; }

cudaError_t launch_rms_norm_rows(const float* in, float* out_f32, uint16_t* out_bf16, const float* weight, int rows,
                                 int count, float eps, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    rms_norm_rows_kernel<<<rows, 256, 0, stream>>>(in, out_f32, out_bf16, weight, count, eps);
    return cudaGetLastError();
}

cudaError_t launch_add_rows(float* dst, const float* src, int64_t count, cudaStream_t stream) {
    if (count <= 0) return cudaSuccess;
    add_kernel<<<blocks_for(count, 256), 256, 0, stream>>>(dst, src, count);
    return cudaGetLastError();
}

cudaError_t launch_pack_swiglu(const uint16_t* gate, const uint16_t* up, const uint16_t* down, int inter, int hidden,
                               uint16_t* w13, uint16_t* w2, int sms, cudaStream_t stream) {
    if (inter <= 0 || hidden <= 0 || inter % 64 != 0 || hidden % 128 != 0) return cudaErrorInvalidValue;
    const int64_t vectors = int64_t(3) * inter * hidden / 8;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((vectors + 255) / 256, int64_t(sms) * 8));
    pack_swiglu_kernel<<<grid, 256, 0, stream>>>(gate, up, down, inter, hidden, w13, w2);
    return cudaGetLastError();
}

// Loads every kernel of this file (see preload_kernels in moe_internal.h).
cudaError_t preload_ops_kernels() {
    cudaFuncAttributes a{};
    const void* kernels[] = {
        reinterpret_cast<const void*>(matvec_kernel<uint16_t>), reinterpret_cast<const void*>(matvec_kernel<float>),
        reinterpret_cast<const void*>(softmax_rows_kernel),     reinterpret_cast<const void*>(silu_multiply_kernel),
        reinterpret_cast<const void*>(axpy_kernel),             reinterpret_cast<const void*>(rms_norm_rows_kernel),
        reinterpret_cast<const void*>(add_kernel),              reinterpret_cast<const void*>(pack_swiglu_kernel),
    };
    for (const void* k : kernels)
        if (const cudaError_t e = cudaFuncGetAttributes(&a, k); e != cudaSuccess) return e;
    return cudaSuccess;
}

}  // namespace lm

using lm::blocks_for;
using lm::finish;

extern "C" {

const char* lm_kernel_description(void) {
    // The device code of this library is compiled for sm_100a only (no PTX for JIT),
    // so the description is fixed at build time, as the reference's is.
    return "sm_100a kernels: tcgen05/TMEM tensor cores fed by TMA -- the whole MoE layer in one cooperative "
           "launch up to 256 tokens, grouped SwiGLU GEMMs (1-CTA and CTA-pair) above, warp-per-token router; "
           "bf16 weights, f32 accumulate";
}

lm_status lm_gemm_matvec_bf16(const uint16_t* weights, const float* input, float* out, int64_t rows, int64_t cols,
                              void* stream) {
    if (rows < 0 || cols < 0 || (rows > 0 && (weights == nullptr || input == nullptr || out == nullptr)))
        return LM_ERR_INVALID_ARGUMENT;
    if (rows == 0) return LM_OK;
    lm::matvec_kernel<uint16_t><<<blocks_for(rows * 32, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        weights, input, out, rows, cols, 1.0f, 0);
    return finish(cudaGetLastError());
}

lm_status lm_gemm_matvec_bf16_accumulate(const uint16_t* weights, const float* input, float* out, int64_t rows,
                                         int64_t cols, float scale, void* stream) {
    if (rows < 0 || cols < 0 || (rows > 0 && (weights == nullptr || input == nullptr || out == nullptr)))
        return LM_ERR_INVALID_ARGUMENT;
    if (rows == 0) return LM_OK;
    lm::matvec_kernel<uint16_t><<<blocks_for(rows * 32, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        weights, input, out, rows, cols, scale, 1);
    return finish(cudaGetLastError());
}

lm_status lm_gemm_matvec_f32(const float* weights, const float* input, float* out, int64_t rows, int64_t cols,
                             void* stream) {
    if (rows < 0 || cols < 0 || (rows > 0 && (weights == nullptr || input == nullptr || out == nullptr)))
        return LM_ERR_INVALID_ARGUMENT;
    if (rows == 0) return LM_OK;
    lm::matvec_kernel<float><<<blocks_for(rows * 32, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        weights, input, out, rows, cols, 1.0f, 0);
    return finish(cudaGetLastError());
}

lm_status lm_gemm_softmax(float* values, int64_t rows, int64_t count, void* stream) {
    if (rows < 0 || count < 0 || (rows > 0 && count > 0 && values == nullptr)) return LM_ERR_INVALID_ARGUMENT;
    if (rows == 0 || count == 0) return LM_OK;  // src/Gemm.cpp:210-212
    lm::softmax_rows_kernel<<<static_cast<unsigned>(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(values, count);
    return finish(cudaGetLastError());
}

lm_status lm_gemm_silu_multiply(const float* gate, const float* up, float* destination, int64_t count, void* stream) {
    if (count < 0 || (count > 0 && (gate == nullptr || up == nullptr || destination == nullptr)))
        return LM_ERR_INVALID_ARGUMENT;
    if (count == 0) return LM_OK;
    lm::silu_multiply_kernel<<<blocks_for(count, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(gate, up,
                                                                                                    destination, count);
    return finish(cudaGetLastError());
}

lm_status lm_gemm_rms_norm(float* values, const float* weight, int64_t rows, int64_t count, float epsilon,
                           void* stream) {
    if (rows < 0 || count < 0 || (rows > 0 && count > 0 && (values == nullptr || weight == nullptr)))
        return LM_ERR_INVALID_ARGUMENT;
    if (rows == 0 || count == 0) return LM_OK;
    return finish(lm::launch_rms_norm_rows(values, values, nullptr, weight, static_cast<int>(rows),
                                           static_cast<int>(count), epsilon, static_cast<cudaStream_t>(stream)));
}

lm_status lm_gemm_axpy(float scale, const float* source, float* destination, int64_t count, void* stream) {
    if (count < 0 || (count > 0 && (source == nullptr || destination == nullptr))) return LM_ERR_INVALID_ARGUMENT;
    if (count == 0) return LM_OK;
    lm::axpy_kernel<<<blocks_for(count, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(scale, source,
                                                                                           destination, count);
    return finish(cudaGetLastError());
}

}  // extern "C"
