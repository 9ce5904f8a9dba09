// Host <-> device transfers of lm_moe_forward_host done by SMs over mapped pinned memory.
//
// A copy-engine transfer costs about 8 us even for a few KB on B200 (measured: a 4 KB
// host-to-device copy takes 9.1 us between events), and the host entry point makes three
// per call (x in, y out, the status word out).  When the caller's buffers are pinned they
// are mapped into the device's address space, so a kernel can read x straight from host
// memory and write y and the status word straight back.  The pull kernel lets the forward's
// first kernel launch while it runs (programmatic dependent launch; that kernel waits for it
// before touching x), and the push kernel is itself a programmatic dependent of the
// forward's last kernel, so its launch overlaps that kernel's tail.  Both use few CTAs with
// no shared memory, so they fit on an SM beside a CTA of the fused decode kernel.
#include "moe_internal.h"
#include "ptx.cuh"

namespace lm {
namespace {

constexpr int kIoThreads = 256;
constexpr int kIoUnroll = 4;  // 16-byte loads of a thread in flight together

// dst[i] = src[i] for n 16-byte words; every load of a thread's batch issued before any store.
__device__ __forceinline__ void copy16(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * kIoThreads;
    for (size_t base = static_cast<size_t>(blockIdx.x) * kIoThreads + threadIdx.x; base < n;
         base += stride * kIoUnroll) {
        uint4 v[kIoUnroll];
#pragma unroll
        for (int u = 0; u < kIoUnroll; ++u)
            if (base + u * stride < n) v[u] = src[base + u * stride];
#pragma unroll
        for (int u = 0; u < kIoUnroll; ++u)
            if (base + u * stride < n) dst[base + u * stride] = v[u];
    }
}

// x (and the optional logit bias) from mapped host memory into the device staging buffers.
__global__ void __launch_bounds__(kIoThreads) host_pull_kernel(const uint4* src0, uint4* dst0, size_t n0,
                                                               const uint4* src1, uint4* dst1, size_t n1) {
    pdl_launch_dependents();
    copy16(src0, dst0, n0);
    if (n1 > 0) copy16(src1, dst1, n1);
}

// y into mapped host memory once the forward has finished, and the status word with it.
__global__ void __launch_bounds__(kIoThreads) host_push_kernel(const uint4* src, uint4* dst, size_t n,
                                                               const int* status, int* status_host) {
    pdl_wait();
    copy16(src, dst, n);
    if (blockIdx.x == 0 && threadIdx.x == 0) *status_host = *reinterpret_cast<const volatile int*>(status);
}

int io_grid(size_t n16, int sms) {
    const size_t per_cta = static_cast<size_t>(kIoThreads) * kIoUnroll;
    const size_t want = (n16 + per_cta - 1) / per_cta;
    return static_cast<int>(want < 1 ? 1 : (want > static_cast<size_t>(sms) ? sms : want));
}

}  // namespace

bool host_io_eligible(const void* p, size_t bytes) {
    return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (bytes & 15u) == 0;
}

cudaError_t launch_host_pull(void* dst0, const void* src0_mapped, size_t bytes0, void* dst1,
                             const void* src1_mapped, size_t bytes1, int sms, cudaStream_t stream) {
    const size_t n0 = bytes0 / 16, n1 = src1_mapped != nullptr ? bytes1 / 16 : 0;
    host_pull_kernel<<<io_grid(n0 > n1 ? n0 : n1, sms), kIoThreads, 0, stream>>>(
        static_cast<const uint4*>(src0_mapped), static_cast<uint4*>(dst0), n0, static_cast<const uint4*>(src1_mapped),
        static_cast<uint4*>(dst1), n1);
    return cudaGetLastError();
}

cudaError_t launch_host_push(void* dst_mapped, const void* src, size_t bytes, const int32_t* status,
                             int32_t* status_host_mapped, int sms, cudaStream_t stream) {
    const size_t n = bytes / 16;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(io_grid(n, sms));
    cfg.blockDim = dim3(kIoThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, host_push_kernel, static_cast<const uint4*>(src), static_cast<uint4*>(dst_mapped),
                              n, static_cast<const int*>(status), static_cast<int*>(status_host_mapped));
}

cudaError_t preload_host_io_kernels() {
    cudaFuncAttributes a;
    cudaError_t e = cudaFuncGetAttributes(&a, host_pull_kernel);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, host_push_kernel);
    return e;
}

}  // namespace lm
