// ep_peer.cu -- readiness flags of the copy-engine expert-parallel exchange.
//
// In that exchange every rank pulls the rows it needs straight out of its peers'
// device memory (IPC-mapped buffers) with cudaMemcpyAsync on copy-engine streams, so
// the GEMMs keep every SM.  A pull may start only once the peer's kernels that wrote
// the rows have finished; the peer announces that by storing an epoch number, with
// system-scope release, into a flag slot of every other rank's flag buffer, and the
// puller's copy stream first runs a one-warp kernel that waits for its own flag slot
// to reach the epoch.  Each rank only polls its own memory.  The wait is bounded: after
// the limit it records kDevTimeoutExchange in the status word and returns, so a peer
// that never signals ends the forward with an error instead of a hang.
#include "moe_internal.h"
#include "ptx.cuh"

namespace lm {
namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Lane r < n stores `epoch` into slot `slot` of rank r's flag buffer (r != self):
// everything this GPU wrote before this kernel is visible to the peer first.
__global__ void ep_signal_kernel(EpPeerFlags peers, int self, int slot, uint32_t epoch) {
    __threadfence_system();
    const int r = threadIdx.x;
    if (r < peers.n && r != self) st_release_sys_u32(peers.flags[r] + slot, epoch);
}

// Waits until flags[slot] has reached `epoch` (wrap-safe), at most limit_ns.  The wait
// that gives up first records (slot, value seen, epoch wanted) in diag[0..2].
__global__ void ep_wait_kernel(const uint32_t* flags, int slot, uint32_t epoch, int32_t* status, uint32_t* diag,
                               uint64_t limit_ns) {
    if (threadIdx.x != 0) return;
    const uint32_t* f = flags + slot;
    if (static_cast<int32_t>(ld_acquire_sys_u32(f) - epoch) >= 0) return;
    const uint64_t start = global_timer_ns();
    while (static_cast<int32_t>(ld_acquire_sys_u32(f) - epoch) < 0) {
        if (*reinterpret_cast<volatile int32_t*>(status) != 0) return;  // another wait already failed
        if (global_timer_ns() - start > limit_ns) {
            if (atomicCAS(status, 0, kDevTimeoutExchange) == 0) {
                diag[0] = static_cast<uint32_t>(slot);
                diag[1] = ld_acquire_sys_u32(f);
                diag[2] = epoch;
            }
            return;
        }
        __nanosleep(200);
    }
}

}  // namespace

cudaError_t launch_ep_signal(const EpPeerFlags& peers, int self, int slot, uint32_t epoch, cudaStream_t stream) {
    if (peers.n < 1 || peers.n > kEpCopyMaxRanks) return cudaErrorInvalidValue;
    ep_signal_kernel<<<1, 32, 0, stream>>>(peers, self, slot, epoch);
    return cudaGetLastError();
}

cudaError_t launch_ep_wait(const uint32_t* flags, int slot, uint32_t epoch, int32_t* status, uint32_t* diag,
                           uint64_t limit_ns, cudaStream_t stream) {
    ep_wait_kernel<<<1, 32, 0, stream>>>(flags, slot, epoch, status, diag, limit_ns);
    return cudaGetLastError();
}

cudaError_t preload_ep_peer_kernels() {
    cudaFuncAttributes a{};
    cudaError_t e = cudaFuncGetAttributes(&a, reinterpret_cast<const void*>(ep_signal_kernel));
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, reinterpret_cast<const void*>(ep_wait_kernel));
    return e;
}

}  // namespace lm
