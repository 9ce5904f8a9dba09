// tensor_map.cpp -- host-side encoding of TMA descriptors (CUtensorMap).
//
// cuTensorMapEncodeTiled is a driver-API function that only fills a 128-byte
// descriptor on the host.  It is fetched through the runtime's entry-point query
// so the library does not link libcuda directly.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

namespace lm {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult status{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
            status == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        }
    });
    return fn;
}

}  // namespace

// A row-major [rows, cols] bf16 matrix read in boxes of [box_rows, box_cols]
// with the 128-byte swizzle the UMMA shared-memory descriptors expect.  Rows of a
// box past the end read as zeros.
bool encode_tensor_map_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                            uint32_t box_cols, std::string& error) {
    auto fn = encode_fn();
    if (fn == nullptr) {
        error = "cuTensorMapEncodeTiled is unavailable (no CUDA driver?)";
        return false;
    }
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 2) % 16 != 0 || box_cols * 2 != 128) {
        error = "tensor map: base must be 16-byte aligned, rows a multiple of 16 bytes, boxes 128 bytes wide";
        return false;
    }
    if (rows == 0) rows = 1;  // an empty operand is never read, but the descriptor must be valid
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t elem_strides[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                          elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        error = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r)) + " (rows " +
                std::to_string(rows) + ", cols " + std::to_string(cols) + ", box " + std::to_string(box_rows) + "x" +
                std::to_string(box_cols) + ")";
        return false;
    }
    return true;
}

}  // namespace lm
