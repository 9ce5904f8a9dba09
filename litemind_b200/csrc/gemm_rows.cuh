// gemm_rows.cuh -- checked output-row addressing shared by the grouped GEMM kernels.
#pragma once

#include "moe_internal.h"
#include "ptx.cuh"

namespace lm {

// Where routed row `row`'s down output goes in args.y_rows (expert parallelism):
// y_rows_map[row], or row itself without a map.  A row or destination outside
// y_rows_cap returns -1 and records kDevBadRow, so a bad schedule or map costs an
// error status instead of a stray store.
__device__ __forceinline__ int y_row_dst(const GemmArgs& args, int row) {
    int dst = row;
    if (args.y_rows_map != nullptr) dst = (row >= 0 && row < args.y_rows_cap) ? args.y_rows_map[row] : -1;
    if (dst < 0 || dst >= args.y_rows_cap) {
        atomicCAS(args.status, 0, kDevBadRow);
        return -1;
    }
    return dst;
}

}  // namespace lm
