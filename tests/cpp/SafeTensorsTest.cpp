// SafeTensorsTest.cpp -- the SafeTensors header lookup through the C ABI, as a C++
// loader would use it before lm_moe_load_safetensors: argv[1] is a shard written by
// the Python checkpoint writer with a BF16 tensor "w" [6, 8] and an F32 tensor "b" [4];
// argv[2] a truncated copy of it.
#include <cstdint>
#include <string>

#include "Expect.hpp"
#include "litemind_moe.h"

int main(int argc, char** argv) {
    Expect expect("SafeTensorsTest");
        if (argc < 3) return 2;
    int32_t dtype = -1, ndim = -1;
    int64_t shape[LM_SAFETENSORS_MAX_DIMS] = {};
    uint64_t offset = 0, nbytes = 0;
    char error[512];

    expect(lm_safetensors_info(argv[1], "w", &dtype, &ndim, shape, &offset, &nbytes, error, sizeof(error)) == LM_OK,
          "w is found");
    expect(dtype == LM_DTYPE_BF16 && ndim == 2 && shape[0] == 6 && shape[1] == 8 && nbytes == 96, "w metadata");
    expect(offset % 8 == 0, "payload starts 8-byte aligned");
    expect(lm_safetensors_info(argv[1], "b", &dtype, &ndim, shape, &offset, &nbytes, error, sizeof(error)) == LM_OK &&
              dtype == LM_DTYPE_F32 && ndim == 1 && shape[0] == 4 && nbytes == 16,
          "b metadata");
    expect(lm_safetensors_info(argv[1], "missing", &dtype, &ndim, shape, &offset, &nbytes, error, sizeof(error)) ==
              LM_ERR_NOT_LOADED,
          "absent tensor");
    expect(std::string(error).find("missing") != std::string::npos, "absent tensor is named in the error");
    expect(lm_safetensors_info(argv[2], "w", &dtype, &ndim, shape, &offset, &nbytes, error, sizeof(error)) ==
              LM_ERR_INVALID_ARGUMENT,
          "truncated shard is rejected");
    expect(std::string(error).find("extends past the end") != std::string::npos, "truncation is explained");
    return expect.finish();
}
