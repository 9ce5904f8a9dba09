// SafeTensors.hpp -- read-only view of SafeTensors checkpoint shards for the HBM
// expert loader.
//
// The format (the one the reference's SafeTensor reads, src/SafeTensor.cpp:87-152):
// an 8-byte little-endian header length, a JSON object mapping tensor names to
// {"dtype", "shape", "data_offsets": [begin, end]} (offsets relative to the end of
// the header; an optional "__metadata__" entry is ignored), then the payload.  A
// shard is memory-mapped and only its header is parsed; payload pages are read when
// the loader copies a tensor to the device.  The checks and their messages follow
// the reference's: implausible header length, non-object header, unknown dtype,
// malformed shape or offsets, payload size not matching shape x dtype, payload past
// the end of the file.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace lm::host {

enum class StDtype : int { Unknown = 0, BF16 = 1, F16 = 2, F32 = 3, Other = 4 };

struct StTensor {
    std::string name;
    StDtype dtype{StDtype::Unknown};
    std::string dtype_text;
    std::vector<int64_t> shape;
    uint64_t offset{};  // file-absolute
    uint64_t nbytes{};
    const uint8_t* data{};  // inside the shard's mapping
};

class StShard {
public:
    StShard() = default;
    ~StShard();
    StShard(const StShard&) = delete;
    StShard& operator=(const StShard&) = delete;
    StShard(StShard&& o) noexcept;
    StShard& operator=(StShard&&) = delete;

    bool open(const std::string& path, std::string& error);
    const std::vector<StTensor>& tensors() const { return tensors_; }

private:
    void close();
    std::string path_;
    const uint8_t* map_{nullptr};
    size_t size_{0};
    std::vector<StTensor> tensors_;
};

// Several shards of one checkpoint, looked up by tensor name.
class StCheckpoint {
public:
    bool open(const std::vector<std::string>& paths, std::string& error);
    const StTensor* find(const std::string& name) const;

    // A tensor that must exist with this shape and dtype (WeightStore::require,
    // src/WeightStore.cpp:119-140).
    const StTensor* require(const std::string& name, const std::vector<int64_t>& shape, StDtype dtype,
                            std::string& error) const;
    // A float tensor of this shape widened to f32 from BF16, F16 or F32
    // (WeightStore::read_float32).
    bool read_float32(const std::string& name, const std::vector<int64_t>& shape, std::vector<float>& out,
                      std::string& error) const;

private:
    std::vector<StShard> shards_;
    std::unordered_map<std::string, const StTensor*> index_;
};

std::string shape_text(const std::vector<int64_t>& shape);

}  // namespace lm::host
