// SafeTensors.cpp -- header parsing and memory mapping of SafeTensors shards.
#include "SafeTensors.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <utility>

namespace lm::host {
namespace {

constexpr uint64_t kMaxHeader = 512ull << 20;  // larger: treated as not a SafeTensors file

// A small JSON value tree: enough for a SafeTensors header.
struct JValue {
    enum Kind { Null, Bool, Number, String, Array, Object } kind{Null};
    double number{};
    bool boolean{};
    std::string text;
    std::vector<JValue> items;                            // Array
    std::vector<std::pair<std::string, JValue>> members;  // Object, in file order

    const JValue* get(const std::string& key) const {
        for (const auto& m : members)
            if (m.first == key) return &m.second;
        return nullptr;
    }
};

class JParser {
public:
    JParser(const char* p, size_t n) : p_(p), end_(p + n) {}

    bool parse(JValue& out, std::string& error) {
        if (!value(out, 0)) {
            error = error_.empty() ? "malformed JSON" : error_;
            return false;
        }
        ws();
        if (p_ != end_) {
            error = "trailing characters after the JSON header";
            return false;
        }
        return true;
    }

private:
    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool fail(const char* what) {
        if (error_.empty()) error_ = what;
        return false;
    }
    bool value(JValue& v, int depth) {
        if (depth > 64) return fail("JSON nested too deeply");
        ws();
        if (p_ >= end_) return fail("unexpected end of JSON");
        switch (*p_) {
            case '{': return object(v, depth);
            case '[': return array(v, depth);
            case '"': v.kind = JValue::String; return string(v.text);
            case 't': return literal("true", v, JValue::Bool, true);
            case 'f': return literal("false", v, JValue::Bool, false);
            case 'n': return literal("null", v, JValue::Null, false);
            default: return number(v);
        }
    }
    bool literal(const char* word, JValue& v, JValue::Kind kind, bool b) {
        const size_t n = std::strlen(word);
        if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, word, n) != 0) return fail("bad JSON literal");
        p_ += n;
        v.kind = kind;
        v.boolean = b;
        return true;
    }
    bool number(JValue& v) {
        const char* start = p_;
        if (p_ < end_ && (*p_ == '-' || *p_ == '+')) ++p_;
        bool digits = false;
        while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                             ((*p_ == '-' || *p_ == '+') && (p_[-1] == 'e' || p_[-1] == 'E')))) {
            digits |= (*p_ >= '0' && *p_ <= '9');
            ++p_;
        }
        if (!digits) return fail("bad JSON number");
        v.kind = JValue::Number;
        v.number = std::strtod(std::string(start, p_).c_str(), nullptr);
        return true;
    }
    bool string(std::string& s) {
        ++p_;  // opening quote
        while (p_ < end_ && *p_ != '"') {
            if (*p_ == '\\') {
                if (++p_ >= end_) break;
                const char c = *p_++;
                switch (c) {
                    case '"': s += '"'; break;
                    case '\\': s += '\\'; break;
                    case '/': s += '/'; break;
                    case 'b': s += '\b'; break;
                    case 'f': s += '\f'; break;
                    case 'n': s += '\n'; break;
                    case 'r': s += '\r'; break;
                    case 't': s += '\t'; break;
                    case 'u': {
                        if (end_ - p_ < 4) return fail("bad JSON escape");
                        unsigned cp = 0;
                        for (int i = 0; i < 4; ++i) {
                            const char h = *p_++;
                            cp = cp * 16 + (h >= '0' && h <= '9' ? h - '0' : (h | 32) >= 'a' && (h | 32) <= 'f' ? (h | 32) - 'a' + 10 : 99);
                            if (cp > 0xFFFF) return fail("bad JSON escape");
                        }
                        // UTF-8 encode (names are ASCII in practice; surrogates kept as-is).
                        if (cp < 0x80) {
                            s += static_cast<char>(cp);
                        } else if (cp < 0x800) {
                            s += static_cast<char>(0xC0 | (cp >> 6));
                            s += static_cast<char>(0x80 | (cp & 0x3F));
                        } else {
                            s += static_cast<char>(0xE0 | (cp >> 12));
                            s += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
                            s += static_cast<char>(0x80 | (cp & 0x3F));
                        }
                        break;
                    }
                    default: return fail("bad JSON escape");
                }
            } else {
                s += *p_++;
            }
        }
        if (p_ >= end_) return fail("unterminated JSON string");
        ++p_;  // closing quote
        return true;
    }
    bool array(JValue& v, int depth) {
        v.kind = JValue::Array;
        ++p_;
        ws();
        if (p_ < end_ && *p_ == ']') {
            ++p_;
            return true;
        }
        while (true) {
            v.items.emplace_back();
            if (!value(v.items.back(), depth + 1)) return false;
            ws();
            if (p_ < end_ && *p_ == ',') {
                ++p_;
                continue;
            }
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            return fail("malformed JSON array");
        }
    }
    bool object(JValue& v, int depth) {
        v.kind = JValue::Object;
        ++p_;
        ws();
        if (p_ < end_ && *p_ == '}') {
            ++p_;
            return true;
        }
        while (true) {
            ws();
            if (p_ >= end_ || *p_ != '"') return fail("malformed JSON object");
            std::string key;
            if (!string(key)) return false;
            ws();
            if (p_ >= end_ || *p_ != ':') return fail("malformed JSON object");
            ++p_;
            v.members.emplace_back(std::move(key), JValue{});
            if (!value(v.members.back().second, depth + 1)) return false;
            ws();
            if (p_ < end_ && *p_ == ',') {
                ++p_;
                continue;
            }
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            return fail("malformed JSON object");
        }
    }

    const char* p_;
    const char* end_;
    std::string error_;
};

StDtype parse_dtype(const std::string& t, size_t& elem) {
    static const struct {
        const char* name;
        StDtype d;
        size_t bytes;
    } table[] = {{"BF16", StDtype::BF16, 2}, {"F16", StDtype::F16, 2},  {"F32", StDtype::F32, 4},
                 {"F64", StDtype::Other, 8}, {"I8", StDtype::Other, 1}, {"I16", StDtype::Other, 2},
                 {"I32", StDtype::Other, 4}, {"I64", StDtype::Other, 8}, {"U8", StDtype::Other, 1},
                 {"BOOL", StDtype::Other, 1}};
    for (const auto& e : table)
        if (t == e.name) {
            elem = e.bytes;
            return e.d;
        }
    elem = 0;
    return StDtype::Unknown;
}

float half_to_float(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    float v;
    if (exp == 0) {
        v = std::ldexp(static_cast<float>(man), -24);  // subnormal (or zero)
    } else if (exp == 31) {
        v = man ? std::nanf("") : INFINITY;
    } else {
        v = std::ldexp(static_cast<float>(man | 0x400u), static_cast<int>(exp) - 25);
    }
    return sign ? -v : v;
}

float bf16_to_float(uint16_t b) {
    const uint32_t u = static_cast<uint32_t>(b) << 16;
    float v;
    std::memcpy(&v, &u, 4);
    return v;
}

}  // namespace

std::string shape_text(const std::vector<int64_t>& shape) {
    std::string s = "[";
    for (size_t i = 0; i < shape.size(); ++i) s += (i ? ", " : "") + std::to_string(shape[i]);
    return s + "]";
}

StShard::~StShard() { close(); }

StShard::StShard(StShard&& o) noexcept
    : path_(std::move(o.path_)), map_(std::exchange(o.map_, nullptr)), size_(std::exchange(o.size_, 0)),
      tensors_(std::move(o.tensors_)) {}

void StShard::close() {
    if (map_ != nullptr) munmap(const_cast<uint8_t*>(map_), size_);
    map_ = nullptr;
    size_ = 0;
    tensors_.clear();
}

bool StShard::open(const std::string& path, std::string& error) {
    close();
    path_ = path;
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        error = "cannot open " + path + ": " + std::strerror(errno);
        return false;
    }
    struct stat st{};
    if (fstat(fd, &st) != 0) {
        error = "cannot stat " + path;
        ::close(fd);
        return false;
    }
    size_ = static_cast<size_t>(st.st_size);
    if (size_ < 8) {
        ::close(fd);
        error = path + " is too small to be a SafeTensors shard.";
        return false;
    }
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
        error = "cannot map " + path;
        size_ = 0;
        return false;
    }
    map_ = static_cast<const uint8_t*>(m);
    uint64_t header = 0;
    for (int i = 0; i < 8; ++i) header |= static_cast<uint64_t>(map_[i]) << (8 * i);
    if (header == 0 || header > kMaxHeader || header > size_ - 8) {
        error = path + " declares an implausible SafeTensors header length of " + std::to_string(header) + " bytes.";
        close();
        return false;
    }
    JValue doc;
    std::string jerr;
    if (!JParser(reinterpret_cast<const char*>(map_ + 8), header).parse(doc, jerr)) {
        error = path + ": " + jerr;
        close();
        return false;
    }
    if (doc.kind != JValue::Object) {
        error = path + ": the SafeTensors header must be a JSON object.";
        close();
        return false;
    }
    const uint64_t payload = 8 + header;
    for (const auto& [name, entry] : doc.members) {
        if (name == "__metadata__") continue;
        auto bad = [&](const std::string& why) {
            error = path + ": tensor '" + name + "' " + why;
            close();
            return false;
        };
        if (entry.kind != JValue::Object) return bad("entry is not a JSON object.");
        StTensor t;
        t.name = name;
        const JValue* dt = entry.get("dtype");
        t.dtype_text = (dt != nullptr && dt->kind == JValue::String) ? dt->text : "?";
        size_t elem = 0;
        t.dtype = parse_dtype(t.dtype_text, elem);
        if (t.dtype == StDtype::Unknown) return bad("uses an unsupported dtype '" + t.dtype_text + "'.");
        const JValue* sh = entry.get("shape");
        if (sh == nullptr || sh->kind != JValue::Array) return bad("has no shape array.");
        // Every number below is a JSON double: it must be a non-negative integer no
        // larger than the shard (2^53 bounds what a double holds exactly), checked
        // before any cast; products are checked against overflow.
        constexpr double kExact = 9007199254740992.0;  // 2^53
        auto whole = [](const JValue& v) {
            return v.kind == JValue::Number && v.number >= 0 && v.number == std::floor(v.number) && v.number <= kExact;
        };
        uint64_t count = 1;
        for (const JValue& d : sh->items) {
            if (!whole(d)) return bad("has a non-numeric dimension.");
            const uint64_t dim = static_cast<uint64_t>(d.number);
            t.shape.push_back(static_cast<int64_t>(dim));
            if (dim != 0 && count > UINT64_MAX / dim) return bad("has a shape whose element count overflows.");
            count *= dim;
        }
        const JValue* off = entry.get("data_offsets");
        if (off == nullptr || off->kind != JValue::Array || off->items.size() != 2 || !whole(off->items[0]) ||
            !whole(off->items[1]))
            return bad("has a malformed data_offsets pair.");
        const uint64_t b = static_cast<uint64_t>(off->items[0].number);
        const uint64_t e = static_cast<uint64_t>(off->items[1].number);
        if (e < b) return bad("has data_offsets in descending order.");
        if (payload > size_ || e > size_ - payload) return bad("extends past the end of the shard.");
        if (count > UINT64_MAX / elem) return bad("has a shape whose byte size overflows.");
        t.offset = payload + b;
        t.nbytes = count * elem;
        if (t.nbytes != e - b)
            return bad("declares " + std::to_string(e - b) + " payload bytes but its shape and dtype need " +
                       std::to_string(t.nbytes) + ".");
        t.data = map_ + t.offset;
        tensors_.push_back(std::move(t));
    }
    if (tensors_.empty()) {
        error = path + " contains no tensors.";
        close();
        return false;
    }
    return true;
}

bool StCheckpoint::open(const std::vector<std::string>& paths, std::string& error) {
    shards_.clear();
    index_.clear();
    shards_.reserve(paths.size());
    for (const std::string& p : paths) {
        StShard s;
        if (!s.open(p, error)) return false;
        shards_.push_back(std::move(s));
    }
    for (const StShard& s : shards_)
        for (const StTensor& t : s.tensors()) index_[t.name] = &t;
    return true;
}

const StTensor* StCheckpoint::find(const std::string& name) const {
    const auto it = index_.find(name);
    return it == index_.end() ? nullptr : it->second;
}

const StTensor* StCheckpoint::require(const std::string& name, const std::vector<int64_t>& shape, StDtype dtype,
                                      std::string& error) const {
    const StTensor* t = find(name);
    if (t == nullptr) {
        error = "The checkpoint has no tensor named '" + name + "'.";
        return nullptr;
    }
    if (t->shape != shape) {
        error = "Tensor '" + name + "' has shape " + shape_text(t->shape) + " but config.json implies " +
                shape_text(shape) + ".";
        return nullptr;
    }
    if (t->dtype != dtype) {
        error = "Tensor '" + name + "' is stored as " + t->dtype_text + " but this build reads " +
                (dtype == StDtype::BF16 ? "BF16" : dtype == StDtype::F16 ? "F16" : "F32") + " here.";
        return nullptr;
    }
    return t;
}

bool StCheckpoint::read_float32(const std::string& name, const std::vector<int64_t>& shape, std::vector<float>& out,
                                std::string& error) const {
    const StTensor* t = find(name);
    if (t == nullptr) {
        error = "The checkpoint has no tensor named '" + name + "'.";
        return false;
    }
    if (t->shape != shape) {
        error = "Tensor '" + name + "' has shape " + shape_text(t->shape) + " but config.json implies " +
                shape_text(shape) + ".";
        return false;
    }
    uint64_t n = 1;
    for (int64_t d : shape) n *= static_cast<uint64_t>(d);
    out.resize(n);
    switch (t->dtype) {
        case StDtype::F32:
            std::memcpy(out.data(), t->data, n * 4);
            return true;
        case StDtype::BF16:
            for (uint64_t i = 0; i < n; ++i) {
                uint16_t v;
                std::memcpy(&v, t->data + 2 * i, 2);
                out[i] = bf16_to_float(v);
            }
            return true;
        case StDtype::F16:
            for (uint64_t i = 0; i < n; ++i) {
                uint16_t v;
                std::memcpy(&v, t->data + 2 * i, 2);
                out[i] = half_to_float(v);
            }
            return true;
        default:
            error = "Tensor '" + name + "' is stored as " + t->dtype_text + "; expected BF16, F16 or F32.";
            return false;
    }
}

}  // namespace lm::host
