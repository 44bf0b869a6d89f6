// gguf.h -- GGUF v2/v3 reader (mmap) and v3 writer for the host side.
//
// Reader rules follow GgufReader::parse_from_bytes (src/gguf/mod.rs:1091-1358):
// little endian, u64 string lengths, tensor data section aligned to
// general.alignment (U32 or U64, default 32).  Arrays of element types other
// than I32/F32/String are skipped assuming 4-byte elements, as the reference
// does (src/gguf/mod.rs:1533-1536).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace nx {

struct GgufValue {
    int vtype = -1;  // GgufValueType id (src/gguf/mod.rs:150-165)
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
};

struct GgufTensor {
    std::string name;
    std::vector<uint64_t> shape;
    int type = 0;
    uint64_t offset = 0;  // relative to the data section
    size_t elems() const {
        size_t n = 1;
        for (uint64_t d : shape) n *= (size_t)d;
        return n;
    }
};

class GgufFile {
public:
    ~GgufFile();
    // returns 0 or an NEXUS_E_* code; err receives a message
    int open(const std::string &path, std::string &err);
    const GgufTensor *find(const std::string &name) const;
    // bytes of a tensor inside the map, nullptr when out of bounds
    const uint8_t *data(const GgufTensor &t, size_t *nbytes) const;
    bool get_usize(const std::string &key, uint64_t *out) const;
    bool get_f32(const std::string &key, float *out) const;
    const std::vector<GgufTensor> &tensors() const { return tensors_; }

private:
    const uint8_t *map_ = nullptr;
    size_t len_ = 0;
    uint32_t version_ = 0;
    uint64_t alignment_ = 32;
    uint64_t data_offset_ = 0;
    std::map<std::string, GgufValue> kv_;
    std::vector<GgufTensor> tensors_;
};

// Minimal GGUF v3 writer in the layout nexus-convert produces
// (tools/nexus-convert/main.rs:345-383): sorted metadata keys, tensor table,
// data padded to the alignment after the table and after every tensor.
struct GgufWriteTensor {
    std::string name;
    std::vector<uint64_t> shape;
    int type;
    uint64_t nbytes;
};

}  // namespace nx
