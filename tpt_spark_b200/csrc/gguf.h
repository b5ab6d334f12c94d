// gguf.h -- GGUF v2/v3 reader over a read-only mmap.
//
// Replaces candle's gguf_file::Content::read as used by the reference loader
// (src-tauri/src/engine/wgpu_loader.rs:96-111) and extract_meta (:305-406).
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace tptc {

struct GgufValue {
    enum Kind { U64, I64, F64, BOOL, STR, ARR, NONE } kind = NONE;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    std::string s;
    uint32_t arr_type = 0;
    uint64_t arr_len = 0;
};

struct GgufTensor {
    std::string name;
    std::vector<uint64_t> ne;  // innermost first
    uint32_t type = 0;
    uint64_t offset = 0;       // relative to the data section
    uint64_t nbytes = 0;
    uint64_t n_elems() const {
        uint64_t n = 1;
        for (auto d : ne) n *= d;
        return n;
    }
};

struct GgufFile {
    std::string path;
    int fd = -1;
    const uint8_t* map = nullptr;
    uint64_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32;
    uint64_t data_offset = 0;
    std::map<std::string, GgufValue> kv;
    std::vector<GgufTensor> tensors;

    ~GgufFile();
    // Returns 0 or a TPTC_ERR_* code, with a message in `err`.
    int open(const std::string& p, std::string& err);
    void close();
    const GgufTensor* find(const std::string& name) const;
    bool get_u64(const std::string& key, uint64_t& out) const;
    bool get_f32(const std::string& key, float& out) const;
    bool get_str(const std::string& key, std::string& out) const;
    const uint8_t* tensor_data(const GgufTensor& t) const { return map + data_offset + t.offset; }
};

// (elements per block, bytes per block) of a GGML type; (0, 0) for unsupported types.
void ggml_block_info(uint32_t type, uint64_t& elems, uint64_t& bytes);

}  // namespace tptc
