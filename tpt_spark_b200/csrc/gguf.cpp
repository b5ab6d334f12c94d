// gguf.cpp -- GGUF v2/v3 reader (format: magic "GGUF", u32 version, u64 tensor count,
// u64 kv count, typed key/values, tensor infos, data section aligned to general.alignment).
#include "gguf.h"

#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "tptc.h"

namespace tptc {

void ggml_block_info(uint32_t type, uint64_t& elems, uint64_t& bytes) {
    switch (type) {
    case TPTC_TYPE_F32: elems = 1; bytes = 4; return;
    case TPTC_TYPE_F16: elems = 1; bytes = 2; return;
    case TPTC_TYPE_Q8_0: elems = 32; bytes = 34; return;
    case TPTC_TYPE_Q4_K: elems = 256; bytes = 144; return;
    case TPTC_TYPE_Q6_K: elems = 256; bytes = 210; return;
    case TPTC_TYPE_Q4_0: elems = 32; bytes = 18; return;
    case TPTC_TYPE_Q4_1: elems = 32; bytes = 20; return;
    case TPTC_TYPE_Q5_0: elems = 32; bytes = 22; return;
    case TPTC_TYPE_Q5_1: elems = 32; bytes = 24; return;
    case TPTC_TYPE_Q2_K: elems = 256; bytes = 84; return;
    case TPTC_TYPE_Q3_K: elems = 256; bytes = 110; return;
    case TPTC_TYPE_Q5_K: elems = 256; bytes = 176; return;
    default: elems = 0; bytes = 0; return;
    }
}

namespace {

struct Cursor {
    const uint8_t* p;
    uint64_t size, pos = 0;
    bool bad = false;
    bool need(uint64_t n) {
        if (bad || n > size - pos) {
            bad = true;
            return false;
        }
        return true;
    }
    template <class T>
    T rd() {
        T v{};
        if (need(sizeof(T))) {
            memcpy(&v, p + pos, sizeof(T));
            pos += sizeof(T);
        }
        return v;
    }
    std::string str() {
        uint64_t n = rd<uint64_t>();
        if (!need(n) || n > (1u << 24)) {
            bad = true;
            return {};
        }
        std::string s(reinterpret_cast<const char*>(p + pos), n);
        pos += n;
        return s;
    }
};

// GGUF value types.
enum : uint32_t { U8 = 0, I8, U16, I16, U32, I32, F32, BOOLT, STRT, ARRT, U64T, I64T, F64T };

bool read_scalar(Cursor& c, uint32_t t, GgufValue& v) {
    switch (t) {
    case U8: v.kind = GgufValue::U64; v.u = c.rd<uint8_t>(); break;
    case I8: v.kind = GgufValue::I64; v.i = c.rd<int8_t>(); break;
    case U16: v.kind = GgufValue::U64; v.u = c.rd<uint16_t>(); break;
    case I16: v.kind = GgufValue::I64; v.i = c.rd<int16_t>(); break;
    case U32: v.kind = GgufValue::U64; v.u = c.rd<uint32_t>(); break;
    case I32: v.kind = GgufValue::I64; v.i = c.rd<int32_t>(); break;
    case F32: v.kind = GgufValue::F64; v.f = c.rd<float>(); break;
    case BOOLT: v.kind = GgufValue::BOOL; v.u = c.rd<uint8_t>(); break;
    case STRT: v.kind = GgufValue::STR; v.s = c.str(); break;
    case U64T: v.kind = GgufValue::U64; v.u = c.rd<uint64_t>(); break;
    case I64T: v.kind = GgufValue::I64; v.i = c.rd<int64_t>(); break;
    case F64T: v.kind = GgufValue::F64; v.f = c.rd<double>(); break;
    default: return false;
    }
    return !c.bad;
}

bool skip_value(Cursor& c, uint32_t t) {
    GgufValue v;
    return read_scalar(c, t, v);
}

}  // namespace

GgufFile::~GgufFile() { close(); }

void GgufFile::close() {
    if (map) munmap(const_cast<uint8_t*>(map), size);
    if (fd >= 0) ::close(fd);
    map = nullptr;
    fd = -1;
}

int GgufFile::open(const std::string& p, std::string& err) {
    close();
    path = p;
    fd = ::open(p.c_str(), O_RDONLY);
    if (fd < 0) {
        err = "opening " + p + ": " + strerror(errno);
        return TPTC_ERR_IO;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
        err = "stat " + p + ": " + strerror(errno);
        return TPTC_ERR_IO;
    }
    size = static_cast<uint64_t>(st.st_size);
    if (size < 24) {
        err = p + ": file too small for a GGUF header";
        return TPTC_ERR_FORMAT;
    }
    void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
        err = "mmap " + p + ": " + strerror(errno);
        return TPTC_ERR_IO;
    }
    map = static_cast<const uint8_t*>(m);
    madvise(m, size, MADV_SEQUENTIAL);
    Cursor c{map, size};
    if (memcmp(map, "GGUF", 4) != 0) {
        err = p + ": bad magic (not a GGUF file)";
        return TPTC_ERR_FORMAT;
    }
    c.pos = 4;
    version = c.rd<uint32_t>();
    if (version < 2 || version > 3) {
        err = p + ": unsupported GGUF version " + std::to_string(version);
        return TPTC_ERR_FORMAT;
    }
    uint64_t n_tensors = c.rd<uint64_t>(), n_kv = c.rd<uint64_t>();
    if (n_tensors > (1u << 20) || n_kv > (1u << 20)) {
        err = p + ": implausible tensor/kv counts";
        return TPTC_ERR_FORMAT;
    }
    for (uint64_t i = 0; i < n_kv && !c.bad; i++) {
        std::string key = c.str();
        uint32_t t = c.rd<uint32_t>();
        GgufValue v;
        if (t == ARRT) {
            v.kind = GgufValue::ARR;
            v.arr_type = c.rd<uint32_t>();
            v.arr_len = c.rd<uint64_t>();
            for (uint64_t j = 0; j < v.arr_len && !c.bad; j++)
                if (!skip_value(c, v.arr_type)) c.bad = true;
        } else if (!read_scalar(c, t, v)) {
            c.bad = true;
        }
        kv[key] = v;
    }
    if (c.bad) {
        err = p + ": truncated or malformed metadata";
        return TPTC_ERR_FORMAT;
    }
    uint64_t al;
    if (get_u64("general.alignment", al) && al > 0 && (al & (al - 1)) == 0) alignment = al;
    tensors.resize(n_tensors);
    for (uint64_t i = 0; i < n_tensors && !c.bad; i++) {
        GgufTensor& t = tensors[i];
        t.name = c.str();
        uint32_t nd = c.rd<uint32_t>();
        if (nd == 0 || nd > 4) {
            c.bad = true;
            break;
        }
        t.ne.resize(nd);
        for (uint32_t d = 0; d < nd; d++) t.ne[d] = c.rd<uint64_t>();
        t.type = c.rd<uint32_t>();
        t.offset = c.rd<uint64_t>();
        uint64_t be, bb;
        ggml_block_info(t.type, be, bb);
        if (be == 0) {
            t.nbytes = 0;  // unsupported type: rejected by the loader only if the tensor is used
        } else {
            uint64_t n = t.n_elems();
            if (n % be != 0) {
                err = p + ": tensor " + t.name + " element count is not a whole number of blocks";
                return TPTC_ERR_FORMAT;
            }
            t.nbytes = n / be * bb;
        }
    }
    if (c.bad) {
        err = p + ": truncated or malformed tensor infos";
        return TPTC_ERR_FORMAT;
    }
    data_offset = (c.pos + alignment - 1) / alignment * alignment;
    for (auto& t : tensors) {
        // wgpu_loader.rs:130 -- a tensor must lie inside the file.
        if (t.offset > size || data_offset + t.offset > size || t.nbytes > size - data_offset - t.offset) {
            err = "tensor '" + t.name + "' extends past end of file";
            return TPTC_ERR_FORMAT;
        }
    }
    return TPTC_OK;
}

const GgufTensor* GgufFile::find(const std::string& name) const {
    for (auto& t : tensors)
        if (t.name == name) return &t;
    return nullptr;
}

bool GgufFile::get_u64(const std::string& key, uint64_t& out) const {
    auto it = kv.find(key);
    if (it == kv.end()) return false;
    if (it->second.kind == GgufValue::U64) out = it->second.u;
    else if (it->second.kind == GgufValue::I64 && it->second.i >= 0) out = static_cast<uint64_t>(it->second.i);
    else return false;
    return true;
}

bool GgufFile::get_f32(const std::string& key, float& out) const {
    auto it = kv.find(key);
    if (it == kv.end()) return false;
    if (it->second.kind == GgufValue::F64) out = static_cast<float>(it->second.f);
    else if (it->second.kind == GgufValue::U64) out = static_cast<float>(it->second.u);
    else if (it->second.kind == GgufValue::I64) out = static_cast<float>(it->second.i);
    else return false;
    return true;
}

bool GgufFile::get_str(const std::string& key, std::string& out) const {
    auto it = kv.find(key);
    if (it == kv.end() || it->second.kind != GgufValue::STR) return false;
    out = it->second.s;
    return true;
}

}  // namespace tptc
