// SBB1 scenario blob: reader (mmap) and writer.
//
// The on-disk format is the reference's interchange format and is kept byte for
// byte so blobs are portable between the reference's C core and this library:
//   header   52 B : "SBB1", u32 version = 1, u32 n_sections, u64 dir_off,
//                   u64 names_off, u64 names_len, u64 total, u64 reserved
//   directory 56 B per section: u32 name_off, u32 dtype, u32 ndim, u32 reserved,
//                   u64 shape[4], u64 data_off
//   names    NUL-terminated ASCII; data area starts 64-byte aligned.
// dtype codes: 0 f64, 1 f32, 2 i64, 3 i32, 4 i8, 5 u8, 6 u32, 7 str.
// (reference: complete_port/pysim/sbb.py:1-53, complete_port/csim/sb_baked.c:19-73)
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace sbb {

enum DType : uint32_t { F64 = 0, F32 = 1, I64 = 2, I32 = 3, I8 = 4, U8 = 5, U32 = 6, STR = 7 };

struct Section {
    std::string name;
    uint32_t dtype = 0;
    uint32_t ndim = 0;
    uint64_t shape[4] = {1, 1, 1, 1};
    uint64_t count = 0;
    uint64_t data_off = 0;
};

size_t dtype_size(uint32_t dt);

// Read-only view of a blob file. Every accessor checks the dtype and returns
// nullptr on a missing or mistyped section, so callers can report which
// section is wrong instead of reading garbage.
class Reader {
public:
    Reader() = default;
    ~Reader();
    Reader(const Reader&) = delete;
    Reader& operator=(const Reader&) = delete;

    // Returns an empty string on success, otherwise a one-line error.
    std::string open(const std::string& path);
    void close();

    const Section* find(const char* name) const;
    const void* data(const Section* s) const { return map_ + s->data_off; }
    uint64_t count(const char* name) const {
        const Section* s = find(name);
        return s ? s->count : 0;
    }
    template <class T> const T* get(const char* name, uint32_t dt) const {
        const Section* s = find(name);
        if (!s || s->dtype != dt) return nullptr;
        return reinterpret_cast<const T*>(data(s));
    }
    const double* f64(const char* n) const { return get<double>(n, F64); }
    const int64_t* i64(const char* n) const { return get<int64_t>(n, I64); }
    const int32_t* i32(const char* n) const { return get<int32_t>(n, I32); }
    const uint8_t* u8(const char* n) const { return get<uint8_t>(n, U8); }
    double f64_1(const char* n, double dflt) const {
        const double* p = f64(n);
        return p ? p[0] : dflt;
    }
    int64_t i64_1(const char* n, int64_t dflt) const {
        const int64_t* p = i64(n);
        return p ? p[0] : dflt;
    }
    const std::vector<Section>& sections() const { return sec_; }
    const std::string& path() const { return path_; }
    size_t size() const { return size_; }
    const uint8_t* base() const { return map_; }

private:
    const uint8_t* map_ = nullptr;
    size_t size_ = 0;
    std::vector<Section> sec_;
    std::string path_;
};

// Accumulates typed sections and writes one blob. Each section's data is
// 64-byte aligned (the format records every offset explicitly, so readers do
// not depend on the padding).
class Writer {
public:
    void add(const std::string& name, uint32_t dtype, const void* data, std::vector<uint64_t> shape);
    template <class T> void add_vec(const std::string& name, uint32_t dtype, const std::vector<T>& v) {
        add(name, dtype, v.data(), {static_cast<uint64_t>(v.size())});
    }
    void add_f64(const std::string& name, const std::vector<double>& v) { add_vec(name, F64, v); }
    void add_i32(const std::string& name, const std::vector<int32_t>& v) { add_vec(name, I32, v); }
    void add_i64(const std::string& name, const std::vector<int64_t>& v) { add_vec(name, I64, v); }
    void add_u8(const std::string& name, const std::vector<uint8_t>& v) { add_vec(name, U8, v); }
    void add_scalar(const std::string& name, double v) { add_f64(name, std::vector<double>{v}); }
    void add_str(const std::string& name, const std::string& s);
    // Returns an empty string on success.
    std::string write(const std::string& path) const;

private:
    struct Pending {
        std::string name;
        uint32_t dtype;
        std::vector<uint64_t> shape;
        std::vector<uint8_t> bytes;
    };
    std::vector<Pending> sec_;
};

}  // namespace sbb
