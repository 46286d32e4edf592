// SBB1 reader/writer (format described in sbb.h).
#include "sbb.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>

namespace sbb {

static const size_t kHeader = 52;
static const size_t kDirEntry = 56;

size_t dtype_size(uint32_t dt) {
    switch (dt) {
        case F64: case I64: return 8;
        case F32: case I32: case U32: return 4;
        case I8: case U8: case STR: return 1;
        default: return 0;
    }
}

static uint32_t rd32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }
static uint64_t rd64(const uint8_t* p) { uint64_t v; memcpy(&v, p, 8); return v; }

Reader::~Reader() { close(); }

void Reader::close() {
    if (map_) munmap(const_cast<uint8_t*>(map_), size_);
    map_ = nullptr;
    size_ = 0;
    sec_.clear();
}

std::string Reader::open(const std::string& path) {
    close();
    path_ = path;
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return "cannot open " + path;
    struct stat st;
    if (fstat(fd, &st) != 0) { ::close(fd); return "cannot stat " + path; }
    size_t size = static_cast<size_t>(st.st_size);
    if (size < kHeader) { ::close(fd); return "truncated header in " + path; }
    void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) return "mmap failed for " + path;
    map_ = static_cast<const uint8_t*>(m);
    size_ = size;
    if (memcmp(map_, "SBB1", 4) != 0) { close(); return "bad magic in " + path; }
    if (rd32(map_ + 4) != 1u) { close(); return "unsupported SBB version in " + path; }
    const uint32_t n_sec = rd32(map_ + 8);
    const uint64_t dir_off = rd64(map_ + 12);
    const uint64_t names_off = rd64(map_ + 20);
    const uint64_t names_len = rd64(map_ + 28);
    if (dir_off + (uint64_t)n_sec * kDirEntry > size || names_off + names_len > size) {
        close();
        return "directory or names run past the end of " + path;
    }
    sec_.resize(n_sec);
    for (uint32_t i = 0; i < n_sec; i++) {
        const uint8_t* e = map_ + dir_off + (size_t)i * kDirEntry;
        Section& s = sec_[i];
        uint32_t name_off = rd32(e);
        s.dtype = rd32(e + 4);
        s.ndim = rd32(e + 8);
        for (int k = 0; k < 4; k++) s.shape[k] = rd64(e + 16 + 8 * k);
        s.data_off = rd64(e + 48);
        if (name_off >= names_len || s.ndim > 4 || dtype_size(s.dtype) == 0) {
            close();
            return "corrupt directory entry " + std::to_string(i) + " in " + path;
        }
        const char* nm = reinterpret_cast<const char*>(map_ + names_off + name_off);
        size_t maxlen = names_len - name_off;
        s.name.assign(nm, strnlen(nm, maxlen));
        s.count = 1;
        for (uint32_t k = 0; k < s.ndim; k++) s.count *= s.shape[k];
        if (s.data_off + s.count * dtype_size(s.dtype) > size) {
            close();
            return "section " + s.name + " runs past the end of " + path;
        }
    }
    return "";
}

const Section* Reader::find(const char* name) const {
    for (const Section& s : sec_)
        if (s.name == name) return &s;
    return nullptr;
}

void Writer::add(const std::string& name, uint32_t dtype, const void* data, std::vector<uint64_t> shape) {
    Pending p;
    p.name = name;
    p.dtype = dtype;
    p.shape = std::move(shape);
    uint64_t cnt = 1;
    for (uint64_t d : p.shape) cnt *= d;
    size_t nb = (size_t)cnt * dtype_size(dtype);
    p.bytes.resize(nb);
    if (nb) memcpy(p.bytes.data(), data, nb);
    sec_.push_back(std::move(p));
}

void Writer::add_str(const std::string& name, const std::string& s) {
    add(name, STR, s.data(), {static_cast<uint64_t>(s.size())});
}

std::string Writer::write(const std::string& path) const {
    std::string names;
    std::vector<uint32_t> name_off;
    for (const Pending& p : sec_) {
        name_off.push_back((uint32_t)names.size());
        names += p.name;
        names.push_back('\0');
    }
    const uint64_t dir_off = kHeader;
    const uint64_t names_off = dir_off + kDirEntry * sec_.size();
    uint64_t cur = names_off + names.size();
    std::vector<uint64_t> data_off;
    for (const Pending& p : sec_) {
        cur = (cur + 63) & ~uint64_t(63);
        data_off.push_back(cur);
        cur += p.bytes.size();
    }
    const uint64_t total = cur;
    std::vector<uint8_t> out(total, 0);
    auto w32 = [&](size_t off, uint32_t v) { memcpy(&out[off], &v, 4); };
    auto w64 = [&](size_t off, uint64_t v) { memcpy(&out[off], &v, 8); };
    memcpy(&out[0], "SBB1", 4);
    w32(4, 1);
    w32(8, (uint32_t)sec_.size());
    w64(12, dir_off);
    w64(20, names_off);
    w64(28, names.size());
    w64(36, total);
    w64(44, 0);
    for (size_t i = 0; i < sec_.size(); i++) {
        const Pending& p = sec_[i];
        size_t e = dir_off + i * kDirEntry;
        w32(e, name_off[i]);
        w32(e + 4, p.dtype);
        w32(e + 8, (uint32_t)p.shape.size());
        w32(e + 12, 0);
        for (int k = 0; k < 4; k++) w64(e + 16 + 8 * k, k < (int)p.shape.size() ? p.shape[k] : 1);
        w64(e + 48, data_off[i]);
        if (!p.bytes.empty()) memcpy(&out[data_off[i]], p.bytes.data(), p.bytes.size());
    }
    memcpy(&out[names_off], names.data(), names.size());
    std::string tmp = path + ".tmp";
    FILE* f = fopen(tmp.c_str(), "wb");
    if (!f) return "cannot create " + tmp;
    size_t wr = fwrite(out.data(), 1, out.size(), f);
    if (fclose(f) != 0 || wr != out.size()) return "short write to " + tmp;
    if (rename(tmp.c_str(), path.c_str()) != 0) return "cannot rename " + tmp;
    return "";
}

}  // namespace sbb
