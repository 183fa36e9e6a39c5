#include "engine/fire_file.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace fb {

namespace {
uint32_t u32(const uint8_t* p) { uint32_t v; std::memcpy(&v, p, 4); return v; }
uint64_t u64(const uint8_t* p) { uint64_t v; std::memcpy(&v, p, 8); return v; }
constexpr size_t kHeader = 32, kRecord = 96;
}  // namespace

FireFile::~FireFile() { close(); }

void FireFile::close() {
    if (map_ != nullptr) munmap(map_, map_size_);
    map_ = nullptr;
    map_size_ = 0;
    tensors_.clear();
    index_.clear();
}

bool FireFile::open(const std::string& path, std::string* err) {
    close();
    auto fail = [&](const std::string& m) { if (err) *err = "FireFile: " + m; close(); return false; };
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return fail("cannot open " + path);
    struct stat st;
    if (fstat(fd, &st) != 0) { ::close(fd); return fail("cannot stat " + path); }
    const size_t size = static_cast<size_t>(st.st_size);
    if (size < kHeader) { ::close(fd); return fail("file shorter than the header"); }
    void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) return fail("mmap failed");
    map_ = m;
    map_size_ = size;
    const uint8_t* d = static_cast<const uint8_t*>(m);
    if (std::memcmp(d, "FIRECKPT", 8) != 0) return fail("bad magic");
    version_ = u32(d + 8);
    if (version_ != 1 && version_ != 2) return fail("unsupported format version");
    const uint64_t count = u32(d + 12), dir = u64(d + 16), data = u64(d + 24);
    if (dir != kHeader || data != kHeader + kRecord * count || data > size) return fail("bad directory");
    uint64_t expect = data;
    tensors_.reserve(count);
    for (uint64_t i = 0; i < count; ++i) {
        const uint8_t* r = d + kHeader + i * kRecord;
        FireTensor t;
        const char* nm = reinterpret_cast<const char*>(r);
        const size_t len = strnlen(nm, 64);
        if (len == 0 || len == 64) return fail("bad tensor name");
        t.name.assign(nm, len);
        for (size_t j = len; j < 64; ++j)
            if (r[j] != 0) return fail("name padding not zero: " + t.name);
        t.offset = u64(r + 64);
        t.size = u64(r + 72);
        const uint32_t s0 = u32(r + 80), s1 = u32(r + 84);
        t.dtype = r[88];
        const uint8_t nd = r[89];
        const uint8_t kind = r[90];
        const uint32_t group = u32(r + 91);
        const uint8_t reserved = r[95];
        if (t.dtype != kWireF32 && t.dtype != kWireU8 && t.dtype != kWireBF16) return fail("bad dtype: " + t.name);
        if (version_ == 1 && t.dtype != kWireF32) return fail("v1 holds FP32 only: " + t.name);
        if ((nd != 1 && nd != 2) || s0 == 0 || (nd == 2 && s1 == 0) || (nd == 1 && s1 != 0))
            return fail("bad shape: " + t.name);
        t.shape = nd == 1 ? std::vector<int64_t>{s0} : std::vector<int64_t>{s0, s1};
        if (kind == 0) {
            if (group != 0 || reserved != 0) return fail("bad metadata: " + t.name);
        } else if (version_ == 2 && kind == 1 && t.dtype == kWireU8 && group != 0 && group % 2 == 0 &&
                   reserved == 0 && nd == 2 && (uint64_t(s1) * 2) % group == 0) {
            t.group_size = group;
        } else {
            return fail("invalid quantization metadata: " + t.name);
        }
        const uint64_t esize = t.dtype == kWireF32 ? 4 : (t.dtype == kWireBF16 ? 2 : 1);
        if (t.size != uint64_t(s0) * (nd == 2 ? s1 : 1) * esize) return fail("byte size mismatch: " + t.name);
        uint64_t aligned = expect;
        if (version_ == 2) aligned = (expect + 3) & ~uint64_t(3);
        if (t.offset != aligned || t.offset + t.size > size) return fail("bad payload range: " + t.name);
        for (uint64_t o = expect; o < aligned; ++o)
            if (d[o] != 0) return fail("alignment padding not zero: " + t.name);
        t.data = d + t.offset;
        expect = t.offset + t.size;
        if (index_.count(t.name)) return fail("duplicate tensor: " + t.name);
        index_[t.name] = tensors_.size();
        tensors_.push_back(std::move(t));
    }
    return true;
}

const FireTensor* FireFile::find(const std::string& name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}

}  // namespace fb
