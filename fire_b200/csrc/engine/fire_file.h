// Read-only mmap of a .fire v1/v2 container with Fire's validation rules
// (src/model/fire_reader.cpp:100-385): 32-byte header, 96-byte records, v1 FP32
// payloads back to back, v2 payloads padded with zeros to 4 bytes, INT4 group
// metadata only on UInt8 qweight records. Malformed input is reported, never fatal.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace fb {

enum WireDType : uint8_t { kWireF32 = 1, kWireU8 = 2, kWireBF16 = 3 };

struct FireTensor {
    std::string name;
    uint8_t dtype = 0;
    std::vector<int64_t> shape;
    uint64_t offset = 0;
    uint64_t size = 0;
    uint32_t group_size = 0;  // INT4 group size on qweight records, else 0
    const uint8_t* data = nullptr;
};

class FireFile {
  public:
    FireFile() = default;
    ~FireFile();
    FireFile(const FireFile&) = delete;
    FireFile& operator=(const FireFile&) = delete;

    // Returns true on success; otherwise *err says why.
    bool open(const std::string& path, std::string* err);
    const FireTensor* find(const std::string& name) const;
    size_t count() const { return tensors_.size(); }
    uint32_t version() const { return version_; }
    const std::vector<FireTensor>& tensors() const { return tensors_; }

  private:
    void close();
    void* map_ = nullptr;
    size_t map_size_ = 0;
    uint32_t version_ = 0;
    std::vector<FireTensor> tensors_;
    std::unordered_map<std::string, size_t> index_;
};

}  // namespace fb
