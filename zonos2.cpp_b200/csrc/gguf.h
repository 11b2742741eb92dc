// gguf.h — ggml-free GGUF v3 reader (mmap) and writer.
//
// Replaces the gguf_* / ggml context calls of the reference loader
// (src/zonos2.cpp:15-121): header, metadata key/values, tensor index and the
// aligned data section. ggml's `ne` order is kept: ne[0] is the contiguous
// (row) dimension, so a numpy array of shape [E, rows, K] has ne = {K, rows, E}.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace z2b {

// ggml_type values used by zonos2 files (ggml/include/ggml.h numbering).
enum GType : uint32_t {
    GT_F32 = 0, GT_F16 = 1, GT_Q8_0 = 8, GT_Q4_K = 12, GT_Q6_K = 14, GT_BF16 = 30,
};

// Bytes per block and weights per block of the supported storage types.
bool gtype_info(uint32_t t, int* block_elems, int* block_bytes);
const char* gtype_name(uint32_t t);
// Row size in bytes for `ne0` weights of type t (ne0 must be a multiple of the block).
size_t gtype_row_bytes(uint32_t t, int64_t ne0);

enum GVal : uint32_t {
    GV_U8 = 0, GV_I8 = 1, GV_U16 = 2, GV_I16 = 3, GV_U32 = 4, GV_I32 = 5, GV_F32 = 6,
    GV_BOOL = 7, GV_STR = 8, GV_ARR = 9, GV_U64 = 10, GV_I64 = 11, GV_F64 = 12,
};

struct GKV {
    uint32_t type = 0;          // GVal
    uint32_t arr_type = 0;      // element type when type == GV_ARR
    uint64_t u = 0;             // integer / bool scalar
    double f = 0.0;             // float scalar
    std::string s;              // string scalar
    std::vector<int64_t> ai;    // integer array
    std::vector<double> af;     // float array
};

struct GTensor {
    std::string name;
    uint32_t type = 0;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;        // relative to the data section
    const uint8_t* data = nullptr;
    size_t nbytes = 0;
    int64_t nelements() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
};

class GGUFFile {
public:
    ~GGUFFile();
    // Parses the file; returns false and sets err on malformed input.
    bool open(const char* path, std::string& err);
    const GKV* kv(const std::string& key) const;
    const GTensor* tensor(const std::string& name) const;
    const std::vector<GTensor>& tensors() const { return tensors_; }
    uint32_t alignment() const { return alignment_; }
private:
    int fd_ = -1;
    uint8_t* map_ = nullptr;
    size_t size_ = 0;
    uint32_t alignment_ = 32;
    std::map<std::string, GKV> kvs_;
    std::vector<GTensor> tensors_;
    std::map<std::string, size_t> index_;
};

// Streaming writer: declare KVs and tensors (name, type, ne, byte size), then
// write the header and fill each tensor's bytes at its final file offset.
class GGUFWriter {
public:
    void add_u32(const std::string& k, uint32_t v);
    void add_f32(const std::string& k, float v);
    void add_str(const std::string& k, const std::string& v);
    void add_arr_i32(const std::string& k, const std::vector<int32_t>& v);
    // Returns the tensor's index.
    int add_tensor(const std::string& name, uint32_t type, int n_dims, const int64_t* ne);
    // Lays out offsets and writes the header; afterwards tensor data may be written.
    bool begin(const char* path, std::string& err);
    bool write_tensor(int idx, const void* data, size_t nbytes, size_t at, std::string& err);
    size_t tensor_bytes(int idx) const { return items_[idx].nbytes; }
    bool finish(std::string& err);
private:
    struct Item { std::string name; uint32_t type; int n_dims; int64_t ne[4]; size_t nbytes; uint64_t off; };
    std::vector<std::pair<std::string, GKV>> kv_;
    std::vector<Item> items_;
    int fd_ = -1;
    uint64_t data_start_ = 0;
    uint32_t alignment_ = 32;
};

// IEEE half <-> float (round-to-nearest-even), host side.
uint16_t f32_to_f16(float f);
float f16_to_f32(uint16_t h);

}  // namespace z2b
