// gguf.cpp — GGUF v3 reader/writer (see gguf.h).
#include "gguf.h"

#include <cerrno>
#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace z2b {

bool gtype_info(uint32_t t, int* be, int* bb) {
    switch (t) {
        case GT_F32:  *be = 1;   *bb = 4;   return true;
        case GT_F16:  *be = 1;   *bb = 2;   return true;
        case GT_BF16: *be = 1;   *bb = 2;   return true;
        case GT_Q8_0: *be = 32;  *bb = 34;  return true;
        case GT_Q4_K: *be = 256; *bb = 144; return true;
        case GT_Q6_K: *be = 256; *bb = 210; return true;
        default: return false;
    }
}

const char* gtype_name(uint32_t t) {
    switch (t) {
        case GT_F32: return "f32"; case GT_F16: return "f16"; case GT_BF16: return "bf16";
        case GT_Q8_0: return "q8_0"; case GT_Q4_K: return "q4_k"; case GT_Q6_K: return "q6_k";
        default: return "unsupported";
    }
}

size_t gtype_row_bytes(uint32_t t, int64_t ne0) {
    int be = 0, bb = 0;
    if (!gtype_info(t, &be, &bb) || ne0 % be) return 0;
    return (size_t)(ne0 / be) * (size_t)bb;
}

uint16_t f32_to_f16(float f) {
    uint32_t x; std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));   // inf / nan
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);                                // overflow -> inf
    if (e <= 0) {                                                                   // subnormal / zero
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const int shift = 14 - e;                                                  // 1 - e + 13
        uint32_t h = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;                         // may carry into exp
    return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) x = sign;
        else {
            int e = -1;
            do { e++; man <<= 1; } while (!(man & 0x400u));
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f; std::memcpy(&f, &x, 4);
    return f;
}

// ---------------------------------------------------------------- reader

namespace {
struct Cursor {
    const uint8_t* p; const uint8_t* end; bool ok = true;
    template <class T> T get() {
        T v{};
        if ((size_t)(end - p) < sizeof(T)) { ok = false; return v; }
        std::memcpy(&v, p, sizeof(T)); p += sizeof(T); return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || (uint64_t)(end - p) < n) { ok = false; return {}; }
        std::string s((const char*)p, (size_t)n); p += n; return s;
    }
};

bool read_scalar(Cursor& c, uint32_t type, GKV& kv, bool into_array) {
    int64_t iv = 0; double fv = 0.0; bool is_int = true;
    switch (type) {
        case GV_U8:  iv = c.get<uint8_t>(); break;
        case GV_I8:  iv = c.get<int8_t>(); break;
        case GV_U16: iv = c.get<uint16_t>(); break;
        case GV_I16: iv = c.get<int16_t>(); break;
        case GV_U32: iv = c.get<uint32_t>(); break;
        case GV_I32: iv = c.get<int32_t>(); break;
        case GV_U64: iv = (int64_t)c.get<uint64_t>(); break;
        case GV_I64: iv = c.get<int64_t>(); break;
        case GV_BOOL: iv = c.get<uint8_t>(); break;
        case GV_F32: fv = c.get<float>(); is_int = false; break;
        case GV_F64: fv = c.get<double>(); is_int = false; break;
        case GV_STR: {
            std::string s = c.str();
            if (!into_array) kv.s = s;
            return c.ok;
        }
        default: return false;
    }
    if (into_array) { if (is_int) kv.ai.push_back(iv); else kv.af.push_back(fv); }
    else { kv.u = (uint64_t)iv; kv.f = is_int ? (double)iv : fv; }
    return c.ok;
}
}  // namespace

GGUFFile::~GGUFFile() {
    if (map_) munmap(map_, size_);
    if (fd_ >= 0) close(fd_);
}

bool GGUFFile::open(const char* path, std::string& err) {
    fd_ = ::open(path, O_RDONLY);
    if (fd_ < 0) { err = std::string("cannot open '") + path + "': " + strerror(errno); return false; }
    struct stat st;
    if (fstat(fd_, &st) != 0) { err = "fstat failed"; return false; }
    size_ = (size_t)st.st_size;
    if (size_ < 24) { err = "file too small for a GGUF header"; return false; }
    map_ = (uint8_t*)mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (map_ == MAP_FAILED) { map_ = nullptr; err = "mmap failed"; return false; }
    Cursor c{map_, map_ + size_};
    if (c.get<uint32_t>() != 0x46554747u) { err = "bad magic (not a GGUF file)"; return false; }
    const uint32_t version = c.get<uint32_t>();
    if (version != 3 && version != 2) { err = "unsupported GGUF version " + std::to_string(version); return false; }
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    if (n_tensors > (1u << 20) || n_kv > (1u << 20)) { err = "implausible tensor/kv count"; return false; }
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        std::string key = c.str();
        GKV kv; kv.type = c.get<uint32_t>();
        if (kv.type == GV_ARR) {
            kv.arr_type = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            if (n > size_) { err = "implausible array length"; return false; }
            for (uint64_t j = 0; j < n && c.ok; ++j)
                if (!read_scalar(c, kv.arr_type, kv, true)) { err = "bad array element in '" + key + "'"; return false; }
        } else if (!read_scalar(c, kv.type, kv, false)) {
            err = "bad value for key '" + key + "'"; return false;
        }
        kvs_[key] = kv;
    }
    if (const GKV* a = kv("general.alignment")) alignment_ = (uint32_t)a->u;
    if (alignment_ == 0 || (alignment_ & (alignment_ - 1))) { err = "bad alignment"; return false; }
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        GTensor t;
        t.name = c.str();
        t.n_dims = (int)c.get<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) { err = "bad n_dims for '" + t.name + "'"; return false; }
        for (int d = 0; d < t.n_dims; ++d) t.ne[d] = (int64_t)c.get<uint64_t>();
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        tensors_.push_back(t);
    }
    if (!c.ok) { err = "truncated GGUF header"; return false; }
    const size_t hdr = (size_t)(c.p - map_);
    const size_t data_start = (hdr + alignment_ - 1) / alignment_ * alignment_;
    for (size_t i = 0; i < tensors_.size(); ++i) {
        GTensor& t = tensors_[i];
        int be = 0, bb = 0;
        if (!gtype_info(t.type, &be, &bb)) { t.nbytes = 0; t.data = nullptr; index_[t.name] = i; continue; }
        if (t.ne[0] % be) { err = "row length not a multiple of the block for '" + t.name + "'"; return false; }
        t.nbytes = (size_t)(t.nelements() / be) * (size_t)bb;
        if (data_start + t.offset + t.nbytes > size_) { err = "tensor '" + t.name + "' runs past end of file"; return false; }
        t.data = map_ + data_start + t.offset;
        index_[t.name] = i;
    }
    return true;
}

const GKV* GGUFFile::kv(const std::string& key) const {
    auto it = kvs_.find(key);
    return it == kvs_.end() ? nullptr : &it->second;
}

const GTensor* GGUFFile::tensor(const std::string& name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}

// ---------------------------------------------------------------- writer

void GGUFWriter::add_u32(const std::string& k, uint32_t v) { GKV kv; kv.type = GV_U32; kv.u = v; kv_.push_back({k, kv}); }
void GGUFWriter::add_f32(const std::string& k, float v) { GKV kv; kv.type = GV_F32; kv.f = v; kv_.push_back({k, kv}); }
void GGUFWriter::add_str(const std::string& k, const std::string& v) { GKV kv; kv.type = GV_STR; kv.s = v; kv_.push_back({k, kv}); }
void GGUFWriter::add_arr_i32(const std::string& k, const std::vector<int32_t>& v) {
    GKV kv; kv.type = GV_ARR; kv.arr_type = GV_I32;
    for (int32_t x : v) kv.ai.push_back(x);
    kv_.push_back({k, kv});
}

int GGUFWriter::add_tensor(const std::string& name, uint32_t type, int n_dims, const int64_t* ne) {
    Item it; it.name = name; it.type = type; it.n_dims = n_dims;
    int64_t n = 1;
    for (int d = 0; d < 4; ++d) { it.ne[d] = d < n_dims ? ne[d] : 1; n *= it.ne[d]; }
    int be = 1, bb = 4;
    gtype_info(type, &be, &bb);
    it.nbytes = (size_t)(n / be) * (size_t)bb;
    it.off = 0;
    items_.push_back(it);
    return (int)items_.size() - 1;
}

namespace {
void put_str(std::vector<uint8_t>& b, const std::string& s) {
    const uint64_t n = s.size();
    b.insert(b.end(), (const uint8_t*)&n, (const uint8_t*)&n + 8);
    b.insert(b.end(), s.begin(), s.end());
}
template <class T> void put(std::vector<uint8_t>& b, T v) { b.insert(b.end(), (const uint8_t*)&v, (const uint8_t*)&v + sizeof(T)); }
}  // namespace

bool GGUFWriter::begin(const char* path, std::string& err) {
    std::vector<uint8_t> b;
    put<uint32_t>(b, 0x46554747u);
    put<uint32_t>(b, 3);
    put<uint64_t>(b, items_.size());
    put<uint64_t>(b, kv_.size());
    for (auto& kv : kv_) {
        put_str(b, kv.first);
        put<uint32_t>(b, kv.second.type);
        switch (kv.second.type) {
            case GV_U32: put<uint32_t>(b, (uint32_t)kv.second.u); break;
            case GV_F32: put<float>(b, (float)kv.second.f); break;
            case GV_STR: put_str(b, kv.second.s); break;
            case GV_ARR:
                put<uint32_t>(b, kv.second.arr_type);
                put<uint64_t>(b, kv.second.ai.size());
                for (int64_t x : kv.second.ai) put<int32_t>(b, (int32_t)x);
                break;
            default: err = "writer: unsupported kv type"; return false;
        }
    }
    uint64_t off = 0;
    for (auto& it : items_) {
        it.off = off;
        off += (it.nbytes + alignment_ - 1) / alignment_ * alignment_;
        put_str(b, it.name);
        put<uint32_t>(b, (uint32_t)it.n_dims);
        for (int d = 0; d < it.n_dims; ++d) put<uint64_t>(b, (uint64_t)it.ne[d]);
        put<uint32_t>(b, it.type);
        put<uint64_t>(b, it.off);
    }
    data_start_ = (b.size() + alignment_ - 1) / alignment_ * alignment_;
    b.resize(data_start_, 0);
    fd_ = ::open(path, O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd_ < 0) { err = std::string("cannot create '") + path + "': " + strerror(errno); return false; }
    if (ftruncate(fd_, (off_t)(data_start_ + off)) != 0) { err = "ftruncate failed"; return false; }
    if (pwrite(fd_, b.data(), b.size(), 0) != (ssize_t)b.size()) { err = "header write failed"; return false; }
    return true;
}

bool GGUFWriter::write_tensor(int idx, const void* data, size_t nbytes, size_t at, std::string& err) {
    const Item& it = items_[idx];
    if (at + nbytes > it.nbytes) { err = "write past tensor end: " + it.name; return false; }
    const uint8_t* p = (const uint8_t*)data;
    size_t done = 0;
    while (done < nbytes) {
        ssize_t w = pwrite(fd_, p + done, nbytes - done, (off_t)(data_start_ + it.off + at + done));
        if (w <= 0) { err = "tensor write failed: " + it.name; return false; }
        done += (size_t)w;
    }
    return true;
}

bool GGUFWriter::finish(std::string& err) {
    if (fd_ >= 0 && close(fd_) != 0) { err = "close failed"; fd_ = -1; return false; }
    fd_ = -1;
    return true;
}

}  // namespace z2b
