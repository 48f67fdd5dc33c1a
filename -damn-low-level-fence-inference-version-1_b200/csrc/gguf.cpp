// gguf.cpp — GGUF v2/v3 reader (see gguf.h). File-format steps follow the GGUF specification in
// the order the reference parser uses them (src/gguf/gguf_parser.cpp:143-350): header, metadata
// key/values (general.alignment honoured, 0 ignored), tensor infos (<= 4 dims), data start
// aligned up from the end of the infos, tensor size = ceil(n_elements / block) * type_size.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <stdexcept>

namespace fence {

GGMLTypeInfo ggml_type_info(GGMLType t) {
    switch (t) {
        case GGMLType::F32: return {1, 4};
        case GGMLType::F16: return {1, 2};
        case GGMLType::BF16: return {1, 2};
        case GGMLType::Q4_0: return {32, 18};
        case GGMLType::Q4_1: return {32, 20};
        case GGMLType::Q5_0: return {32, 22};
        case GGMLType::Q5_1: return {32, 24};
        case GGMLType::Q8_0: return {32, 34};
        case GGMLType::Q8_1: return {32, 40};
        case GGMLType::Q2_K: return {256, 84};
        case GGMLType::Q3_K: return {256, 110};
        case GGMLType::Q4_K: return {256, 144};
        case GGMLType::Q5_K: return {256, 176};
        case GGMLType::Q6_K: return {256, 210};
        case GGMLType::Q8_K: return {256, 292};
        case GGMLType::I8: return {1, 1};
        case GGMLType::I16: return {1, 2};
        case GGMLType::I32: return {1, 4};
        case GGMLType::I64: return {1, 8};
        case GGMLType::F64: return {1, 8};
        default:
            // same fallback as the reference (gguf_parser.cpp:47-50): warn, treat as F32
            fprintf(stderr, "WARNING: unknown GGMLType %u, assuming F32\n", (unsigned)t);
            return {1, 4};
    }
}

const char* ggml_type_name(GGMLType t) {
    switch (t) {
        case GGMLType::F32: return "F32";
        case GGMLType::F16: return "F16";
        case GGMLType::BF16: return "BF16";
        case GGMLType::Q4_0: return "Q4_0";
        case GGMLType::Q4_1: return "Q4_1";
        case GGMLType::Q5_0: return "Q5_0";
        case GGMLType::Q5_1: return "Q5_1";
        case GGMLType::Q8_0: return "Q8_0";
        case GGMLType::Q8_1: return "Q8_1";
        case GGMLType::Q2_K: return "Q2_K";
        case GGMLType::Q3_K: return "Q3_K";
        case GGMLType::Q4_K: return "Q4_K";
        case GGMLType::Q5_K: return "Q5_K";
        case GGMLType::Q6_K: return "Q6_K";
        case GGMLType::Q8_K: return "Q8_K";
        case GGMLType::I8: return "I8";
        case GGMLType::I16: return "I16";
        case GGMLType::I32: return "I32";
        case GGMLType::I64: return "I64";
        case GGMLType::F64: return "F64";
        default: return "UNKNOWN";
    }
}

namespace {
// Bounds-checked little-endian reader over the mapping.
struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    template <typename T>
    T get() {
        if ((size_t)(end - p) < sizeof(T)) throw std::runtime_error("GGUF: unexpected end of file");
        T v;
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if ((uint64_t)(end - p) < n) throw std::runtime_error("GGUF: string runs past end of file");
        std::string s(reinterpret_cast<const char*>(p), (size_t)n);
        p += n;
        return s;
    }
    void skip(GGUFValueType t) {
        static const int sizes[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        const uint32_t ti = (uint32_t)t;
        if (ti == (uint32_t)GGUFValueType::STRING) {
            const uint64_t n = get<uint64_t>();
            if ((uint64_t)(end - p) < n) throw std::runtime_error("GGUF: string runs past end of file");
            p += n;
        } else if (ti == (uint32_t)GGUFValueType::ARRAY) {
            const auto at = get<GGUFValueType>();
            const uint64_t n = get<uint64_t>();
            for (uint64_t i = 0; i < n; ++i) skip(at);
        } else if (ti < 13) {
            if ((size_t)(end - p) < (size_t)sizes[ti]) throw std::runtime_error("GGUF: unexpected end of file");
            p += sizes[ti];
        } else {
            throw std::runtime_error("GGUF: unknown value type " + std::to_string(ti));
        }
    }
};
}  // namespace

bool GGUFFile::fail(const std::string& msg) {
    err_ = msg;
    fprintf(stderr, "%s\n", msg.c_str());
    close();
    err_ = msg;
    return false;
}

bool GGUFFile::open(const std::string& path) {
    if (map_) close();
    path_ = path;
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) return fail("GGUF: cannot open '" + path + "': " + strerror(errno));
    struct stat st;
    if (fstat(fd_, &st) < 0) return fail(std::string("GGUF: fstat failed: ") + strerror(errno));
    size_ = (size_t)st.st_size;
    if (size_ == 0) return fail("GGUF: file is empty");
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) return fail(std::string("GGUF: mmap failed: ") + strerror(errno));
    map_ = m;
    madvise(map_, size_, MADV_SEQUENTIAL);
    const uint8_t* base = static_cast<const uint8_t*>(map_);
    bool ok;
    try {
        ok = parse(base, base + size_);
    } catch (const std::exception& ex) {
        return fail(std::string("GGUF: parse error: ") + ex.what());
    }
    if (!ok) return false;
    madvise(map_, size_, MADV_RANDOM);
    return true;
}

bool GGUFFile::parse(const uint8_t* base, const uint8_t* end) {
    Cursor c{base, end};
    const uint32_t magic = c.get<uint32_t>();
    if (magic != 0x46554747u) {
        char b[96];
        snprintf(b, sizeof b, "GGUF: invalid magic 0x%08X (expected 0x46554747 'GGUF')", magic);
        return fail(b);
    }
    version_ = c.get<uint32_t>();
    if (version_ < 2 || version_ > 3)
        return fail("GGUF: unsupported version " + std::to_string(version_) + " (expected 2 or 3)");
    n_tensors_ = c.get<uint64_t>();
    n_kv_ = c.get<uint64_t>();

    kv_.reserve((size_t)std::min<uint64_t>(n_kv_, 1u << 16));
    for (uint64_t i = 0; i < n_kv_; ++i) {
        GGUFMetadataKV kv;
        kv.key = c.str();
        kv.type = c.get<GGUFValueType>();
        bool stored = true;
        switch (kv.type) {
            case GGUFValueType::UINT8: kv.value = c.get<uint8_t>(); break;
            case GGUFValueType::INT8: kv.value = c.get<int8_t>(); break;
            case GGUFValueType::UINT16: kv.value = c.get<uint16_t>(); break;
            case GGUFValueType::INT16: kv.value = c.get<int16_t>(); break;
            case GGUFValueType::UINT32: kv.value = c.get<uint32_t>(); break;
            case GGUFValueType::INT32: kv.value = c.get<int32_t>(); break;
            case GGUFValueType::FLOAT32: kv.value = c.get<float>(); break;
            case GGUFValueType::BOOL: kv.value = (bool)(c.get<uint8_t>() != 0); break;
            case GGUFValueType::STRING: kv.value = c.str(); break;
            case GGUFValueType::UINT64: kv.value = c.get<uint64_t>(); break;
            case GGUFValueType::INT64: kv.value = c.get<int64_t>(); break;
            case GGUFValueType::FLOAT64: kv.value = c.get<double>(); break;
            case GGUFValueType::ARRAY: {
                const auto at = c.get<GGUFValueType>();
                const uint64_t n = c.get<uint64_t>();
                if (at == GGUFValueType::STRING) {
                    std::vector<std::string> v;
                    v.reserve((size_t)std::min<uint64_t>(n, 1u << 20));
                    for (uint64_t k = 0; k < n; ++k) v.push_back(c.str());
                    str_arrays_[kv.key] = std::move(v);
                } else {
                    for (uint64_t k = 0; k < n; ++k) c.skip(at);
                }
                stored = false;
                break;
            }
            default:
                return fail("GGUF: unknown metadata value type " + std::to_string((uint32_t)kv.type) +
                            " for key '" + kv.key + "'");
        }
        if (stored && kv.key == "general.alignment" && kv.type == GGUFValueType::UINT32) {
            const uint32_t a = std::get<uint32_t>(kv.value);
            if (a == 0)
                fprintf(stderr, "GGUF: general.alignment is 0, ignoring (keeping default %u)\n", alignment_);
            else
                alignment_ = a;
        }
        if (stored) {
            kv_index_[kv.key] = kv_.size();
            kv_.push_back(std::move(kv));
        }
    }

    tensors_.reserve((size_t)std::min<uint64_t>(n_tensors_, 1u << 20));
    for (uint64_t i = 0; i < n_tensors_; ++i) {
        GGUFTensorInfo ti;
        ti.name = c.str();
        ti.n_dims = c.get<uint32_t>();
        if (ti.n_dims > 4)
            return fail("GGUF: tensor '" + ti.name + "' has " + std::to_string(ti.n_dims) + " dims (max 4)");
        for (uint32_t d = 0; d < ti.n_dims; ++d) ti.dims[d] = c.get<uint64_t>();
        ti.type = c.get<GGMLType>();
        ti.offset = c.get<uint64_t>();
        tensor_index_[ti.name] = tensors_.size();
        tensors_.push_back(std::move(ti));
    }

    const size_t header_end = (size_t)(c.p - base);
    data_off_ = header_end + (alignment_ - header_end % alignment_) % alignment_;
    for (auto& ti : tensors_) {
        const GGMLTypeInfo info = ggml_type_info(ti.type);
        const uint64_t n = ti.n_elements();
        const uint64_t nbytes = (n + info.block_size - 1) / info.block_size * info.type_size;
        const uint64_t abs = (uint64_t)data_off_ + ti.offset;
        if (abs >= size_ || nbytes > size_ - abs) {
            char b[256];
            snprintf(b, sizeof b, "GGUF: tensor '%s' data [%llu, %llu) exceeds file size %zu", ti.name.c_str(),
                     (unsigned long long)abs, (unsigned long long)(abs + nbytes), size_);
            return fail(b);
        }
        ti.data = base + abs;
        ti.data_size_bytes = (size_t)nbytes;
    }
    return true;
}

void GGUFFile::close() {
    if (map_) munmap(map_, size_);
    map_ = nullptr;
    if (fd_ >= 0) ::close(fd_);
    fd_ = -1;
    size_ = 0;
    data_off_ = 0;
    version_ = 0;
    n_tensors_ = n_kv_ = 0;
    alignment_ = 32;
    kv_.clear();
    tensors_.clear();
    kv_index_.clear();
    tensor_index_.clear();
    str_arrays_.clear();
}

GGUFFile::~GGUFFile() { close(); }
GGUFFile::GGUFFile(GGUFFile&& o) noexcept { *this = std::move(o); }
GGUFFile& GGUFFile::operator=(GGUFFile&& o) noexcept {
    if (this != &o) {
        close();
        path_ = std::move(o.path_);
        err_ = std::move(o.err_);
        map_ = o.map_;
        o.map_ = nullptr;
        size_ = o.size_;
        o.size_ = 0;
        fd_ = o.fd_;
        o.fd_ = -1;
        version_ = o.version_;
        n_tensors_ = o.n_tensors_;
        n_kv_ = o.n_kv_;
        alignment_ = o.alignment_;
        data_off_ = o.data_off_;
        kv_ = std::move(o.kv_);
        tensors_ = std::move(o.tensors_);
        kv_index_ = std::move(o.kv_index_);
        tensor_index_ = std::move(o.tensor_index_);
        str_arrays_ = std::move(o.str_arrays_);
    }
    return *this;
}

const GGUFTensorInfo* GGUFFile::find_tensor(const std::string& name) const {
    auto it = tensor_index_.find(name);
    return it == tensor_index_.end() ? nullptr : &tensors_[it->second];
}
const GGUFMetadataKV* GGUFFile::find_metadata(const std::string& key) const {
    auto it = kv_index_.find(key);
    return it == kv_index_.end() ? nullptr : &kv_[it->second];
}
const std::vector<std::string>* GGUFFile::get_string_array(const std::string& key) const {
    auto it = str_arrays_.find(key);
    return it == str_arrays_.end() ? nullptr : &it->second;
}

namespace {
template <typename T>
T typed_get(const GGUFFile& f, const std::string& key, GGUFValueType want, const char* tname) {
    const GGUFMetadataKV* kv = f.find_metadata(key);
    if (!kv) throw std::runtime_error("GGUF: metadata key not found: " + key);
    if (kv->type != want) throw std::runtime_error("GGUF: key '" + key + "' is not " + tname);
    return std::get<T>(kv->value);
}
}  // namespace

std::string GGUFFile::get_string(const std::string& k) const {
    return typed_get<std::string>(*this, k, GGUFValueType::STRING, "a string");
}
uint32_t GGUFFile::get_u32(const std::string& k) const { return typed_get<uint32_t>(*this, k, GGUFValueType::UINT32, "u32"); }
int32_t GGUFFile::get_i32(const std::string& k) const { return typed_get<int32_t>(*this, k, GGUFValueType::INT32, "i32"); }
float GGUFFile::get_f32(const std::string& k) const { return typed_get<float>(*this, k, GGUFValueType::FLOAT32, "f32"); }
bool GGUFFile::get_bool(const std::string& k) const { return typed_get<bool>(*this, k, GGUFValueType::BOOL, "bool"); }
uint64_t GGUFFile::get_u64(const std::string& k) const { return typed_get<uint64_t>(*this, k, GGUFValueType::UINT64, "u64"); }

}  // namespace fence
