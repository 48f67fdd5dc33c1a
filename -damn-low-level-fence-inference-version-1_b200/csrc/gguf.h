// gguf.h — zero-copy mmap GGUF v2/v3 reader with the reference's GGUFFile contract
// (src/gguf/gguf_parser.h:27-217): same type enums, tensor-info fields, lookups and strictly typed
// metadata getters that throw std::runtime_error on a missing key or a type mismatch.
//
// Differences, all stricter: every tensor's data range must lie inside the file (the reference
// checks only the start offset, gguf_parser.cpp:331), and string arrays are kept (the reference
// skips all arrays) so the CLI can read tokenizer.ggml.tokens.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <variant>
#include <vector>

namespace fence {

enum class GGMLType : uint32_t {
    F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q8_1 = 9,
    Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, Q8_K = 15,
    IQ2_XXS = 16, IQ2_XS = 17, IQ3_XXS = 18, IQ1_S = 19, IQ4_NL = 20, IQ3_S = 21, IQ2_S = 22,
    IQ4_XS = 23, I8 = 24, I16 = 25, I32 = 26, I64 = 27, F64 = 28, IQ1_M = 29, BF16 = 30,
    TQ1_0 = 34, TQ2_0 = 35, MXFP4 = 39,
};

enum class GGUFValueType : uint32_t {
    UINT8 = 0, INT8 = 1, UINT16 = 2, INT16 = 3, UINT32 = 4, INT32 = 5, FLOAT32 = 6, BOOL = 7,
    STRING = 8, ARRAY = 9, UINT64 = 10, INT64 = 11, FLOAT64 = 12,
};

struct GGMLTypeInfo {
    uint32_t block_size;  // elements per block
    uint32_t type_size;   // bytes per block
};
GGMLTypeInfo ggml_type_info(GGMLType t);
const char* ggml_type_name(GGMLType t);

struct GGUFTensorInfo {
    std::string name;
    uint32_t n_dims = 0;
    uint64_t dims[4] = {1, 1, 1, 1};
    GGMLType type = GGMLType::F32;
    uint64_t offset = 0;           // relative to the tensor-data start
    const void* data = nullptr;    // into the mapping
    size_t data_size_bytes = 0;
    uint64_t n_elements() const {
        uint64_t n = 1;
        for (uint32_t i = 0; i < n_dims; ++i) n *= dims[i];
        return n;
    }
};

using GGUFMetadataValue = std::variant<uint8_t, int8_t, uint16_t, int16_t, uint32_t, int32_t, float,
                                       bool, std::string, uint64_t, int64_t, double>;

struct GGUFMetadataKV {
    std::string key;
    GGUFValueType type;
    GGUFMetadataValue value;
};

class GGUFFile {
public:
    GGUFFile() = default;
    ~GGUFFile();
    GGUFFile(const GGUFFile&) = delete;
    GGUFFile& operator=(const GGUFFile&) = delete;
    GGUFFile(GGUFFile&& o) noexcept;
    GGUFFile& operator=(GGUFFile&& o) noexcept;

    bool open(const std::string& path);  // false on error, reason on stderr and in last_error()
    void close();
    bool is_open() const { return map_ != nullptr; }

    uint32_t version() const { return version_; }
    uint64_t tensor_count() const { return n_tensors_; }
    uint64_t metadata_count() const { return n_kv_; }
    uint32_t alignment() const { return alignment_; }

    const std::vector<GGUFMetadataKV>& metadata() const { return kv_; }
    const GGUFMetadataKV* find_metadata(const std::string& key) const;
    std::string get_string(const std::string& key) const;
    uint32_t get_u32(const std::string& key) const;
    int32_t get_i32(const std::string& key) const;
    float get_f32(const std::string& key) const;
    bool get_bool(const std::string& key) const;
    uint64_t get_u64(const std::string& key) const;
    // string arrays (e.g. tokenizer.ggml.tokens); nullptr when absent
    const std::vector<std::string>* get_string_array(const std::string& key) const;

    const std::vector<GGUFTensorInfo>& tensors() const { return tensors_; }
    const GGUFTensorInfo* find_tensor(const std::string& name) const;

    const std::string& path() const { return path_; }
    size_t file_size() const { return size_; }
    size_t data_offset() const { return data_off_; }
    const std::string& last_error() const { return err_; }

private:
    std::string path_, err_;
    void* map_ = nullptr;
    size_t size_ = 0;
    int fd_ = -1;
    uint32_t version_ = 0;
    uint64_t n_tensors_ = 0, n_kv_ = 0;
    uint32_t alignment_ = 32;
    size_t data_off_ = 0;
    std::vector<GGUFMetadataKV> kv_;
    std::vector<GGUFTensorInfo> tensors_;
    std::unordered_map<std::string, size_t> kv_index_, tensor_index_;
    std::unordered_map<std::string, std::vector<std::string>> str_arrays_;

    bool parse(const uint8_t* base, const uint8_t* end);
    bool fail(const std::string& msg);
};

}  // namespace fence
