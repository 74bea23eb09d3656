// gguf.h -- GGUF model files on the host: the container format
// (src/gguf.rs:227-320), ModelMeta::from_gguf (src/model_loader.rs:41-127),
// WeightStore::validate (:192-234) and the tensor views load_gguf returns
// (:291-309).  The tensor data is memory-mapped, not copied.
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace velo {

// GgufValue (gguf.rs:103-118); `type` is the GGUF value type id (0..12).
struct GgufValue {
    uint32_t type = 0;
    uint64_t u = 0;  // u8 / u16 / u32 / u64 / bool
    int64_t i = 0;   // i8 / i16 / i32 / i64
    double f = 0.0;  // f32 / f64
    std::string s;
    std::vector<GgufValue> arr;
};

// TensorInfo (gguf.rs:198-207): shape as stored (innermost dimension first).
struct GgufTensor {
    std::string name;
    std::vector<uint64_t> shape;
    uint32_t ggml_type = 0;
    uint64_t offset = 0, nbytes = 0;
};

// ModelMeta (model_loader.rs:21-37)
struct GgufModelMeta {
    std::string arch;
    uint64_t n_vocab = 0, n_embd = 0, n_layer = 0, n_head = 0, n_head_kv = 0, n_ctx = 0, n_ff = 0,
             head_dim = 0;
    float rope_freq_base = 0.0f, norm_eps = 0.0f;
    int32_t quantization = 0;  // 0 Q4_0, 1 Q4K (infer_quantization, :143-153)
};

struct GgufFile {
    uint32_t version = 0;
    std::map<std::string, GgufValue> meta;
    std::map<std::string, GgufTensor> tensors;
    uint64_t data_offset = 0;
    const uint8_t* data = nullptr;  // data section (mapped), data_bytes long
    uint64_t data_bytes = 0;
    void* map_base = nullptr;
    size_t map_len = 0;
    ~GgufFile();
};

// block_params (gguf.rs:71-91): false for an unknown type id.
bool ggml_block_params(uint32_t type, uint64_t* block_bytes, uint64_t* block_elems);

// GgufFile::read of an in-memory header (buf, n); positions past n are an
// I/O error (VELO_ERR_IO), format errors VELO_ERR_GGUF.
int32_t gguf_read_header(const uint8_t* buf, size_t n, GgufFile& out, uint64_t* header_end);
// GgufFile::read + read_all_tensors of a file (mapped).
int32_t gguf_open(const char* path, GgufFile& out);
int32_t gguf_model_meta(const GgufFile& g, GgufModelMeta& out);
int32_t gguf_validate(const GgufFile& g, const GgufModelMeta& m);

}  // namespace velo
