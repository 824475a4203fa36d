// Minimal GGUF v3 reader for flow.gguf (memory-mapped, read-only).
//
// Format (little-endian): "GGUF", u32 version, i64 n_tensors, i64 n_kv, the
// metadata key/value section, the tensor-info section (name, u32 n_dims,
// i64 ne[n_dims], i32 ggml_type, u64 offset), zero padding to the alignment
// (KV "general.alignment", default 32), then the data blob.  `ne` is the
// PyTorch shape reversed; tensor data is row-major PyTorch order.
// Format reference: hardenedlinux/larynx docs/WEIGHT_FORMAT.md:15-110.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace lx {

enum GgmlType : int32_t { GGML_F32 = 0, GGML_F16 = 1, GGML_BF16 = 30 };

struct GgufTensor {
  std::string name;
  std::vector<int64_t> ne;  // ggml order (innermost first)
  int32_t type = 0;
  uint64_t offset = 0;      // from the start of the data blob
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : ne) n *= d;
    return n;
  }
  // PyTorch shape (ne reversed)
  std::vector<int64_t> shape() const { return std::vector<int64_t>(ne.rbegin(), ne.rend()); }
};

class GgufFile {
 public:
  GgufFile() = default;
  ~GgufFile();
  GgufFile(const GgufFile&) = delete;
  GgufFile& operator=(const GgufFile&) = delete;

  // Returns 0 on success, else an LX_ERR_* code with `error()` set.
  int open(const std::string& path);
  const std::string& error() const { return err_; }
  const GgufTensor* find(const std::string& name) const;
  // Copy a tensor to fp32 (F32, F16 and BF16 sources).  Checks the PyTorch
  // shape.  Returns 0 or an LX_ERR_* code.
  int read_f32(const std::string& name, const std::vector<int64_t>& shape, std::vector<float>& out);
  size_t n_tensors() const { return tensors_.size(); }

 private:
  std::string err_;
  void* map_ = nullptr;
  size_t map_size_ = 0;
  std::vector<GgufTensor> tensors_;
  std::unordered_map<std::string, size_t> index_;
};

}  // namespace lx
