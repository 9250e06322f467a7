// Minimal GGUF (v2/v3) reader over mmap. Replaces the gguf.h API that
// ModelLoader::load uses in the reference (src/model_loader.cpp:99-166); ggml
// itself is not a dependency of this library.
#pragma once
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace pkc {

enum GgmlType : uint32_t {
  GT_F32 = 0,
  GT_F16 = 1,
  GT_Q4_0 = 2,
  GT_Q4_1 = 3,
  GT_Q5_0 = 6,
  GT_Q5_1 = 7,
  GT_Q8_0 = 8,
  GT_Q4_K = 12,
  GT_Q6_K = 14,
  GT_BF16 = 30,
};

struct GgufTensor {
  std::string name;
  int n_dims = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  uint32_t type = 0;
  uint64_t offset = 0;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t nelem() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
};

struct GgufValue {
  uint32_t type = 0;  // GGUF value type id
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  uint32_t arr_type = 0;
  std::vector<int64_t> arr_i;
  std::vector<std::string> arr_s;
};

// Bytes of `n` elements of a GGML type along a row (n multiple of the block).
// Returns 0 for unsupported types.
size_t ggml_row_bytes(uint32_t type, int64_t n);

class GgufFile {
 public:
  GgufFile() = default;
  ~GgufFile();
  GgufFile(const GgufFile&) = delete;
  GgufFile& operator=(const GgufFile&) = delete;

  bool open(const std::string& path, std::string& err);

  const GgufTensor* tensor(const std::string& name) const;
  const GgufValue* value(const std::string& key) const;
  uint32_t u32(const std::string& key, uint32_t def = 0) const;
  int32_t i32(const std::string& key, int32_t def = 0) const;
  float f32(const std::string& key, float def = 0.f) const;
  bool boolean(const std::string& key, bool def = false) const;
  std::string str(const std::string& key, const std::string& def = "") const;
  std::vector<int64_t> int_array(const std::string& key) const;
  const std::vector<GgufTensor>& tensors() const { return tensors_; }

 private:
  void* map_ = nullptr;
  size_t size_ = 0;
  std::vector<GgufTensor> tensors_;
  std::unordered_map<std::string, size_t> index_;
  std::unordered_map<std::string, GgufValue> kv_;
};

// Dequantise / convert `n` consecutive elements of a tensor row to f32.
bool ggml_to_f32(uint32_t type, const uint8_t* src, int64_t n, float* dst);

}  // namespace pkc
