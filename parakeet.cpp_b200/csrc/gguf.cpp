#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "half.hpp"

namespace pkc {

namespace {

enum GgufValType : uint32_t {
  V_U8 = 0, V_I8 = 1, V_U16 = 2, V_I16 = 3, V_U32 = 4, V_I32 = 5, V_F32 = 6, V_BOOL = 7,
  V_STR = 8, V_ARR = 9, V_U64 = 10, V_I64 = 11, V_F64 = 12,
};

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (p + sizeof(T) > end) { ok = false; return v; }
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t n = get<uint64_t>();
    if (!ok || n > (uint64_t)(end - p)) { ok = false; return {}; }
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case V_U8: case V_I8: case V_BOOL: return 1;
    case V_U16: case V_I16: return 2;
    case V_U32: case V_I32: case V_F32: return 4;
    case V_U64: case V_I64: case V_F64: return 8;
    default: return 0;
  }
}

bool read_scalar(Cursor& c, uint32_t t, GgufValue& v) {
  switch (t) {
    case V_U8: v.i = c.get<uint8_t>(); break;
    case V_I8: v.i = c.get<int8_t>(); break;
    case V_U16: v.i = c.get<uint16_t>(); break;
    case V_I16: v.i = c.get<int16_t>(); break;
    case V_U32: v.i = c.get<uint32_t>(); break;
    case V_I32: v.i = c.get<int32_t>(); break;
    case V_U64: v.i = (int64_t)c.get<uint64_t>(); break;
    case V_I64: v.i = c.get<int64_t>(); break;
    case V_F32: v.f = c.get<float>(); v.i = (int64_t)v.f; break;
    case V_F64: v.f = c.get<double>(); v.i = (int64_t)v.f; break;
    case V_BOOL: v.i = c.get<uint8_t>() != 0; break;
    case V_STR: v.s = c.str(); break;
    default: return false;
  }
  if (t != V_F32 && t != V_F64) v.f = (double)v.i;
  return c.ok;
}

}  // namespace

size_t ggml_row_bytes(uint32_t type, int64_t n) {
  switch (type) {
    case GT_F32: return (size_t)n * 4;
    case GT_F16: case GT_BF16: return (size_t)n * 2;
    case GT_Q8_0: return n % 32 ? 0 : (size_t)(n / 32) * 34;
    case GT_Q4_0: return n % 32 ? 0 : (size_t)(n / 32) * 18;
    case GT_Q4_1: return n % 32 ? 0 : (size_t)(n / 32) * 20;
    case GT_Q5_0: return n % 32 ? 0 : (size_t)(n / 32) * 22;
    case GT_Q5_1: return n % 32 ? 0 : (size_t)(n / 32) * 24;
    case GT_Q4_K: return n % 256 ? 0 : (size_t)(n / 256) * 144;
    case GT_Q6_K: return n % 256 ? 0 : (size_t)(n / 256) * 210;
    default: return 0;
  }
}

GgufFile::~GgufFile() {
  if (map_) munmap(map_, size_);
}

bool GgufFile::open(const std::string& path, std::string& err) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) { err = "cannot open " + path; return false; }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    ::close(fd);
    err = "cannot stat or file too small: " + path;
    return false;
  }
  size_ = (size_t)st.st_size;
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) { map_ = nullptr; err = "mmap failed: " + path; return false; }
  const uint8_t* base = static_cast<const uint8_t*>(map_);
  Cursor c{base, base + size_};
  if (std::memcmp(base, "GGUF", 4) != 0) { err = "not a GGUF file: " + path; return false; }
  c.p += 4;
  const uint32_t version = c.get<uint32_t>();
  if (version < 2 || version > 3) { err = "unsupported GGUF version " + std::to_string(version); return false; }
  const uint64_t n_tensors = c.get<uint64_t>();
  const uint64_t n_kv = c.get<uint64_t>();
  if (!c.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) { err = "corrupt GGUF header"; return false; }
  for (uint64_t k = 0; k < n_kv; ++k) {
    std::string key = c.str();
    GgufValue v;
    v.type = c.get<uint32_t>();
    if (!c.ok) { err = "corrupt GGUF key/value section"; return false; }
    if (v.type == V_ARR) {
      v.arr_type = c.get<uint32_t>();
      const uint64_t n = c.get<uint64_t>();
      if (!c.ok || n > (uint64_t)(c.end - c.p)) { err = "corrupt GGUF array " + key; return false; }
      if (v.arr_type == V_STR) {
        v.arr_s.reserve(n);
        for (uint64_t i = 0; i < n && c.ok; ++i) v.arr_s.push_back(c.str());
      } else {
        const size_t sz = scalar_size(v.arr_type);
        if (!sz || n * sz > (uint64_t)(c.end - c.p)) { err = "bad GGUF array type in " + key; return false; }
        v.arr_i.reserve(n);
        for (uint64_t i = 0; i < n; ++i) {
          GgufValue e;
          read_scalar(c, v.arr_type, e);
          v.arr_i.push_back(e.i);
        }
      }
    } else if (!read_scalar(c, v.type, v)) {
      err = "bad GGUF value for " + key;
      return false;
    }
    if (!c.ok) { err = "truncated GGUF key/value section"; return false; }
    kv_[key] = std::move(v);
  }
  tensors_.reserve(n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensor t;
    t.name = c.str();
    t.n_dims = (int)c.get<uint32_t>();
    if (!c.ok || t.n_dims < 1 || t.n_dims > 4) { err = "corrupt GGUF tensor info"; return false; }
    for (int d = 0; d < t.n_dims; ++d) t.ne[d] = (int64_t)c.get<uint64_t>();
    t.type = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    if (!c.ok) { err = "truncated GGUF tensor info"; return false; }
    tensors_.push_back(t);
  }
  uint64_t align = 32;
  if (const GgufValue* a = value("general.alignment")) align = (uint64_t)a->i;
  if (align == 0 || (align & (align - 1))) { err = "bad general.alignment"; return false; }
  const uint64_t hdr = (uint64_t)(c.p - base);
  const uint64_t data_start = (hdr + align - 1) / align * align;
  for (size_t i = 0; i < tensors_.size(); ++i) {
    GgufTensor& t = tensors_[i];
    const size_t row = ggml_row_bytes(t.type, t.ne[0]);
    t.nbytes = row * (size_t)(t.ne[1] * t.ne[2] * t.ne[3]);
    if (row == 0) t.nbytes = 0;  // unsupported type: flagged when used
    if (data_start + t.offset + t.nbytes > size_) {
      err = "tensor " + t.name + " extends past the end of the file (truncated GGUF?)";
      return false;
    }
    t.data = base + data_start + t.offset;
    index_[t.name] = i;
  }
  return true;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
  auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}
const GgufValue* GgufFile::value(const std::string& key) const {
  auto it = kv_.find(key);
  return it == kv_.end() ? nullptr : &it->second;
}
uint32_t GgufFile::u32(const std::string& key, uint32_t def) const {
  const GgufValue* v = value(key);
  return v ? (uint32_t)v->i : def;
}
int32_t GgufFile::i32(const std::string& key, int32_t def) const {
  const GgufValue* v = value(key);
  return v ? (int32_t)v->i : def;
}
float GgufFile::f32(const std::string& key, float def) const {
  const GgufValue* v = value(key);
  return v ? (float)v->f : def;
}
bool GgufFile::boolean(const std::string& key, bool def) const {
  const GgufValue* v = value(key);
  return v ? v->i != 0 : def;
}
std::string GgufFile::str(const std::string& key, const std::string& def) const {
  const GgufValue* v = value(key);
  return v ? v->s : def;
}
std::vector<int64_t> GgufFile::int_array(const std::string& key) const {
  const GgufValue* v = value(key);
  return v ? v->arr_i : std::vector<int64_t>{};
}

bool ggml_to_f32(uint32_t type, const uint8_t* src, int64_t n, float* dst) {
  switch (type) {
    case GT_F32:
      std::memcpy(dst, src, (size_t)n * 4);
      return true;
    case GT_F16: {
      const uint16_t* h = reinterpret_cast<const uint16_t*>(src);
      for (int64_t i = 0; i < n; ++i) dst[i] = f16_to_f32(h[i]);
      return true;
    }
    case GT_BF16: {
      const uint16_t* h = reinterpret_cast<const uint16_t*>(src);
      for (int64_t i = 0; i < n; ++i) dst[i] = bf16_to_f32(h[i]);
      return true;
    }
    case GT_Q8_0: {
      // block: f16 scale d, 32 x int8; value = d * q
      if (n % 32) return false;
      for (int64_t b = 0; b < n / 32; ++b) {
        const uint8_t* blk = src + b * 34;
        uint16_t dh;
        std::memcpy(&dh, blk, 2);
        const float d = f16_to_f32(dh);
        const int8_t* q = reinterpret_cast<const int8_t*>(blk + 2);
        for (int i = 0; i < 32; ++i) dst[b * 32 + i] = d * (float)q[i];
      }
      return true;
    }
    case GT_Q4_K: {
      // super-block of 256: f16 d, f16 dmin, 12 bytes of 6-bit (scale, min) for
      // 8 sub-blocks of 32, 128 bytes of nibbles (sub-block 2j in the low and
      // 2j+1 in the high nibbles of bytes [32j, 32j+32)); value = d*sc*q - dmin*m
      if (n % 256) return false;
      for (int64_t b = 0; b < n / 256; ++b) {
        const uint8_t* blk = src + b * 144;
        uint16_t dh, mh;
        std::memcpy(&dh, blk, 2);
        std::memcpy(&mh, blk + 2, 2);
        const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
        const uint8_t* sc = blk + 4;
        const uint8_t* qs = blk + 16;
        uint8_t s[8], m[8];
        for (int j = 0; j < 4; ++j) {
          s[j] = sc[j] & 63;
          m[j] = sc[j + 4] & 63;
          s[j + 4] = (uint8_t)((sc[j + 8] & 0x0F) | ((sc[j] >> 6) << 4));
          m[j + 4] = (uint8_t)((sc[j + 8] >> 4) | ((sc[j + 4] >> 6) << 4));
        }
        float* o = dst + b * 256;
        for (int j = 0; j < 4; ++j) {
          const float d1 = d * s[2 * j], m1 = dmin * m[2 * j];
          const float d2 = d * s[2 * j + 1], m2 = dmin * m[2 * j + 1];
          for (int l = 0; l < 32; ++l) {
            o[64 * j + l] = d1 * (float)(qs[32 * j + l] & 0x0F) - m1;
            o[64 * j + 32 + l] = d2 * (float)(qs[32 * j + l] >> 4) - m2;
          }
        }
      }
      return true;
    }
    default:
      return false;
  }
}

}  // namespace pkc
