#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "../../include/larynx_flow.h"

namespace lx {

namespace {

struct Reader {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (static_cast<size_t>(end - p) < sizeof(T)) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || static_cast<uint64_t>(end - p) < n) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
  void skip(uint64_t n) {
    if (static_cast<uint64_t>(end - p) < n) {
      ok = false;
      return;
    }
    p += n;
  }
};

// gguf_type value sizes (docs/WEIGHT_FORMAT.md:47-60); 0 = variable
int scalar_size(int32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
  }
}

bool skip_value(Reader& r, int32_t type, int depth = 0) {
  if (depth > 4) return false;
  if (type == 8) {  // string
    r.str();
    return r.ok;
  }
  if (type == 9) {  // array
    const int32_t et = r.get<int32_t>();
    const uint64_t n = r.get<uint64_t>();
    if (!r.ok) return false;
    const int es = scalar_size(et);
    if (es > 0) {
      r.skip(n * static_cast<uint64_t>(es));
      return r.ok;
    }
    for (uint64_t i = 0; i < n && r.ok; ++i)
      if (!skip_value(r, et, depth + 1)) return false;
    return r.ok;
  }
  const int s = scalar_size(type);
  if (s == 0) return false;
  r.skip(s);
  return r.ok;
}

inline float half_to_float(uint16_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal
      exp = 127 - 15 + 1;
      while ((man & 0x400u) == 0) {
        man <<= 1;
        --exp;
      }
      man &= 0x3FFu;
      bits = sign | (exp << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

}  // namespace

GgufFile::~GgufFile() {
  if (map_) munmap(map_, map_size_);
}

int GgufFile::open(const std::string& path) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) {
    err_ = "cannot open " + path;
    return LX_ERR_IO;
  }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    ::close(fd);
    err_ = "cannot stat or file too small: " + path;
    return st.st_size < 24 ? LX_ERR_FORMAT : LX_ERR_IO;
  }
  map_size_ = static_cast<size_t>(st.st_size);
  map_ = mmap(nullptr, map_size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    err_ = "mmap failed: " + path;
    return LX_ERR_IO;
  }
  const uint8_t* base = static_cast<const uint8_t*>(map_);
  Reader r{base, base + map_size_};
  const uint32_t magic = r.get<uint32_t>();
  const uint32_t version = r.get<uint32_t>();
  const int64_t n_tensors = r.get<int64_t>();
  const int64_t n_kv = r.get<int64_t>();
  if (!r.ok || magic != 0x46554747u /* "GGUF" */) {
    err_ = "not a GGUF file: " + path;
    return LX_ERR_FORMAT;
  }
  if (version != 3) {
    err_ = "unsupported GGUF version " + std::to_string(version);
    return LX_ERR_FORMAT;
  }
  if (n_tensors < 0 || n_kv < 0 || n_tensors > (1 << 20) || n_kv > (1 << 20)) {
    err_ = "implausible GGUF counts";
    return LX_ERR_FORMAT;
  }
  uint64_t alignment = 32;
  for (int64_t i = 0; i < n_kv; ++i) {
    const std::string key = r.str();
    const int32_t type = r.get<int32_t>();
    if (!r.ok) break;
    if (key == "general.alignment" && type == 4) {
      alignment = r.get<uint32_t>();
      continue;
    }
    if (!skip_value(r, type)) {
      r.ok = false;
      break;
    }
  }
  if (!r.ok || alignment == 0 || (alignment & (alignment - 1)) != 0) {
    err_ = "malformed GGUF metadata section";
    return LX_ERR_FORMAT;
  }
  tensors_.resize(static_cast<size_t>(n_tensors));
  for (int64_t i = 0; i < n_tensors && r.ok; ++i) {
    GgufTensor& t = tensors_[i];
    t.name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    if (!r.ok || nd > 8) {
      r.ok = false;
      break;
    }
    t.ne.resize(nd);
    for (uint32_t d = 0; d < nd; ++d) t.ne[d] = r.get<int64_t>();
    t.type = r.get<int32_t>();
    t.offset = r.get<uint64_t>();
  }
  if (!r.ok) {
    err_ = "malformed GGUF tensor-info section";
    return LX_ERR_FORMAT;
  }
  const uint64_t hdr = static_cast<uint64_t>(r.p - base);
  const uint64_t data_off = (hdr + alignment - 1) / alignment * alignment;
  for (auto& t : tensors_) {
    size_t es = t.type == GGML_F32 ? 4 : (t.type == GGML_F16 || t.type == GGML_BF16) ? 2 : 0;
    int64_t n = 1;
    for (int64_t d : t.ne) {
      if (d < 0) {
        err_ = "negative dimension in tensor " + t.name;
        return LX_ERR_FORMAT;
      }
      n *= d;
    }
    t.nbytes = es * static_cast<size_t>(n);
    const uint64_t start = data_off + t.offset;
    if (es != 0 && (start > map_size_ || t.nbytes > map_size_ - start)) {
      err_ = "tensor " + t.name + " extends past the end of the file";
      return LX_ERR_FORMAT;
    }
    t.data = es != 0 ? base + start : nullptr;
    index_[t.name] = static_cast<size_t>(&t - tensors_.data());
  }
  return LX_OK;
}

const GgufTensor* GgufFile::find(const std::string& name) const {
  auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

int GgufFile::read_f32(const std::string& name, const std::vector<int64_t>& shape, std::vector<float>& out) {
  const GgufTensor* t = find(name);
  if (!t) {
    err_ = "missing tensor '" + name + "' in flow.gguf";
    return LX_ERR_FORMAT;
  }
  // ggml trims trailing 1s from ne; compare the non-trivial shapes
  std::vector<int64_t> want = shape, got = t->shape();
  while (!want.empty() && want.front() == 1 && want.size() > got.size()) want.erase(want.begin());
  if (want != got) {
    std::string w, g;
    for (auto d : shape) w += std::to_string(d) + ",";
    for (auto d : got) g += std::to_string(d) + ",";
    err_ = "tensor '" + name + "' has shape (" + g + ") expected (" + w + ")";
    return LX_ERR_SHAPE;
  }
  if (!t->data) {
    err_ = "tensor '" + name + "' has unsupported ggml type " + std::to_string(t->type);
    return LX_ERR_FORMAT;
  }
  const size_t n = static_cast<size_t>(t->numel());
  out.resize(n);
  if (t->type == GGML_F32) {
    std::memcpy(out.data(), t->data, n * 4);
  } else if (t->type == GGML_F16) {
    const uint16_t* s = reinterpret_cast<const uint16_t*>(t->data);
    for (size_t i = 0; i < n; ++i) out[i] = half_to_float(s[i]);
  } else {
    const uint16_t* s = reinterpret_cast<const uint16_t*>(t->data);
    for (size_t i = 0; i < n; ++i) {
      const uint32_t b = static_cast<uint32_t>(s[i]) << 16;
      std::memcpy(&out[i], &b, 4);
    }
  }
  return LX_OK;
}

}  // namespace lx
