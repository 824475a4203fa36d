// Pre-laid-out weight cache: the device layout that lx_flow_load_gguf builds
// from flow.gguf (bf16 K-major stacked projections, fused QKV, conv weights
// per (group, tap), the rotary table and the modulation tables of the default
// schedule) written to one file and loaded back with plain copies, without
// GGUF parsing, fp32 -> bf16 conversion, re-layout or the modulation GEMVs.
//
// File "LXFL", version 1, little-endian:
//   char   magic[4] = "LXFL"
//   u32    version = 1
//   u32    n_sections
//   u32    layout[12]  the engine constants the layout depends on (DIM, FF,
//                      MEL, HEADS, HDIM, DEPTH, CONV_K, CONV_G, ROPE_MAX,
//                      n_sched, MAX_STEPS, 0); a mismatch is LX_ERR_FORMAT
//   u64    source_bytes        size of the flow.gguf it came from
//   u64    source_fnv1a        FNV-1a 64 of the first 1 MiB of that file
//   n_sections x { char name[32] (NUL padded), u32 dtype (0 f32, 1 bf16),
//                  u32 reserved, u64 elements, u64 offset (from file start) }
//   section data, each starting on a 4096-byte boundary
#include <sys/stat.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/larynx_flow.h"
#include "engine.h"

namespace lx {

namespace {

constexpr uint32_t LAYOUT_VERSION = 1;
constexpr size_t LAYOUT_ALIGN = 4096;

struct Section {
  const char* name;
  void** ptr;
  size_t count;
  uint32_t dtype;  // 0 f32, 1 bf16
};

struct SectionRecord {
  char name[32];
  uint32_t dtype;
  uint32_t reserved;
  uint64_t count;
  uint64_t offset;
};

std::vector<Section> model_sections(Model& W) {
  const size_t D = DIM;
  return {
      {"wqkv", reinterpret_cast<void**>(&W.wqkv), static_cast<size_t>(DEPTH) * QKV_N * D, 1},
      {"bqkv", reinterpret_cast<void**>(&W.bqkv), static_cast<size_t>(DEPTH) * QKV_N, 0},
      {"wo", reinterpret_cast<void**>(&W.wo), static_cast<size_t>(DEPTH) * D * D, 1},
      {"bo", reinterpret_cast<void**>(&W.bo), static_cast<size_t>(DEPTH) * D, 0},
      {"w1", reinterpret_cast<void**>(&W.w1), static_cast<size_t>(DEPTH) * FF * D, 1},
      {"b1", reinterpret_cast<void**>(&W.b1), static_cast<size_t>(DEPTH) * FF, 0},
      {"w2", reinterpret_cast<void**>(&W.w2), static_cast<size_t>(DEPTH) * D * FF, 1},
      {"b2", reinterpret_cast<void**>(&W.b2), static_cast<size_t>(DEPTH) * D, 0},
      {"adaln_w", reinterpret_cast<void**>(&W.adaln_w), static_cast<size_t>(DEPTH) * MOD_N * D, 0},
      {"adaln_b", reinterpret_cast<void**>(&W.adaln_b), static_cast<size_t>(DEPTH) * MOD_N, 0},
      {"win_x", reinterpret_cast<void**>(&W.win_x), D * MEL, 1},
      {"win_c", reinterpret_cast<void**>(&W.win_c), D * COND_K, 1},
      {"bin", reinterpret_cast<void**>(&W.bin), D, 0},
      {"wconv0", reinterpret_cast<void**>(&W.wconv[0]), D * 64 * CONV_K, 1},
      {"bconv0", reinterpret_cast<void**>(&W.bconv[0]), D, 0},
      {"wconv1", reinterpret_cast<void**>(&W.wconv[1]), D * 64 * CONV_K, 1},
      {"bconv1", reinterpret_cast<void**>(&W.bconv[1]), D, 0},
      {"wout", reinterpret_cast<void**>(&W.wout), static_cast<size_t>(MEL) * D, 1},
      {"bout", reinterpret_cast<void**>(&W.bout), MEL, 0},
      {"final_w", reinterpret_cast<void**>(&W.final_w), 2 * D * D, 0},
      {"final_b", reinterpret_cast<void**>(&W.final_b), 2 * D, 0},
      {"tmlp0_w", reinterpret_cast<void**>(&W.tmlp0_w), D * 256, 0},
      {"tmlp0_b", reinterpret_cast<void**>(&W.tmlp0_b), D, 0},
      {"tmlp2_w", reinterpret_cast<void**>(&W.tmlp2_w), D * D, 0},
      {"tmlp2_b", reinterpret_cast<void**>(&W.tmlp2_b), D, 0},
      {"emb", reinterpret_cast<void**>(&W.emb), static_cast<size_t>(6561) * MEL, 0},
      {"spk_w", reinterpret_cast<void**>(&W.spk_w), static_cast<size_t>(MEL) * 192, 0},
      {"spk_b", reinterpret_cast<void**>(&W.spk_b), MEL, 0},
      {"pre1_w", reinterpret_cast<void**>(&W.pre1_w), D * MEL * 4, 0},
      {"pre1_b", reinterpret_cast<void**>(&W.pre1_b), D, 0},
      {"pre2_w", reinterpret_cast<void**>(&W.pre2_w), static_cast<size_t>(MEL) * D * 3, 0},
      {"pre2_b", reinterpret_cast<void**>(&W.pre2_b), MEL, 0},
      {"rope", reinterpret_cast<void**>(&W.rope), static_cast<size_t>(ROPE_MAX) * 32 * 2, 0},
      // modulation tables: the n_sched filled entries of their MAX_STEPS rows
      {"mod", reinterpret_cast<void**>(&W.mod), static_cast<size_t>(N_STEPS_DEFAULT) * DEPTH * MOD_N, 0},
      {"mod_final", reinterpret_cast<void**>(&W.mod_final), static_cast<size_t>(N_STEPS_DEFAULT) * 2 * D, 0},
      {"temb", reinterpret_cast<void**>(&W.temb), static_cast<size_t>(N_STEPS_DEFAULT) * D, 0},
  };
}

// allocation size of a section's device buffer (the tables keep MAX_STEPS rows)
size_t alloc_elems(const Section& s) {
  if (!std::strcmp(s.name, "mod")) return static_cast<size_t>(MAX_STEPS) * DEPTH * MOD_N;
  if (!std::strcmp(s.name, "mod_final")) return static_cast<size_t>(MAX_STEPS) * 2 * DIM;
  if (!std::strcmp(s.name, "temb")) return static_cast<size_t>(MAX_STEPS) * DIM;
  return s.count;
}

void layout_constants(uint32_t (&c)[12]) {
  const uint32_t v[12] = {DIM, FF, MEL, HEADS, HDIM, DEPTH, CONV_K, CONV_G, ROPE_MAX, N_STEPS_DEFAULT, MAX_STEPS, 0};
  std::memcpy(c, v, sizeof(c));
}

uint64_t fnv1a_prefix(const std::string& path, uint64_t* bytes) {
  uint64_t h = 1469598103934665603ull;
  *bytes = 0;
  struct stat st;
  if (path.empty() || stat(path.c_str(), &st) != 0) return 0;
  *bytes = static_cast<uint64_t>(st.st_size);
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return 0;
  std::vector<unsigned char> buf(1 << 20);
  const size_t n = std::fread(buf.data(), 1, buf.size(), f);
  std::fclose(f);
  for (size_t i = 0; i < n; ++i) {
    h ^= buf[i];
    h *= 1099511628211ull;
  }
  return h;
}

size_t elem_bytes(uint32_t dtype) { return dtype == 1 ? 2 : 4; }

size_t align_up(size_t v) { return (v + LAYOUT_ALIGN - 1) / LAYOUT_ALIGN * LAYOUT_ALIGN; }

}  // namespace

int save_layout_file(Model& W, const std::string& gguf_path, const char* path, std::string* msg) {
  auto fail = [&](int code, const std::string& m) {
    *msg = m;
    return code;
  };
  std::vector<Section> secs = model_sections(W);
  const size_t head = 4 + 4 + 4 + 12 * 4 + 8 + 8 + secs.size() * sizeof(SectionRecord);
  std::vector<SectionRecord> recs(secs.size());
  size_t off = align_up(head);
  for (size_t i = 0; i < secs.size(); ++i) {
    std::memset(&recs[i], 0, sizeof(SectionRecord));
    std::strncpy(recs[i].name, secs[i].name, sizeof(recs[i].name) - 1);
    recs[i].dtype = secs[i].dtype;
    recs[i].count = secs[i].count;
    recs[i].offset = off;
    off = align_up(off + secs[i].count * elem_bytes(secs[i].dtype));
  }
  const std::string tmp = std::string(path) + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) return fail(LX_ERR_IO, std::string("cannot create ") + tmp);
  uint32_t c[12];
  layout_constants(c);
  uint64_t src_bytes = 0;
  const uint64_t src_hash = fnv1a_prefix(gguf_path, &src_bytes);
  const uint32_t version = LAYOUT_VERSION, nsec = static_cast<uint32_t>(secs.size());
  bool ok = std::fwrite("LXFL", 1, 4, f) == 4 && std::fwrite(&version, 4, 1, f) == 1 &&
            std::fwrite(&nsec, 4, 1, f) == 1 && std::fwrite(c, 4, 12, f) == 12 &&
            std::fwrite(&src_bytes, 8, 1, f) == 1 && std::fwrite(&src_hash, 8, 1, f) == 1 &&
            std::fwrite(recs.data(), sizeof(SectionRecord), recs.size(), f) == recs.size();
  std::vector<char> host;
  for (size_t i = 0; ok && i < secs.size(); ++i) {
    const size_t nb = secs[i].count * elem_bytes(secs[i].dtype);
    host.resize(nb);
    if (cudaMemcpy(host.data(), *secs[i].ptr, nb, cudaMemcpyDeviceToHost) != cudaSuccess) {
      std::fclose(f);
      std::remove(tmp.c_str());
      return fail(LX_ERR_CUDA, "cudaMemcpy of a weight section failed");
    }
    ok = std::fseek(f, static_cast<long>(recs[i].offset), SEEK_SET) == 0 && std::fwrite(host.data(), 1, nb, f) == nb;
  }
  ok = (std::fclose(f) == 0) && ok;
  if (!ok || std::rename(tmp.c_str(), path) != 0) {
    std::remove(tmp.c_str());
    return fail(LX_ERR_IO, std::string("cannot write ") + path);
  }
  return LX_OK;
}

int load_layout_file(Model& W, std::vector<void*>& allocs, const char* path, std::string* msg) {
  auto fail = [&](int code, const std::string& m) {
    *msg = m;
    return code;
  };
  FILE* f = std::fopen(path, "rb");
  if (!f) return fail(LX_ERR_IO, std::string("cannot open ") + path);
  char magic[4];
  uint32_t version = 0, nsec = 0, c[12], want[12];
  uint64_t src_bytes = 0, src_hash = 0;
  layout_constants(want);
  bool ok = std::fread(magic, 1, 4, f) == 4 && std::fread(&version, 4, 1, f) == 1 && std::fread(&nsec, 4, 1, f) == 1 &&
            std::fread(c, 4, 12, f) == 12 && std::fread(&src_bytes, 8, 1, f) == 1 &&
            std::fread(&src_hash, 8, 1, f) == 1;
  if (!ok || std::memcmp(magic, "LXFL", 4) != 0 || version != LAYOUT_VERSION || nsec > 1024 ||
      std::memcmp(c, want, sizeof(c)) != 0) {
    std::fclose(f);
    return fail(LX_ERR_FORMAT, std::string(path) + " is not a layout file of this library version");
  }
  std::vector<SectionRecord> recs(nsec);
  if (std::fread(recs.data(), sizeof(SectionRecord), nsec, f) != nsec) {
    std::fclose(f);
    return fail(LX_ERR_FORMAT, "truncated layout section table");
  }
  std::vector<Section> secs = model_sections(W);
  std::vector<char> host;
  for (const Section& s : secs) {
    const SectionRecord* r = nullptr;
    for (const auto& x : recs)
      if (std::strncmp(x.name, s.name, sizeof(x.name)) == 0) r = &x;
    if (!r || r->dtype != s.dtype || r->count != s.count) {
      std::fclose(f);
      return fail(LX_ERR_FORMAT, std::string("layout section ") + s.name + " missing or of the wrong size");
    }
    const size_t nb = s.count * elem_bytes(s.dtype);
    host.resize(nb);
    if (std::fseek(f, static_cast<long>(r->offset), SEEK_SET) != 0 || std::fread(host.data(), 1, nb, f) != nb) {
      std::fclose(f);
      return fail(LX_ERR_FORMAT, std::string("layout section ") + s.name + " is truncated");
    }
    void* d = nullptr;
    const size_t alloc = alloc_elems(s) * elem_bytes(s.dtype);
    if (cudaMalloc(&d, alloc) != cudaSuccess) {
      std::fclose(f);
      return fail(LX_ERR_OOM, "cudaMalloc for a weight section failed");
    }
    allocs.push_back(d);
    *s.ptr = d;
    if (cudaMemcpy(d, host.data(), nb, cudaMemcpyHostToDevice) != cudaSuccess) {
      std::fclose(f);
      return fail(LX_ERR_CUDA, "cudaMemcpy of a weight section failed");
    }
  }
  std::fclose(f);
  return LX_OK;
}

}  // namespace lx
