// GGUF v3 reader for StableLM checkpoints (host code), the checks of the
// reference's readGGUF and loadStableGGUF (gguf.go:139-357): the file is
// memory-mapped, its header parsed and validated (magic and version, counts,
// metadata types, tensor ranks, dimensions and types, alignment, bounds,
// overlap), and the StableLM configuration derived from the metadata. Tensor
// data is never copied on the host: the load reads it from the mapping.
#pragma once
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace tcu {

struct GgufValue {
  enum Kind { UINT, INT, FLOAT, BOOL, STR, ARRAY } kind = UINT;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  bool b = false;
  std::string s;
  uint64_t count = 0;  // ARRAY: element count
};

struct GgufTensor {
  std::string name;
  int dtype = 0;               // GGUF type code
  std::vector<int64_t> shape;  // row-major engine order (GGUF lists the contiguous dimension first)
  uint64_t offset = 0, size = 0;  // absolute file offset, bytes
};

struct GgufFile {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t size = 0;
  std::map<std::string, GgufValue> meta;
  std::vector<GgufTensor> tensors;
  std::map<std::string, int> by_name;
  ~GgufFile() {
    if (map) munmap(const_cast<uint8_t*>(map), size);
    if (fd >= 0) close(fd);
  }
};

// Sequential little-endian reader over the header region; the first failure
// sticks (the ggufReader pattern of gguf.go:23-57).
struct GgufReader {
  const uint8_t* p;
  size_t n, pos = 0;
  std::string err;
  bool take(void* dst, size_t k) {
    if (!err.empty()) return false;
    if (k > n - pos) {
      err = "unexpected end of GGUF header";
      return false;
    }
    memcpy(dst, p + pos, k);
    pos += k;
    return true;
  }
  uint32_t u32() {
    uint32_t v = 0;
    take(&v, 4);
    return v;
  }
  uint64_t u64() {
    uint64_t v = 0;
    take(&v, 8);
    return v;
  }
  std::string str() {
    const uint64_t k = u64();
    if (!err.empty()) return {};
    if (k > (16u << 20)) {
      err = "GGUF string too large";
      return {};
    }
    std::string s(k, '\0');
    take(&s[0], k);
    return s;
  }
  // One metadata value (gguf.go:62-127): unsigned types widen to UINT, signed
  // to INT, floats to FLOAT; arrays hold one element type, no nesting.
  GgufValue value(uint32_t kind, bool in_array = false) {
    GgufValue v;
    switch (kind) {
      case 0: { uint8_t x = 0; take(&x, 1); v.kind = GgufValue::UINT; v.u = x; break; }
      case 1: { int8_t x = 0; take(&x, 1); v.kind = GgufValue::INT; v.i = x; break; }
      case 2: { uint16_t x = 0; take(&x, 2); v.kind = GgufValue::UINT; v.u = x; break; }
      case 3: { int16_t x = 0; take(&x, 2); v.kind = GgufValue::INT; v.i = x; break; }
      case 4: v.kind = GgufValue::UINT; v.u = u32(); break;
      case 5: { int32_t x = 0; take(&x, 4); v.kind = GgufValue::INT; v.i = x; break; }
      case 6: { float x = 0; take(&x, 4); v.kind = GgufValue::FLOAT; v.f = x; break; }
      case 7: {
        uint8_t x = 0;
        take(&x, 1);
        if (x > 1 && err.empty()) err = "invalid GGUF boolean";
        v.kind = GgufValue::BOOL;
        v.b = x == 1;
        break;
      }
      case 8: v.kind = GgufValue::STR; v.s = str(); break;
      case 9: {
        const uint32_t ek = u32();
        const uint64_t cnt = u64();
        if (ek == 9 || cnt > (1u << 20) || in_array) {
          if (err.empty()) err = "unsupported GGUF array";
          break;
        }
        v.kind = GgufValue::ARRAY;
        v.count = cnt;
        for (uint64_t j = 0; j < cnt && err.empty(); j++) {
          GgufValue e = value(ek, true);
          if (j == 0 && ek == 8) v.s = e.s;  // keep nothing else of string arrays
        }
        break;
      }
      case 10: v.kind = GgufValue::UINT; v.u = u64(); break;
      case 11: { int64_t x = 0; take(&x, 8); v.kind = GgufValue::INT; v.i = x; break; }
      case 12: { double x = 0; take(&x, 8); v.kind = GgufValue::FLOAT; v.f = x; break; }
      default:
        if (err.empty()) err = "unsupported GGUF metadata type " + std::to_string(kind);
    }
    return v;
  }
};

// readGGUF (gguf.go:139-248) on a memory-mapped file.
inline bool gguf_read(const char* path, GgufFile* g, std::string* err) {
  g->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (g->fd < 0) {
    *err = std::string("open ") + path + ": " + strerror(errno);
    return false;
  }
  struct stat st;
  if (fstat(g->fd, &st) != 0 || st.st_size <= 0) {
    *err = "cannot stat GGUF file";
    return false;
  }
  g->size = (size_t)st.st_size;
  void* m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
  if (m == MAP_FAILED) {
    *err = std::string("mmap: ") + strerror(errno);
    return false;
  }
  g->map = (const uint8_t*)m;
  GgufReader r{g->map, std::min<size_t>(g->size, (size_t)64 << 20)};
  if (r.u32() != 0x46554747u || r.u32() != 3) {
    *err = "expected little-endian GGUF v3";
    return false;
  }
  const uint64_t n_tensors = r.u64(), n_meta = r.u64();
  if (!r.err.empty() || n_tensors == 0 || n_tensors > 10000 || n_meta > 65536) {
    *err = "invalid GGUF counts";
    return false;
  }
  for (uint64_t i = 0; i < n_meta && r.err.empty(); i++) {
    const std::string key = r.str();
    const uint32_t kind = r.u32();
    GgufValue v = r.value(kind);
    if (!r.err.empty()) break;
    if (g->meta.count(key)) {
      *err = "duplicate GGUF key " + key;
      return false;
    }
    g->meta[key] = v;
  }
  for (uint64_t i = 0; i < n_tensors && r.err.empty(); i++) {
    GgufTensor t;
    t.name = r.str();
    const uint32_t rank = r.u32();
    if (!r.err.empty()) break;
    if (rank == 0 || rank > 4) {
      *err = "invalid GGUF tensor rank";
      return false;
    }
    t.shape.assign(rank, 0);
    int64_t n = 1;
    for (uint32_t j = 0; j < rank; j++) {
      const uint64_t dim = r.u64();
      if (!r.err.empty()) break;
      if (dim == 0 || dim > (uint64_t)(INT64_MAX / n) / 4) {
        *err = "invalid GGUF tensor dimensions";
        return false;
      }
      n *= (int64_t)dim;
      t.shape[rank - 1 - j] = (int64_t)dim;
    }
    const uint32_t kind = r.u32();
    if (!r.err.empty()) break;
    const int64_t inner = t.shape.back();
    switch (kind) {
      case 0: t.size = (uint64_t)n * 4; break;
      case 1:
      case 30: t.size = (uint64_t)n * 2; break;
      case 8:
      case 7:
        if (rank != 2 || inner % 32) {
          *err = std::string(kind == 8 ? "Q8_0" : "Q5_1") + " rows must be divisible by 32";
          return false;
        }
        t.size = (uint64_t)(n / 32) * (kind == 8 ? 34 : 24);
        break;
      case 13:
      case 14:
        if (rank != 2 || inner % 256) {
          *err = "K-quant rows must be divisible by 256";
          return false;
        }
        t.size = (uint64_t)(n / 256) * (kind == 14 ? 210 : 176);
        break;
      default:
        *err = "GGUF tensor " + t.name + ": unsupported type " + std::to_string(kind);
        return false;
    }
    t.dtype = (int)kind;
    t.offset = r.u64();
    if (!r.err.empty()) break;
    if (t.offset > (uint64_t)INT64_MAX) {
      *err = "GGUF tensor too large";
      return false;
    }
    if (g->by_name.count(t.name)) {
      *err = "duplicate GGUF tensor " + t.name;
      return false;
    }
    g->by_name[t.name] = (int)g->tensors.size();
    g->tensors.push_back(t);
  }
  if (!r.err.empty()) {
    *err = "GGUF header: " + r.err;
    return false;
  }
  uint64_t align = 32;
  auto al = g->meta.find("general.alignment");
  if (al != g->meta.end()) align = al->second.kind == GgufValue::UINT ? al->second.u : 0;
  if (align == 0 || align > 4096 || (align & (align - 1))) {
    *err = "invalid GGUF alignment";
    return false;
  }
  const uint64_t start = (r.pos + align - 1) & ~(align - 1);
  const uint64_t fsize = g->size;
  std::vector<std::pair<uint64_t, uint64_t>> ranges;
  for (GgufTensor& t : g->tensors) {
    if (t.offset % align || start > fsize || t.offset > fsize - start || t.size > fsize - start - t.offset) {
      *err = "GGUF tensor " + t.name + " outside file or misaligned";
      return false;
    }
    t.offset += start;
    ranges.emplace_back(t.offset, t.size);
  }
  std::sort(ranges.begin(), ranges.end());
  for (size_t i = 1; i < ranges.size(); i++)
    if (ranges[i].first < ranges[i - 1].first + ranges[i - 1].second) {
      *err = "overlapping GGUF tensors";
      return false;
    }
  return true;
}

// ggufNames (gguf.go:250-255): the GGUF name of a Hugging Face tensor name.
inline std::string gguf_name(const std::string& hf) {
  static const std::pair<const char*, const char*> rep[] = {
      {"model.embed_tokens", "token_embd"}, {"lm_head", "output"}, {"model.norm", "output_norm"},
      {"model.layers.", "blk."}, {"input_layernorm", "attn_norm"}, {"self_attn.q_proj", "attn_q"},
      {"self_attn.k_proj", "attn_k"}, {"self_attn.v_proj", "attn_v"}, {"self_attn.o_proj", "attn_output"},
      {"mlp.gate_proj", "ffn_gate"}, {"mlp.up_proj", "ffn_up"}, {"mlp.down_proj", "ffn_down"}};
  std::string out;
  size_t i = 0;
  while (i < hf.size()) {
    bool hit = false;
    for (const auto& kv : rep) {
      const size_t k = strlen(kv.first);
      if (hf.compare(i, k, kv.first) == 0) {
        out += kv.second;
        i += k;
        hit = true;
        break;
      }
    }
    if (!hit) out += hf[i++];
  }
  return out;
}

}  // namespace tcu
