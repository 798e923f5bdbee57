#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>

#include "internal.h"

namespace sem {

namespace {
uint64_t rd64(const uint8_t* p) { uint64_t v; std::memcpy(&v, p, 8); return v; }
uint32_t rd32(const uint8_t* p) { uint32_t v; std::memcpy(&v, p, 4); return v; }

int block_size(uint32_t d) {  // format.go:86-117
  switch (d) {
    case 0: return 4; case 1: return 2; case 2: return 18; case 3: return 20; case 6: return 22; case 7: return 24;
    case 8: return 34; case 9: return 36; case 16: return 1; case 17: return 2; case 18: return 4; case 19: return 8;
    case 20: return 8; default: return 0;
  }
}
int elems_per_block(uint32_t d) {  // format.go:120-131
  switch (d) {
    case 0: case 1: case 16: case 17: case 18: case 19: case 20: return 1;
    case 2: case 3: case 6: case 7: return 16;
    case 8: case 9: return 32;
    default: return 0;
  }
}

struct Cursor {
  const uint8_t* d;
  size_t len, o;
  bool need(size_t n) const { return o + n <= len; }
};

// reader.go:220-271; returns false on truncation or an unknown type.
bool read_value(Cursor& c, uint32_t t, GgufFile& f, const std::string* key) {
  switch (t) {
    case 0: case 1: case 7: if (!c.need(1)) return false; c.o += 1; return true;
    case 2: case 3: if (!c.need(2)) return false; c.o += 2; return true;
    case 4:
      if (!c.need(4)) return false;
      if (key) f.u32[*key] = rd32(c.d + c.o);
      c.o += 4;
      return true;
    case 5: if (!c.need(4)) return false; c.o += 4; return true;
    case 6: {
      if (!c.need(4)) return false;
      uint32_t b = rd32(c.d + c.o);
      float v;
      std::memcpy(&v, &b, 4);
      if (key) f.f32[*key] = v;
      c.o += 4;
      return true;
    }
    case 10: case 11: case 12: if (!c.need(8)) return false; c.o += 8; return true;
    case 8: {
      if (!c.need(8)) return false;
      uint64_t n = rd64(c.d + c.o);
      c.o += 8;
      if (!c.need(n)) return false;
      if (key) f.str[*key] = std::string(reinterpret_cast<const char*>(c.d + c.o), n);
      c.o += n;
      return true;
    }
    case 9: {
      if (!c.need(12)) return false;
      uint32_t at = rd32(c.d + c.o);
      uint64_t n = rd64(c.d + c.o + 4);
      c.o += 12;
      if (key) f.array_len[*key] = n;
      for (uint64_t i = 0; i < n; ++i)
        if (!read_value(c, at, f, nullptr)) return false;
      return true;
    }
    default: return false;
  }
}
}  // namespace

GgufFile::~GgufFile() {
  if (map_) munmap(map_, map_len_);
}

int GgufFile::open(const char* path) {
  int fd = ::open(path, O_RDONLY);
  if (fd < 0) return set_error(SEM_EINVAL, "open gguf: open file: %s", path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    return set_error(SEM_EINVAL, "open gguf: stat %s", path);
  }
  void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (m == MAP_FAILED) return set_error(SEM_EINVAL, "open gguf: mmap file");
  map_ = m;
  map_len_ = (size_t)st.st_size;
  data = static_cast<const uint8_t*>(m);
  len = map_len_;
  if (len < 24) return set_error(SEM_EFORMAT, "open gguf: file too small for header");
  uint32_t magic = rd32(data);
  if (magic != 0x46554747u) return set_error(SEM_EFORMAT, "open gguf: invalid magic: 0x%08x", magic);
  uint32_t version = rd32(data + 4);
  if (version != 3) return set_error(SEM_EFORMAT, "open gguf: unsupported version: %u", version);
  uint64_t nt = rd64(data + 8), nkv = rd64(data + 16);
  Cursor c{data, len, 24};
  for (uint64_t i = 0; i < nkv; ++i) {
    if (!c.need(8)) return set_error(SEM_EFORMAT, "open gguf: read metadata %llu: truncated", (unsigned long long)i);
    uint64_t kl = rd64(data + c.o);
    c.o += 8;
    if (!c.need(kl + 4)) return set_error(SEM_EFORMAT, "open gguf: read metadata %llu: truncated", (unsigned long long)i);
    std::string key(reinterpret_cast<const char*>(data + c.o), kl);
    c.o += kl;
    uint32_t t = rd32(data + c.o);
    c.o += 4;
    if (!read_value(c, t, *this, &key))
      return set_error(SEM_EFORMAT, "open gguf: read metadata %llu: unknown metadata type: %u", (unsigned long long)i, t);
  }
  tensors.resize(nt);
  for (uint64_t i = 0; i < nt; ++i) {
    GgufTensor& tt = tensors[i];
    if (!c.need(8)) return set_error(SEM_EFORMAT, "open gguf: read tensor info %llu: truncated", (unsigned long long)i);
    uint64_t nl = rd64(data + c.o);
    c.o += 8;
    if (!c.need(nl + 4)) return set_error(SEM_EFORMAT, "open gguf: read tensor info %llu: truncated", (unsigned long long)i);
    tt.name.assign(reinterpret_cast<const char*>(data + c.o), nl);
    c.o += nl;
    uint32_t nd = rd32(data + c.o);
    c.o += 4;
    if (nd > 4 || !c.need(8 * (size_t)nd + 12))
      return set_error(SEM_EFORMAT, "open gguf: read tensor info %llu: truncated", (unsigned long long)i);
    uint64_t total = 1;
    for (uint32_t k = 0; k < nd; ++k) {
      tt.dims.push_back(rd64(data + c.o));
      total *= tt.dims.back();
      c.o += 8;
    }
    tt.dtype = rd32(data + c.o);
    tt.offset = rd64(data + c.o + 4);
    c.o += 12;
    int bs = block_size(tt.dtype), epb = elems_per_block(tt.dtype);
    tt.size = (epb > 0 && bs > 0) ? (total + epb - 1) / epb * bs : total * bs;
  }
  data_off = (c.o + 31) & ~size_t(31);
  for (const auto& t : tensors)
    if (data_off + t.offset + t.size > len)
      return set_error(SEM_EFORMAT, "tensor data out of bounds: %s (offset=%llu size=%llu fileSize=%zu)", t.name.c_str(),
                       (unsigned long long)(data_off + t.offset), (unsigned long long)t.size, len);
  return SEM_OK;
}

const GgufTensor* GgufFile::find(const std::string& name) const {
  for (const auto& t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}

int gguf_config(const GgufFile& f, sem_model_config* cfg) {
  *cfg = sem_model_config{};
  cfg->norm_eps = 1e-6f;
  cfg->rope_base = 10000.0f;
  cfg->max_seq_len = 2048;
  std::string arch;
  auto it = f.str.find("general.architecture");
  if (it != f.str.end()) arch = it->second;
  std::string prefix = arch.empty() ? "" : arch + ".";
  auto u = [&](const char* k, uint32_t* out) {
    auto j = f.u32.find(prefix + k);
    if (j == f.u32.end()) return false;
    *out = j->second;
    return true;
  };
  uint32_t v;
  if (!u("embedding_length", &v)) return set_error(SEM_EFORMAT, "parse config: %sembedding_length not found", prefix.c_str());
  cfg->embed_dim = (int32_t)v;
  if (!u("block_count", &v)) return set_error(SEM_EFORMAT, "parse config: %sblock_count not found", prefix.c_str());
  cfg->num_layers = (int32_t)v;
  if (!u("attention.head_count", &v))
    return set_error(SEM_EFORMAT, "parse config: %sattention.head_count not found", prefix.c_str());
  cfg->num_heads = (int32_t)v;
  cfg->num_kv_heads = u("attention.head_count_kv", &v) ? (int32_t)v : cfg->num_heads;
  cfg->head_dim = cfg->embed_dim / cfg->num_heads;
  cfg->attention_scale = 1.0f / (float)std::sqrt((double)cfg->head_dim);
  if (u("feed_forward_length", &v)) {
    cfg->interm_dim = (int32_t)v;
  } else if (const GgufTensor* t = f.find("blk.0.ffn_up.weight")) {
    cfg->interm_dim = t->dims.size() > 1 ? (int32_t)t->dims[1] : 0;
  } else {
    cfg->interm_dim = cfg->embed_dim * 3;
  }
  if (u("context_length", &v)) cfg->max_seq_len = (int32_t)v;
  auto fe = f.f32.find(prefix + "attention.layer_norm_rms_epsilon");
  if (fe != f.f32.end()) cfg->norm_eps = fe->second;
  auto fr = f.f32.find(prefix + "rope.freq_base");
  if (fr != f.f32.end()) cfg->rope_base = fr->second;
  auto tl = f.array_len.find("tokenizer.ggml.tokens");
  cfg->vocab_size = tl != f.array_len.end() ? (int32_t)tl->second : (int32_t)f.tensors.size();
  return SEM_OK;
}

}  // namespace sem
