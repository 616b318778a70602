// gguf.cu -- GGUF model-file reader (host code) feeding the Q2_K device path.
//
// Reads what ggml's gguf_init_from_file reads (ggml 0.9.8; the loader behind
// the reference's llama.cpp runs, llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:28-59):
//   header   magic "GGUF", version (u32), n_tensors (u64), n_kv (u64)
//   n_kv     key (u64 length + bytes), value type (u32), value
//            (arrays: element type u32, count u64, elements)
//   tensors  name, n_dims (u32), ne[n_dims] (u64), ggml type (u32),
//            offset (u64, relative to the data section)
//   data     starts at the first multiple of general.alignment (default 32)
//            after the tensor infos.
// Every length and count is checked against the file size before use, so a
// malformed file is refused with an error instead of read past its end.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "../../include/smeai_gguf.h"
#include "../../include/smeai_q2k.h"

namespace smeai {
namespace {

constexpr uint32_t kGgufMagic = 0x46554747u;  // "GGUF" little-endian
constexpr uint32_t kGgufCtxMagic = 0x47475546u;

enum ValueType : int {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
  kStr = 8, kArr = 9, kU64 = 10, kI64 = 11, kF64 = 12
};

int value_size(int t) {
  switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return 0;
  }
}

// (elements per block, bytes per block) of the ggml types this reader sizes.
bool type_block(int t, int64_t* elems, int64_t* bytes) {
  struct B { int t; int64_t e, b; };
  static const B table[] = {
      {0, 1, 4},     {1, 1, 2},     {2, 32, 18},   {3, 32, 20},   {6, 32, 22},   {7, 32, 24},
      {8, 32, 34},   {9, 32, 36},   {10, 256, 84}, {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
      {14, 256, 210}, {15, 256, 292}, {24, 1, 1},   {25, 1, 2},    {26, 1, 4},    {27, 1, 8},
      {28, 1, 8},    {30, 1, 2}};
  for (const B& e : table)
    if (e.t == t) {
      *elems = e.e;
      *bytes = e.b;
      return true;
    }
  return false;
}

struct KV {
  std::string key;
  int type = 0;
  int arr_type = 0;
  uint64_t arr_n = 0;
  bool is_int = false, is_neg = false;
  uint64_t u = 0;   // integer value (two's complement for negatives)
  double f = 0.0;   // numeric value as double
  std::string s;
};

struct TensorInfo {
  std::string name;
  int type = 0;
  int n_dims = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  uint64_t offset = 0;
  uint64_t nbytes = 0;
};

struct Ctx {
  uint32_t magic = kGgufCtxMagic;
  std::string path;
  int version = 0;
  uint64_t alignment = 32;
  uint64_t data_offset = 0;
  uint64_t file_size = 0;
  std::vector<KV> kv;
  std::vector<TensorInfo> tensors;
  std::unordered_map<std::string, int64_t> kv_index, tensor_index;
};

// Sequential reader over the file with a hard end.
struct Reader {
  FILE* f = nullptr;
  uint64_t pos = 0, size = 0;
  bool ok = true;
  bool raw(void* dst, uint64_t n) {
    if (!ok || n > size - pos) return ok = false;
    if (n && fread(dst, 1, (size_t)n, f) != (size_t)n) return ok = false;
    pos += n;
    return true;
  }
  bool skip(uint64_t n) {
    if (!ok || n > size - pos || fseeko(f, (off_t)n, SEEK_CUR) != 0) return ok = false;
    pos += n;
    return true;
  }
  template <typename T>
  bool get(T& v) { return raw(&v, sizeof(T)); }
  bool str(std::string& s, uint64_t max_len) {
    uint64_t n = 0;
    if (!get(n) || n > max_len || n > size - pos) return ok = false;
    s.resize((size_t)n);
    return raw(n ? &s[0] : nullptr, n);
  }
};

const Ctx* as_ctx(const void* p) {
  const Ctx* c = static_cast<const Ctx*>(p);
  return (c && c->magic == kGgufCtxMagic) ? c : nullptr;
}

int fail(const char* what, const std::string& path) {
  set_last_error("smeai_gguf_open: %s: %s", path.c_str(), what);
  return kBadArgument;
}

int read_value(Reader& r, KV& kv, int type) {
  const int vs = value_size(type);
  if (vs) {
    uint64_t raw = 0;
    if (!r.raw(&raw, (uint64_t)vs)) return kBadArgument;
    kv.is_int = type != kF32 && type != kF64;
    switch (type) {
      case kI8: kv.u = (uint64_t)(int64_t)(int8_t)raw; kv.is_neg = (int8_t)raw < 0; break;
      case kI16: kv.u = (uint64_t)(int64_t)(int16_t)raw; kv.is_neg = (int16_t)raw < 0; break;
      case kI32: kv.u = (uint64_t)(int64_t)(int32_t)raw; kv.is_neg = (int32_t)raw < 0; break;
      case kI64: kv.u = raw; kv.is_neg = (int64_t)raw < 0; break;
      default: kv.u = raw;
    }
    if (type == kF32) {
      float f;
      memcpy(&f, &raw, 4);
      kv.f = f;
    } else if (type == kF64) {
      memcpy(&kv.f, &raw, 8);
    } else {
      kv.f = kv.is_neg ? (double)(int64_t)kv.u : (double)kv.u;
    }
    return kOk;
  }
  if (type == kStr) return r.str(kv.s, 1ull << 30) ? kOk : kBadArgument;
  if (type == kArr) {
    uint32_t et = 0;
    uint64_t n = 0;
    if (!r.get(et) || !r.get(n)) return kBadArgument;
    kv.arr_type = (int)et;
    kv.arr_n = n;
    const int es = value_size((int)et);
    if (es) return (n <= (r.size - r.pos) / (uint64_t)es && r.skip(n * (uint64_t)es)) ? kOk : kBadArgument;
    if (et == kStr) {
      for (uint64_t i = 0; i < n; ++i) {
        uint64_t len = 0;
        if (!r.get(len) || !r.skip(len)) return kBadArgument;
      }
      return kOk;
    }
    if (et == kArr) {  // nested arrays: walk them without keeping them
      for (uint64_t i = 0; i < n; ++i) {
        KV inner;
        if (read_value(r, inner, kArr) != kOk) return kBadArgument;
      }
      return kOk;
    }
    return kBadArgument;
  }
  return kBadArgument;
}

}  // namespace
}  // namespace smeai

using namespace smeai;

extern "C" {

int smeai_gguf_open(const char* path, void** ctx_out) {
  if (!path || !ctx_out) {
    set_last_error("smeai_gguf_open: NULL argument");
    return kBadArgument;
  }
  *ctx_out = nullptr;
  FILE* f = fopen(path, "rb");
  if (!f) {
    set_last_error("smeai_gguf_open: cannot open %s", path);
    return kBadArgument;
  }
  Ctx* c = new (std::nothrow) Ctx();
  if (!c) {
    fclose(f);
    set_last_error("smeai_gguf_open: out of memory");
    return kAllocFailed;
  }
  c->path = path;
  fseeko(f, 0, SEEK_END);
  c->file_size = (uint64_t)ftello(f);
  fseeko(f, 0, SEEK_SET);
  Reader r;
  r.f = f;
  r.size = c->file_size;
  int st = kOk;
  uint32_t magic = 0, version = 0;
  uint64_t n_tensors = 0, n_kv = 0;
  if (!r.get(magic) || magic != kGgufMagic) {
    st = fail("not a GGUF file (bad magic)", c->path);
  } else if (!r.get(version) || (version != 2 && version != 3)) {
    set_last_error("smeai_gguf_open: %s: GGUF version %u not supported (2 and 3 are; a byte-swapped "
                   "version means a big-endian file)", path, version);
    st = kUnsupported;
  } else if (!r.get(n_tensors) || !r.get(n_kv) || n_tensors > (1ull << 24) || n_kv > (1ull << 24)) {
    st = fail("bad tensor or metadata count", c->path);
  }
  c->version = (int)version;
  for (uint64_t i = 0; st == kOk && i < n_kv; ++i) {
    KV kv;
    uint32_t type = 0;
    if (!r.str(kv.key, 1ull << 16) || !r.get(type)) {
      st = fail("truncated metadata", c->path);
      break;
    }
    kv.type = (int)type;
    if (read_value(r, kv, kv.type) != kOk) {
      st = fail("malformed metadata value", c->path);
      break;
    }
    c->kv_index[kv.key] = (int64_t)c->kv.size();
    c->kv.push_back(std::move(kv));
  }
  if (st == kOk) {
    auto it = c->kv_index.find("general.alignment");
    if (it != c->kv_index.end()) {
      const KV& a = c->kv[(size_t)it->second];
      if (!a.is_int || a.is_neg || a.u == 0 || (a.u & (a.u - 1)) || a.u > (1ull << 20))
        st = fail("general.alignment must be a power of two", c->path);
      else
        c->alignment = a.u;
    }
  }
  for (uint64_t i = 0; st == kOk && i < n_tensors; ++i) {
    TensorInfo t;
    uint32_t nd = 0, type = 0;
    if (!r.str(t.name, 1ull << 16) || !r.get(nd) || nd < 1 || nd > 4) {
      st = fail("malformed tensor info", c->path);
      break;
    }
    t.n_dims = (int)nd;
    for (uint32_t d = 0; d < nd; ++d) {
      uint64_t ne = 0;
      if (!r.get(ne) || ne == 0 || ne > (1ull << 40)) {
        st = fail("bad tensor dimension", c->path);
        break;
      }
      t.ne[d] = (int64_t)ne;
    }
    if (st != kOk) break;
    if (!r.get(type) || !r.get(t.offset)) {
      st = fail("truncated tensor info", c->path);
      break;
    }
    t.type = (int)type;
    int64_t be = 0, bb = 0;
    if (type_block(t.type, &be, &bb)) {
      if (t.ne[0] % be) {
        st = fail("row length not a multiple of the type's block size", c->path);
        break;
      }
      const double est = (double)(t.ne[0] / be) * (double)bb * (double)t.ne[1] * (double)t.ne[2] * (double)t.ne[3];
      if (est > 1.0e15) {
        st = fail("tensor too large", c->path);
        break;
      }
      t.nbytes = (uint64_t)(t.ne[0] / be) * (uint64_t)bb * (uint64_t)t.ne[1] * (uint64_t)t.ne[2] *
                 (uint64_t)t.ne[3];
    }
    if (c->tensor_index.count(t.name)) {
      st = fail("duplicate tensor name", c->path);
      break;
    }
    c->tensor_index[t.name] = (int64_t)c->tensors.size();
    c->tensors.push_back(std::move(t));
  }
  if (st == kOk) {
    c->data_offset = (r.pos + c->alignment - 1) / c->alignment * c->alignment;
    for (const TensorInfo& t : c->tensors) {
      if (t.offset % c->alignment || t.offset > c->file_size || c->data_offset > c->file_size - t.offset ||
          t.nbytes > c->file_size - c->data_offset - t.offset) {
        st = fail("tensor data outside the file or misaligned", c->path);
        break;
      }
    }
  }
  fclose(f);
  if (st != kOk) {
    delete c;
    return st;
  }
  *ctx_out = c;
  return kOk;
}

void smeai_gguf_close(void* ctx) {
  Ctx* c = static_cast<Ctx*>(ctx);
  if (!c || c->magic != kGgufCtxMagic) return;
  c->magic = 0;
  delete c;
}

int smeai_gguf_version(const void* ctx) {
  const Ctx* c = as_ctx(ctx);
  return c ? c->version : kBadArgument;
}

uint64_t smeai_gguf_alignment(const void* ctx) {
  const Ctx* c = as_ctx(ctx);
  return c ? c->alignment : 0;
}

uint64_t smeai_gguf_data_offset(const void* ctx) {
  const Ctx* c = as_ctx(ctx);
  return c ? c->data_offset : 0;
}

int64_t smeai_gguf_n_tensors(const void* ctx) {
  const Ctx* c = as_ctx(ctx);
  return c ? (int64_t)c->tensors.size() : kBadArgument;
}

int64_t smeai_gguf_find_tensor(const void* ctx, const char* name) {
  const Ctx* c = as_ctx(ctx);
  if (!c || !name) return -1;
  auto it = c->tensor_index.find(name);
  return it == c->tensor_index.end() ? -1 : it->second;
}

int smeai_gguf_tensor_info(const void* ctx, int64_t id, const char** name, int* ggml_type, int* n_dims,
                           int64_t ne[4], uint64_t* offset, uint64_t* nbytes) {
  const Ctx* c = as_ctx(ctx);
  if (!c || id < 0 || id >= (int64_t)c->tensors.size()) {
    set_last_error("smeai_gguf_tensor_info: bad context or tensor id");
    return kBadArgument;
  }
  const TensorInfo& t = c->tensors[(size_t)id];
  if (name) *name = t.name.c_str();
  if (ggml_type) *ggml_type = t.type;
  if (n_dims) *n_dims = t.n_dims;
  if (ne)
    for (int d = 0; d < 4; ++d) ne[d] = t.ne[d];
  if (offset) *offset = t.offset;
  if (nbytes) *nbytes = t.nbytes;
  return kOk;
}

int smeai_gguf_read_tensor(const void* ctx, int64_t id, void* dst, uint64_t dst_bytes) {
  const Ctx* c = as_ctx(ctx);
  if (!c || !dst || id < 0 || id >= (int64_t)c->tensors.size()) {
    set_last_error("smeai_gguf_read_tensor: bad context, tensor id or destination");
    return kBadArgument;
  }
  const TensorInfo& t = c->tensors[(size_t)id];
  if (!t.nbytes) {
    set_last_error("smeai_gguf_read_tensor: %s: ggml type %d has no size known to this reader", t.name.c_str(),
                   t.type);
    return kUnsupported;
  }
  if (dst_bytes < t.nbytes) {
    set_last_error("smeai_gguf_read_tensor: %s needs %llu bytes", t.name.c_str(), (unsigned long long)t.nbytes);
    return kBadArgument;
  }
  FILE* f = fopen(c->path.c_str(), "rb");
  if (!f) {
    set_last_error("smeai_gguf_read_tensor: cannot reopen %s", c->path.c_str());
    return kBadArgument;
  }
  const bool ok = fseeko(f, (off_t)(c->data_offset + t.offset), SEEK_SET) == 0 &&
                  fread(dst, 1, (size_t)t.nbytes, f) == (size_t)t.nbytes;
  fclose(f);
  if (!ok) {
    set_last_error("smeai_gguf_read_tensor: short read of %s", t.name.c_str());
    return kBadArgument;
  }
  return kOk;
}

int smeai_gguf_load_q2k(const void* ctx, int64_t id, void** w_dev_out) {
  const Ctx* c = as_ctx(ctx);
  if (!c || !w_dev_out || id < 0 || id >= (int64_t)c->tensors.size()) {
    set_last_error("smeai_gguf_load_q2k: bad context, tensor id or output");
    return kBadArgument;
  }
  *w_dev_out = nullptr;
  const TensorInfo& t = c->tensors[(size_t)id];
  if (t.type != SMEAI_GGML_Q2_K || t.n_dims != 2) {
    set_last_error("smeai_gguf_load_q2k: %s is ggml type %d with %d dims (a 2-D Q2_K tensor is required)",
                   t.name.c_str(), t.type, t.n_dims);
    return kUnsupported;
  }
  std::vector<uint8_t> host;
  try {
    host.resize((size_t)t.nbytes);
  } catch (...) {
    set_last_error("smeai_gguf_load_q2k: cannot allocate %llu host bytes", (unsigned long long)t.nbytes);
    return kAllocFailed;
  }
  int st = smeai_gguf_read_tensor(ctx, id, host.data(), t.nbytes);
  if (st != kOk) return st;
  return smeai_q2k_repack(host.data(), t.ne[1], t.ne[0], w_dev_out);
}

int smeai_gguf_load_q3k(const void* ctx, int64_t id, void** w_dev_out) {
  const Ctx* c = as_ctx(ctx);
  if (!c || !w_dev_out || id < 0 || id >= (int64_t)c->tensors.size()) {
    set_last_error("smeai_gguf_load_q3k: bad context, tensor id or output");
    return kBadArgument;
  }
  *w_dev_out = nullptr;
  const TensorInfo& t = c->tensors[(size_t)id];
  if (t.type != SMEAI_GGML_Q3_K || t.n_dims != 2) {
    set_last_error("smeai_gguf_load_q3k: %s is ggml type %d with %d dims (a 2-D Q3_K tensor is required)",
                   t.name.c_str(), t.type, t.n_dims);
    return kUnsupported;
  }
  std::vector<uint8_t> host;
  try {
    host.resize((size_t)t.nbytes);
  } catch (...) {
    set_last_error("smeai_gguf_load_q3k: cannot allocate %llu host bytes", (unsigned long long)t.nbytes);
    return kAllocFailed;
  }
  int st = smeai_gguf_read_tensor(ctx, id, host.data(), t.nbytes);
  if (st != kOk) return st;
  return smeai_q3k_repack(host.data(), t.ne[1], t.ne[0], w_dev_out);
}

int smeai_gguf_load_q6k(const void* ctx, int64_t id, void** w_dev_out) {
  const Ctx* c = as_ctx(ctx);
  if (!c || !w_dev_out || id < 0 || id >= (int64_t)c->tensors.size()) {
    set_last_error("smeai_gguf_load_q6k: bad context, tensor id or output");
    return kBadArgument;
  }
  *w_dev_out = nullptr;
  const TensorInfo& t = c->tensors[(size_t)id];
  if (t.type != SMEAI_GGML_Q6_K || t.n_dims != 2) {
    set_last_error("smeai_gguf_load_q6k: %s is ggml type %d with %d dims (a 2-D Q6_K tensor is required)",
                   t.name.c_str(), t.type, t.n_dims);
    return kUnsupported;
  }
  std::vector<uint8_t> host;
  try {
    host.resize((size_t)t.nbytes);
  } catch (...) {
    set_last_error("smeai_gguf_load_q6k: cannot allocate %llu host bytes", (unsigned long long)t.nbytes);
    return kAllocFailed;
  }
  int st = smeai_gguf_read_tensor(ctx, id, host.data(), t.nbytes);
  if (st != kOk) return st;
  return smeai_q6k_repack(host.data(), t.ne[1], t.ne[0], w_dev_out);
}

int64_t smeai_gguf_n_kv(const void* ctx) {
  const Ctx* c = as_ctx(ctx);
  return c ? (int64_t)c->kv.size() : kBadArgument;
}

int64_t smeai_gguf_find_key(const void* ctx, const char* key) {
  const Ctx* c = as_ctx(ctx);
  if (!c || !key) return -1;
  auto it = c->kv_index.find(key);
  return it == c->kv_index.end() ? -1 : it->second;
}

int smeai_gguf_key_type(const void* ctx, const char* key) {
  const int64_t i = smeai_gguf_find_key(ctx, key);
  return i < 0 ? kBadArgument : as_ctx(ctx)->kv[(size_t)i].type;
}

int smeai_gguf_get_u64(const void* ctx, const char* key, uint64_t* out) {
  const int64_t i = smeai_gguf_find_key(ctx, key);
  if (i < 0 || !out) {
    set_last_error("smeai_gguf_get_u64: key %s not found", key ? key : "(null)");
    return kBadArgument;
  }
  const KV& kv = as_ctx(ctx)->kv[(size_t)i];
  if (!kv.is_int || kv.is_neg) {
    set_last_error("smeai_gguf_get_u64: %s is not a non-negative integer", key);
    return kBadArgument;
  }
  *out = kv.u;
  return kOk;
}

int smeai_gguf_get_f64(const void* ctx, const char* key, double* out) {
  const int64_t i = smeai_gguf_find_key(ctx, key);
  if (i < 0 || !out) {
    set_last_error("smeai_gguf_get_f64: key %s not found", key ? key : "(null)");
    return kBadArgument;
  }
  const KV& kv = as_ctx(ctx)->kv[(size_t)i];
  if (kv.type == kStr || kv.type == kArr) {
    set_last_error("smeai_gguf_get_f64: %s is not numeric", key);
    return kBadArgument;
  }
  *out = kv.f;
  return kOk;
}

int smeai_gguf_get_str(const void* ctx, const char* key, const char** out) {
  const int64_t i = smeai_gguf_find_key(ctx, key);
  if (i < 0 || !out) {
    set_last_error("smeai_gguf_get_str: key %s not found", key ? key : "(null)");
    return kBadArgument;
  }
  const KV& kv = as_ctx(ctx)->kv[(size_t)i];
  if (kv.type != kStr) {
    set_last_error("smeai_gguf_get_str: %s is not a string", key);
    return kBadArgument;
  }
  *out = kv.s.c_str();
  return kOk;
}

}  // extern "C"
