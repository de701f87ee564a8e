// GGUF reader (host code): the file is memory-mapped read-only and parsed in
// place -- header, metadata key/values, tensor infos, alignment and the start
// of the tensor data -- following Inferno.jl src/GGUF.jl:119-165 (read_gguf)
// and :76-117 (read_string / read_value): magic "GGUF", version (2 or 3;
// the reference warns on anything but 3), uint64 tensor and key/value counts,
// strings as uint64 length + bytes (longer than 1 MiB is an error, as in the
// reference), arrays as element type + uint64 count, data aligned to
// general.alignment (default 32).  Every read is bounds-checked against the
// mapping; a malformed file is reported, never read past.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <cstring>
#include <map>
#include <string>
#include <vector>
#include "internal.h"
#include "common.cuh"
#include "gguf_internal.h"
#include "../../include/inferno_b200.h"

namespace inf {

namespace {

enum : uint32_t {
  G_U8 = 0, G_I8 = 1, G_U16 = 2, G_I16 = 3, G_U32 = 4, G_I32 = 5, G_F32 = 6, G_BOOL = 7,
  G_STR = 8, G_ARR = 9, G_U64 = 10, G_I64 = 11, G_F64 = 12
};
constexpr uint64_t MAX_STRING = 1ull << 20;     // src/GGUF.jl:78-81

struct Cursor {
  const uint8_t* p;
  size_t n, off;
  bool ok = true;
  bool take(void* dst, size_t k) {
    if (!ok || k > n - off) return ok = false;
    memcpy(dst, p + off, k);
    off += k;
    return true;
  }
  bool skip(size_t k) {
    if (!ok || k > n - off) return ok = false;
    off += k;
    return true;
  }
  template <class T> T get() {
    T v{};
    take(&v, sizeof v);
    return v;
  }
  bool str(std::string* s) {
    const uint64_t len = get<uint64_t>();
    if (!ok || len > MAX_STRING || len > n - off) return ok = false;
    if (s) s->assign((const char*)p + off, (size_t)len);
    off += (size_t)len;
    return true;
  }
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case G_U8: case G_I8: case G_BOOL: return 1;
    case G_U16: case G_I16: return 2;
    case G_U32: case G_I32: case G_F32: return 4;
    case G_U64: case G_I64: case G_F64: return 8;
    default: return 0;
  }
}

bool read_scalar(Cursor& c, uint32_t t, GgufValue* v) {
  v->type = t;
  switch (t) {
    case G_U8: v->i = c.get<uint8_t>(); break;
    case G_I8: v->i = c.get<int8_t>(); break;
    case G_U16: v->i = c.get<uint16_t>(); break;
    case G_I16: v->i = c.get<int16_t>(); break;
    case G_U32: v->i = c.get<uint32_t>(); break;
    case G_I32: v->i = c.get<int32_t>(); break;
    case G_U64: { const uint64_t u = c.get<uint64_t>(); v->i = (int64_t)u; v->u64 = true; break; }
    case G_I64: v->i = c.get<int64_t>(); break;
    case G_BOOL: v->i = c.get<uint8_t>() != 0; break;
    case G_F32: v->f = c.get<float>(); v->is_float = true; break;
    case G_F64: v->f = c.get<double>(); v->is_float = true; break;
    case G_STR: v->is_string = true; return c.str(&v->s);
    default: return c.ok = false;
  }
  if (!v->is_float) v->f = v->u64 ? (double)(uint64_t)v->i : (double)v->i;
  return c.ok;
}

bool read_value(Cursor& c, uint32_t t, GgufValue* v) {
  if (t != G_ARR) return read_scalar(c, t, v);
  v->type = G_ARR;
  v->arr_type = c.get<uint32_t>();
  v->arr_len = c.get<uint64_t>();
  if (!c.ok) return false;
  if (v->arr_type == G_STR) {
    for (uint64_t i = 0; i < v->arr_len && c.ok; ++i) c.str(nullptr);
    return c.ok;
  }
  if (v->arr_type == G_ARR) {               // nested arrays: walk them
    for (uint64_t i = 0; i < v->arr_len && c.ok; ++i) {
      GgufValue inner;
      read_value(c, G_ARR, &inner);
    }
    return c.ok;
  }
  const size_t es = scalar_size(v->arr_type);
  if (!es || v->arr_len > (c.n - c.off) / es) return c.ok = false;
  v->arr_data = c.p + c.off;
  return c.skip((size_t)(v->arr_len * es));
}

}  // namespace

int gguf_parse(const uint8_t* p, size_t n, InfernoGguf* g) {
  Cursor c{p, n, 0};
  if (c.get<uint32_t>() != 0x46554747u || !c.ok)          // "GGUF" little-endian
    return set_error(INFERNO_EFORMAT, "gguf: not a GGUF file (bad magic)");
  g->version = c.get<uint32_t>();
  if (g->version < 2 || g->version > 3)
    return set_error(INFERNO_EFORMAT, "gguf: version %u not supported (2 or 3)", g->version);
  const uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
  if (!c.ok) return set_error(INFERNO_EFORMAT, "gguf: truncated header");
  for (uint64_t i = 0; i < nkv; ++i) {
    std::string key;
    if (!c.str(&key)) return set_error(INFERNO_EFORMAT, "gguf: metadata key %llu malformed", (unsigned long long)i);
    const uint32_t t = c.get<uint32_t>();
    GgufValue v;
    if (!c.ok || !read_value(c, t, &v))
      return set_error(INFERNO_EFORMAT, "gguf: metadata value of '%s' malformed (type %u)", key.c_str(), t);
    g->kv_order.push_back(key);
    g->kv[key] = std::move(v);
  }
  for (uint64_t i = 0; i < nt; ++i) {
    GgufTensor t;
    if (!c.str(&t.name)) return set_error(INFERNO_EFORMAT, "gguf: tensor info %llu malformed", (unsigned long long)i);
    t.n_dims = c.get<uint32_t>();
    if (!c.ok || t.n_dims < 1 || t.n_dims > 4)
      return set_error(INFERNO_EFORMAT, "gguf: tensor '%s' has %u dims", t.name.c_str(), t.n_dims);
    for (uint32_t d = 0; d < t.n_dims; ++d) t.ne[d] = (int64_t)c.get<uint64_t>();
    t.type = (int)c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    if (!c.ok) return set_error(INFERNO_EFORMAT, "gguf: tensor info of '%s' truncated", t.name.c_str());
    g->tensors.push_back(std::move(t));
  }
  uint64_t align = 32;
  auto it = g->kv.find("general.alignment");
  if (it != g->kv.end() && !it->second.is_string && !it->second.is_float && it->second.type != G_ARR)
    align = (uint64_t)it->second.i;
  if (align == 0) return set_error(INFERNO_EFORMAT, "gguf: general.alignment is 0");
  g->alignment = align;
  g->data_offset = (c.off + align - 1) / align * align;
  if (g->data_offset > n) return set_error(INFERNO_EFORMAT, "gguf: data section beyond the end of the file");
  // sizes and bounds of every tensor's data
  for (auto& t : g->tensors) {
    int64_t elems = 1;
    for (uint32_t d = 0; d < t.n_dims; ++d) {
      if (t.ne[d] <= 0 || elems > ((int64_t)1 << 60) / t.ne[d]) { elems = -1; break; }
      elems *= t.ne[d];
    }
    t.nbytes = 0;
    if (elems > 0 && t.type >= 0 && t.type != T_Q6_KR && bb_of(t.type) > 0 && elems % qk_of(t.type) == 0)
      t.nbytes = (uint64_t)(elems / qk_of(t.type)) * (uint64_t)bb_of(t.type);
    if (t.nbytes && (t.offset > n - g->data_offset || t.nbytes > n - g->data_offset - t.offset))
      return set_error(INFERNO_EFORMAT, "gguf: data of tensor '%s' extends past the end of the file", t.name.c_str());
  }
  return 0;
}

}  // namespace inf

using namespace inf;

extern "C" {

int inferno_gguf_open(const char* path, InfernoGguf** out) {
  if (!path || !out) return set_error(INFERNO_EINVAL, "gguf_open: null argument");
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return set_error(INFERNO_EINVAL, "gguf_open: cannot open %s", path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    close(fd);
    return set_error(INFERNO_EFORMAT, "gguf_open: %s is too short for a GGUF header", path);
  }
  void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) return set_error(INFERNO_EINVAL, "gguf_open: mmap of %s failed", path);
  auto* g = new InfernoGguf();
  g->map = (const uint8_t*)m;
  g->size = (size_t)st.st_size;
  const int rc = gguf_parse(g->map, g->size, g);
  if (rc) {
    inferno_gguf_close(g);
    return rc;
  }
  *out = g;
  return 0;
}

int inferno_gguf_close(InfernoGguf* g) {
  if (!g) return 0;
  if (g->map) munmap((void*)g->map, g->size);
  delete g;
  return 0;
}

int inferno_gguf_version(const InfernoGguf* g) { return g ? (int)g->version : set_error(INFERNO_EINVAL, "null gguf"); }
int64_t inferno_gguf_n_tensors(const InfernoGguf* g) {
  return g ? (int64_t)g->tensors.size() : set_error(INFERNO_EINVAL, "null gguf");
}
int64_t inferno_gguf_n_kv(const InfernoGguf* g) { return g ? (int64_t)g->kv.size() : set_error(INFERNO_EINVAL, "null gguf"); }
int64_t inferno_gguf_data_offset(const InfernoGguf* g) {
  return g ? (int64_t)g->data_offset : set_error(INFERNO_EINVAL, "null gguf");
}

const char* inferno_gguf_key(const InfernoGguf* g, int64_t i) {
  if (!g || i < 0 || i >= (int64_t)g->kv_order.size()) return nullptr;
  return g->kv_order[(size_t)i].c_str();
}

int inferno_gguf_tensor_info(const InfernoGguf* g, int64_t i, const char** name, int* ggml_type, int64_t ne[4],
                             uint64_t* nbytes, const void** data) {
  if (!g || i < 0 || i >= (int64_t)g->tensors.size()) return set_error(INFERNO_EINVAL, "gguf_tensor_info: bad index");
  const GgufTensor& t = g->tensors[(size_t)i];
  if (name) *name = t.name.c_str();
  if (ggml_type) *ggml_type = t.type;
  if (ne)
    for (int d = 0; d < 4; ++d) ne[d] = d < (int)t.n_dims ? t.ne[d] : 1;
  if (nbytes) *nbytes = t.nbytes;
  if (data) *data = g->map + g->data_offset + t.offset;
  return 0;
}

static const GgufValue* kv_find(const InfernoGguf* g, const char* key) {
  if (!g || !key) return nullptr;
  auto it = g->kv.find(key);
  return it == g->kv.end() ? nullptr : &it->second;
}

int inferno_gguf_get_int(const InfernoGguf* g, const char* key, int64_t* out) {
  const GgufValue* v = kv_find(g, key);
  if (!v || !out) return set_error(INFERNO_ENOTFOUND, "gguf: no key %s", key ? key : "(null)");
  if (v->is_string || v->is_float || v->type == G_ARR) return set_error(INFERNO_EINVAL, "gguf: %s is not an integer", key);
  *out = v->i;
  return 0;
}

int inferno_gguf_get_float(const InfernoGguf* g, const char* key, double* out) {
  const GgufValue* v = kv_find(g, key);
  if (!v || !out) return set_error(INFERNO_ENOTFOUND, "gguf: no key %s", key ? key : "(null)");
  if (v->is_string || v->type == G_ARR) return set_error(INFERNO_EINVAL, "gguf: %s is not a number", key);
  *out = v->f;
  return 0;
}

int inferno_gguf_get_string(const InfernoGguf* g, const char* key, const char** out) {
  const GgufValue* v = kv_find(g, key);
  if (!v || !out) return set_error(INFERNO_ENOTFOUND, "gguf: no key %s", key ? key : "(null)");
  if (!v->is_string) return set_error(INFERNO_EINVAL, "gguf: %s is not a string", key);
  *out = v->s.c_str();
  return 0;
}

int inferno_gguf_get_array(const InfernoGguf* g, const char* key, int* elem_type, int64_t* len, const void** data) {
  const GgufValue* v = kv_find(g, key);
  if (!v) return set_error(INFERNO_ENOTFOUND, "gguf: no key %s", key ? key : "(null)");
  if (v->type != G_ARR) return set_error(INFERNO_EINVAL, "gguf: %s is not an array", key);
  if (elem_type) *elem_type = (int)v->arr_type;
  if (len) *len = (int64_t)v->arr_len;
  if (data) *data = v->arr_data;      // null for string / nested arrays
  return 0;
}

}  // extern "C"
