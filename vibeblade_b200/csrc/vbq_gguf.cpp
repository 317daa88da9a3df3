// vbq_gguf.cpp -- GGUF weight source: parse a GGUF v1-v3 file and upload its tensors (or
// block-aligned tensor-parallel shards of them) into device memory as raw blocks.
//
// The parse follows the reference's reader (kevin046/VibeBlade cpp/src/gguf.cpp:14-280,
// cpp/include/gguf.h) rule for rule, so a file reads the same here as in the reference
// engine and fails with the same message:
//   * header: magic "GGUF", version <= 3, n_tensors and n_kv <= 10^6 (gguf.cpp:62-77);
//   * metadata values (gguf.cpp:79-160): u8 / i8 / u32 (kept as a signed 32-bit value) /
//     i32 / u64 / i64 as integers, f32 / f64 as floats, bool, string; arrays of strings,
//     of 32-bit integers (kept signed), of 64-bit integers and of f32 are kept, other
//     arrays skipped by element size; u16 / i16 values are skipped; each kind of value
//     has its own table, so a later key replaces an earlier one of the same kind only
//     (an integer and a string of one name both stay readable, as in the reference);
//   * tensor infos (gguf.cpp:163-193): at most 4 dims, size = tensor_nbytes(type, values);
//   * the data section starts at the next multiple of 32 after the infos (the reference
//     does not read general.alignment);
//   * a tensor's data must end inside the file (gguf.cpp:255-262).
// One deliberate difference: every read is bounds-checked, including the elements of
// integer and float arrays, which the reference reads unchecked (gguf.cpp:116-138); a
// truncated array therefore fails here at the array ("read past end of file").
// What differs besides is the storage: the file is memory-mapped read-only instead of read
// into one heap buffer (a 70B model is tens of GB), and the upload streams the bytes to the
// GPU through two pinned staging buffers, copying a shard's block-aligned column range of
// each row with one 2-D copy per chunk.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>

#include "vbq.h"
#include "vbq_gguf.h"

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& m) {
  g_err = m;
  return code;
}

// block geometry of every ggml type id the reference's tables know
// (cpp/include/ggml_types.h:31-71; unknown ids count as 1 value of 4 bytes, as there)
int64_t blck_size(int32_t t) {
  switch (t) {
    case 2: case 3: case 6: case 7: case 8: case 9: return 32;
    case 10: case 11: case 12: case 13: case 14: case 15: return 256;
    default: return 1;
  }
}
int64_t type_size(int32_t t) {
  switch (t) {
    case 0: return 4;
    case 1: case 30: return 2;
    case 2: return 18;
    case 3: return 20;
    case 6: return 22;
    case 7: return 24;
    case 8: return 34;
    case 9: return 40;
    case 10: return 84;
    case 11: return 110;
    case 12: return 144;
    case 13: return 176;
    case 14: return 210;
    case 15: return 292;
    default: return 4;
  }
}

struct Meta {
  // the table index; the public VBQ_GGUF_META_* kind is this + 1
  enum Kind { kInt, kFloat, kBool, kString, kIntArray, kFloatArray, kStringArray } kind;
  int64_t i = 0;
  double f = 0;  // f32 and f64 values as the reference keeps them (float)
  bool b = false;
  std::string s;
  std::vector<int64_t> ia;
  std::vector<float> fa;
  std::vector<std::string> sa;
};

struct Tensor {
  std::string name;
  int32_t n_dims = 0;
  int64_t dims[4] = {1, 1, 1, 1};
  int32_t type = 0;
  uint64_t offset = 0;  // from the start of the data section
  uint64_t size = 0;
};

}  // namespace

struct vbq_gguf {
  int fd = -1;
  const uint8_t* base = nullptr;
  size_t file_size = 0;
  size_t data_offset = 0;
  uint32_t version = 0;
  std::vector<Tensor> tensors;
  std::unordered_map<std::string, size_t> by_name;  // the last tensor of a name wins
  std::unordered_map<std::string, Meta> meta[7];    // one table per Meta::Kind
  // pinned staging buffers of the uploads (allocated on first use)
  void* stage[2] = {nullptr, nullptr};
  cudaEvent_t stage_done[2] = {nullptr, nullptr};
  size_t stage_bytes = 0;
};

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF"
constexpr uint32_t kMaxVersion = 3;
constexpr size_t kAlign = 32;

// Bounds-checked little-endian reader over the mapping; every error carries the
// reference's message.
struct Cursor {
  const uint8_t* p;
  size_t size, off;
  template <typename T>
  bool get(T* v, std::string* err) {
    if (off + sizeof(T) > size) {
      *err = "GGUF: read past end of file at offset " + std::to_string(off);
      return false;
    }
    std::memcpy(v, p + off, sizeof(T));
    off += sizeof(T);
    return true;
  }
  bool skip(uint64_t n, std::string* err) {
    if (n > size || off + n > size) {
      *err = "GGUF: read past end of file at offset " + std::to_string(off);
      return false;
    }
    off += n;
    return true;
  }
  bool str(std::string* s, std::string* err) {
    if (off + 8 > size) {
      *err = "GGUF: string length extends past end of file";
      return false;
    }
    uint64_t n;
    std::memcpy(&n, p + off, 8);
    off += 8;
    if (n > size || off + n > size) {
      *err = "GGUF: string data extends past end of file";
      return false;
    }
    s->assign(reinterpret_cast<const char*>(p + off), n);
    off += n;
    return true;
  }
};

bool parse_value(Cursor& c, uint32_t vt, Meta* m, bool* keep, std::string* err) {
  *keep = true;
  switch (vt) {
    case 0: { uint8_t v; if (!c.get(&v, err)) return false; m->kind = Meta::kInt; m->i = v; return true; }
    case 1: { int8_t v; if (!c.get(&v, err)) return false; m->kind = Meta::kInt; m->i = v; return true; }
    case 2: case 3: *keep = false; return c.skip(2, err);  // 16-bit values are not kept
    case 4: { uint32_t v; if (!c.get(&v, err)) return false; m->kind = Meta::kInt; m->i = (int32_t)v; return true; }
    case 5: { int32_t v; if (!c.get(&v, err)) return false; m->kind = Meta::kInt; m->i = v; return true; }
    case 6: { float v; if (!c.get(&v, err)) return false; m->kind = Meta::kFloat; m->f = v; return true; }
    case 7: { uint8_t v; if (!c.get(&v, err)) return false; m->kind = Meta::kBool; m->b = v != 0; return true; }
    case 8: m->kind = Meta::kString; return c.str(&m->s, err);
    case 10: { uint64_t v; if (!c.get(&v, err)) return false; m->kind = Meta::kInt; m->i = (int64_t)v; return true; }
    case 11: { int64_t v; if (!c.get(&v, err)) return false; m->kind = Meta::kInt; m->i = v; return true; }
    case 12: { double v; if (!c.get(&v, err)) return false; m->kind = Meta::kFloat; m->f = (float)v; return true; }
    case 9: {
      uint32_t et;
      uint64_t n;
      if (c.off + 12 > c.size) {
        *err = "GGUF: read past end of file at offset " + std::to_string(c.off);
        return false;
      }
      c.get(&et, err);
      c.get(&n, err);
      switch (et) {
        case 8:
          m->kind = Meta::kStringArray;
          for (uint64_t j = 0; j < n; ++j) {
            std::string s;
            if (!c.str(&s, err)) return false;
            m->sa.push_back(std::move(s));
          }
          return true;
        case 4: case 5:
          m->kind = Meta::kIntArray;
          if (n > c.size / 4) return c.skip(n * 4, err);
          for (uint64_t j = 0; j < n; ++j) { int32_t v; if (!c.get(&v, err)) return false; m->ia.push_back(v); }
          return true;
        case 10: case 11:
          m->kind = Meta::kIntArray;
          if (n > c.size / 8) return c.skip(n * 8, err);
          for (uint64_t j = 0; j < n; ++j) { int64_t v; if (!c.get(&v, err)) return false; m->ia.push_back(v); }
          return true;
        case 6:
          m->kind = Meta::kFloatArray;
          if (n > c.size / 4) return c.skip(n * 4, err);
          for (uint64_t j = 0; j < n; ++j) { float v; if (!c.get(&v, err)) return false; m->fa.push_back(v); }
          return true;
        default: {
          *keep = false;
          const uint64_t es = (et == 0 || et == 1 || et == 7) ? 1 : (et == 2 || et == 3) ? 2 : (et == 12) ? 8 : 4;
          if (n > c.size / es) {
            *err = "GGUF: read past end of file at offset " + std::to_string(c.off);
            return false;
          }
          return c.skip(n * es, err);
        }
      }
    }
    default:
      *err = "Unknown GGUF metadata type: " + std::to_string(vt);
      return false;
  }
}

int parse(vbq_gguf* g) {
  std::string err;
  if (g->file_size < 24) return fail(VBQ_ERR_FORMAT, "GGUF file too small for header");
  Cursor c{g->base, g->file_size, 0};
  uint32_t magic;
  uint64_t n_tensors, n_kv;
  c.get(&magic, &err);
  if (magic != kMagic) return fail(VBQ_ERR_FORMAT, "Not a GGUF file (bad magic)");
  c.get(&g->version, &err);
  if (g->version > kMaxVersion)
    return fail(VBQ_ERR_FORMAT, "Unsupported GGUF version: " + std::to_string(g->version));
  c.get(&n_tensors, &err);
  c.get(&n_kv, &err);
  if (n_tensors > 1000000 || n_kv > 1000000) return fail(VBQ_ERR_FORMAT, "GGUF: implausible tensor/kv count");
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key;
    if (!c.str(&key, &err)) return fail(VBQ_ERR_FORMAT, err);
    uint32_t vt;
    if (!c.get(&vt, &err)) return fail(VBQ_ERR_FORMAT, err);
    Meta m;
    bool keep = false;
    if (!parse_value(c, vt, &m, &keep, &err)) return fail(VBQ_ERR_FORMAT, err);
    if (keep) g->meta[m.kind][key] = std::move(m);
  }
  g->tensors.reserve(n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    Tensor t;
    if (!c.str(&t.name, &err)) return fail(VBQ_ERR_FORMAT, err);
    uint32_t nd;
    if (!c.get(&nd, &err)) return fail(VBQ_ERR_FORMAT, err);
    if (nd > 4) return fail(VBQ_ERR_FORMAT, "GGUF: tensor has >4 dimensions");
    t.n_dims = (int32_t)nd;
    if (c.off + (size_t)nd * 8 > c.size)
      return fail(VBQ_ERR_FORMAT, "GGUF: read past end of file at offset " + std::to_string(c.off));
    for (uint32_t d = 0; d < nd; ++d) {
      uint64_t v;
      c.get(&v, &err);
      t.dims[d] = (int64_t)v;
    }
    if (c.off + 12 > c.size)
      return fail(VBQ_ERR_FORMAT, "GGUF: read past end of file at offset " + std::to_string(c.off));
    uint32_t ty;
    c.get(&ty, &err);
    t.type = (int32_t)ty;
    c.get(&t.offset, &err);
    int64_t nv = t.dims[0];
    for (int d = 1; d < t.n_dims; ++d) nv *= t.dims[d];
    const int64_t bs = blck_size(t.type);
    t.size = (uint64_t)(((nv + bs - 1) / bs) * type_size(t.type));
    g->by_name[t.name] = g->tensors.size();
    g->tensors.push_back(std::move(t));
  }
  g->data_offset = (c.off + kAlign - 1) & ~(kAlign - 1);
  if (g->data_offset > g->file_size) return fail(VBQ_ERR_FORMAT, "GGUF: data section starts past end of file");
  return VBQ_OK;
}

const Tensor* tensor_at(const vbq_gguf* g, int64_t i) {
  return (g && i >= 0 && (size_t)i < g->tensors.size()) ? &g->tensors[(size_t)i] : nullptr;
}

// the tensor's bytes, checked to end inside the file (gguf.cpp:255-262)
int tensor_bytes(const vbq_gguf* g, const Tensor& t, const uint8_t** out) {
  const uint64_t end = g->data_offset + t.offset + t.size;
  if (t.offset > g->file_size || t.size > g->file_size || end > g->file_size)
    return fail(VBQ_ERR_FORMAT, "GGUF: tensor '" + t.name + "' data extends past end of file");
  *out = g->base + g->data_offset + t.offset;
  return VBQ_OK;
}

const Meta* meta_of(const vbq_gguf* g, const char* key, Meta::Kind kind) {
  if (!g || !key) return nullptr;
  auto it = g->meta[kind].find(key);
  return it != g->meta[kind].end() ? &it->second : nullptr;
}

}  // namespace

extern "C" {

const char* vbq_gguf_last_error(void) { return g_err.c_str(); }

int vbq_gguf_open(const char* path, vbq_gguf** out) {
  if (!path || !out) return fail(VBQ_ERR_NULL, "vbq_gguf_open: NULL argument");
  *out = nullptr;
  const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(VBQ_ERR_IO, std::string("Cannot open GGUF: ") + path);
  struct stat st;
  if (fstat(fd, &st) < 0) {
    ::close(fd);
    return fail(VBQ_ERR_IO, "Cannot stat GGUF");
  }
  auto* g = new vbq_gguf();
  g->fd = fd;
  g->file_size = (size_t)st.st_size;
  if (g->file_size > 0) {
    void* p = mmap(nullptr, g->file_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) {
      vbq_gguf_close(g);
      return fail(VBQ_ERR_IO, std::string("GGUF: cannot map ") + path);
    }
    g->base = static_cast<const uint8_t*>(p);
  }
  const int rc = parse(g);
  if (rc != VBQ_OK) {
    const std::string keep = g_err;
    vbq_gguf_close(g);
    return fail(rc, keep);
  }
  *out = g;
  g_err.clear();
  return VBQ_OK;
}

void vbq_gguf_close(vbq_gguf* g) {
  if (!g) return;
  for (int i = 0; i < 2; ++i) {
    if (g->stage_done[i]) cudaEventDestroy(g->stage_done[i]);
    if (g->stage[i]) cudaFreeHost(g->stage[i]);
  }
  if (g->base) munmap(const_cast<uint8_t*>(g->base), g->file_size);
  if (g->fd >= 0) ::close(g->fd);
  delete g;
}

int vbq_gguf_version(const vbq_gguf* g, uint32_t* out) {
  if (!g || !out) return fail(VBQ_ERR_NULL, "vbq_gguf_version: NULL argument");
  *out = g->version;
  return VBQ_OK;
}

int vbq_gguf_file_size(const vbq_gguf* g, uint64_t* out) {
  if (!g || !out) return fail(VBQ_ERR_NULL, "vbq_gguf_file_size: NULL argument");
  *out = g->file_size;
  return VBQ_OK;
}

int vbq_gguf_data_offset(const vbq_gguf* g, uint64_t* out) {
  if (!g || !out) return fail(VBQ_ERR_NULL, "vbq_gguf_data_offset: NULL argument");
  *out = g->data_offset;
  return VBQ_OK;
}

int vbq_gguf_n_tensors(const vbq_gguf* g, int64_t* out) {
  if (!g || !out) return fail(VBQ_ERR_NULL, "vbq_gguf_n_tensors: NULL argument");
  *out = (int64_t)g->tensors.size();
  return VBQ_OK;
}

int vbq_gguf_tensor(const vbq_gguf* g, int64_t i, vbq_gguf_tensor_info* out) {
  const Tensor* t = tensor_at(g, i);
  if (!t || !out) return fail(VBQ_ERR_SHAPE, "vbq_gguf_tensor: no tensor " + std::to_string(i));
  out->name = t->name.c_str();
  out->n_dims = t->n_dims;
  for (int d = 0; d < 4; ++d) out->dims[d] = t->dims[d];
  out->type = t->type;
  out->offset = t->offset;
  out->size = t->size;
  return VBQ_OK;
}

int vbq_gguf_find(const vbq_gguf* g, const char* name, int64_t* index) {
  if (!g || !name || !index) return fail(VBQ_ERR_NULL, "vbq_gguf_find: NULL argument");
  auto it = g->by_name.find(name);
  *index = it == g->by_name.end() ? -1 : (int64_t)it->second;
  return VBQ_OK;
}

int vbq_gguf_tensor_data(const vbq_gguf* g, int64_t i, const void** data) {
  const Tensor* t = tensor_at(g, i);
  if (!t || !data) return fail(VBQ_ERR_SHAPE, "vbq_gguf_tensor_data: no tensor " + std::to_string(i));
  const uint8_t* p = nullptr;
  if (int rc = tensor_bytes(g, *t, &p)) return rc;
  *data = p;
  return VBQ_OK;
}

int vbq_gguf_meta_count(const vbq_gguf* g, const char* key, int32_t kind, int64_t* count) {
  if (!g || !key || !count) return fail(VBQ_ERR_NULL, "vbq_gguf_meta_count: NULL argument");
  if (kind < VBQ_GGUF_META_INT || kind > VBQ_GGUF_META_STRING_ARRAY)
    return fail(VBQ_ERR_SHAPE, "vbq_gguf_meta_count: unknown kind " + std::to_string(kind));
  const Meta* m = meta_of(g, key, static_cast<Meta::Kind>(kind - 1));
  if (!m) return fail(VBQ_ERR_NOT_FOUND, std::string("GGUF: no key ") + key + " of kind " + std::to_string(kind));
  switch (m->kind) {
    case Meta::kString: *count = (int64_t)m->s.size(); break;
    case Meta::kIntArray: *count = (int64_t)m->ia.size(); break;
    case Meta::kFloatArray: *count = (int64_t)m->fa.size(); break;
    case Meta::kStringArray: *count = (int64_t)m->sa.size(); break;
    default: *count = 1;
  }
  return VBQ_OK;
}

int vbq_gguf_meta_int(const vbq_gguf* g, const char* key, int64_t* out) {
  const Meta* m = meta_of(g, key, Meta::kInt);
  if (!m || !out) return fail(VBQ_ERR_NOT_FOUND, std::string("GGUF: no integer key ") + (key ? key : ""));
  *out = m->i;
  return VBQ_OK;
}

int vbq_gguf_meta_float(const vbq_gguf* g, const char* key, double* out) {
  const Meta* m = meta_of(g, key, Meta::kFloat);
  if (!m || !out) return fail(VBQ_ERR_NOT_FOUND, std::string("GGUF: no float key ") + (key ? key : ""));
  *out = m->f;
  return VBQ_OK;
}

int vbq_gguf_meta_bool(const vbq_gguf* g, const char* key, int32_t* out) {
  const Meta* m = meta_of(g, key, Meta::kBool);
  if (!m || !out) return fail(VBQ_ERR_NOT_FOUND, std::string("GGUF: no bool key ") + (key ? key : ""));
  *out = m->b ? 1 : 0;
  return VBQ_OK;
}

int vbq_gguf_meta_string(const vbq_gguf* g, const char* key, const char** str, int64_t* len) {
  const Meta* m = meta_of(g, key, Meta::kString);
  if (!m || !str || !len) return fail(VBQ_ERR_NOT_FOUND, std::string("GGUF: no string key ") + (key ? key : ""));
  *str = m->s.data();
  *len = (int64_t)m->s.size();
  return VBQ_OK;
}

int vbq_gguf_meta_int_array(const vbq_gguf* g, const char* key, int64_t* out, int64_t cap, int64_t* count) {
  const Meta* m = meta_of(g, key, Meta::kIntArray);
  if (!m || !count) return fail(VBQ_ERR_NOT_FOUND, std::string("GGUF: no integer array key ") + (key ? key : ""));
  *count = (int64_t)m->ia.size();
  for (int64_t j = 0; out && j < cap && j < *count; ++j) out[j] = m->ia[(size_t)j];
  return VBQ_OK;
}

int vbq_gguf_meta_float_array(const vbq_gguf* g, const char* key, float* out, int64_t cap, int64_t* count) {
  const Meta* m = meta_of(g, key, Meta::kFloatArray);
  if (!m || !count) return fail(VBQ_ERR_NOT_FOUND, std::string("GGUF: no float array key ") + (key ? key : ""));
  *count = (int64_t)m->fa.size();
  for (int64_t j = 0; out && j < cap && j < *count; ++j) out[j] = m->fa[(size_t)j];
  return VBQ_OK;
}

int vbq_gguf_meta_string_at(const vbq_gguf* g, const char* key, int64_t j, const char** str, int64_t* len) {
  const Meta* m = meta_of(g, key, Meta::kStringArray);
  if (!m || !str || !len || j < 0 || j >= (int64_t)m->sa.size())
    return fail(VBQ_ERR_NOT_FOUND, std::string("GGUF: no string array element of ") + (key ? key : ""));
  *str = m->sa[(size_t)j].data();
  *len = (int64_t)m->sa[(size_t)j].size();
  return VBQ_OK;
}

int vbq_gguf_upload(vbq_gguf* g, int64_t i, int64_t row0, int64_t row1, int64_t col0, int64_t col1,
                    void* dst, int64_t dst_row_bytes, void* stream) {
  const Tensor* t = tensor_at(g, i);
  if (!t) return fail(VBQ_ERR_SHAPE, "vbq_gguf_upload: no tensor " + std::to_string(i));
  // the tensor as K rows of N values (dims[0] = N, the rest = K), the layout gemv_dequant reads
  const int64_t N = t->dims[0];
  int64_t K = 1;
  for (int d = 1; d < t->n_dims; ++d) K *= t->dims[d];
  const int64_t bv = blck_size(t->type), bb = type_size(t->type);
  if (N <= 0 || N % bv != 0)
    return fail(VBQ_ERR_SHAPE, "vbq_gguf_upload: rows of '" + t->name + "' are not whole blocks");
  if (row0 < 0 || row1 > K || row0 > row1 || col0 < 0 || col1 > N || col0 > col1 || col0 % bv || col1 % bv)
    return fail(VBQ_ERR_SHAPE, "vbq_gguf_upload: rows [" + std::to_string(row0) + ", " + std::to_string(row1) +
                                   ") x columns [" + std::to_string(col0) + ", " + std::to_string(col1) +
                                   ") is outside '" + t->name + "' or not block-aligned");
  const uint8_t* src = nullptr;
  if (int rc = tensor_bytes(g, *t, &src)) return rc;
  if (!dst && row1 > row0 && col1 > col0) return fail(VBQ_ERR_NULL, "vbq_gguf_upload: dst is NULL");
  const int64_t rb = (N / bv) * bb;
  const int64_t wb = ((col1 - col0) / bv) * bb;  // bytes of a shard row
  if (dst_row_bytes < wb) return fail(VBQ_ERR_SHAPE, "vbq_gguf_upload: dst_row_bytes below the shard's row bytes");
  const int64_t rows = row1 - row0;
  if (rows == 0 || wb == 0) return VBQ_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (!g->stage[0]) {  // two pinned 32 MiB staging buffers, kept for the file's lifetime
    g->stage_bytes = (size_t)32 << 20;
    for (int s = 0; s < 2; ++s) {
      if ((e = cudaHostAlloc(&g->stage[s], g->stage_bytes, cudaHostAllocDefault)) != cudaSuccess ||
          (e = cudaEventCreateWithFlags(&g->stage_done[s], cudaEventDisableTiming)) != cudaSuccess)
        return fail(VBQ_ERR_CUDA, std::string("vbq_gguf_upload: staging buffers: ") + cudaGetErrorString(e));
    }
  }
  if (dst_row_bytes > wb) {  // padding bytes of each destination row read as zero
    if ((e = cudaMemsetAsync(dst, 0, (size_t)(dst_row_bytes * rows), st)) != cudaSuccess)
      return fail(VBQ_ERR_CUDA, std::string("vbq_gguf_upload: memset: ") + cudaGetErrorString(e));
  }
  // chunks of whole rows through the two buffers in turn: copy a chunk on the host while
  // the previous one crosses to the device
  const int64_t chunk_rows = (int64_t)g->stage_bytes / wb;
  if (chunk_rows == 0) return fail(VBQ_ERR_SHAPE, "vbq_gguf_upload: a shard row exceeds the 32 MiB staging buffer");
  const uint8_t* s0 = src + row0 * rb + (col0 / bv) * bb;
  uint8_t* d0 = static_cast<uint8_t*>(dst);
  int s = 0;
  for (int64_t r = 0; r < rows; r += chunk_rows, s ^= 1) {
    const int64_t n = rows - r < chunk_rows ? rows - r : chunk_rows;
    if ((e = cudaEventSynchronize(g->stage_done[s])) != cudaSuccess)
      return fail(VBQ_ERR_CUDA, std::string("vbq_gguf_upload: ") + cudaGetErrorString(e));
    uint8_t* buf = static_cast<uint8_t*>(g->stage[s]);
    for (int64_t j = 0; j < n; ++j) std::memcpy(buf + j * wb, s0 + (r + j) * rb, (size_t)wb);
    if ((e = cudaMemcpy2DAsync(d0 + r * dst_row_bytes, (size_t)dst_row_bytes, buf, (size_t)wb, (size_t)wb,
                               (size_t)n, cudaMemcpyHostToDevice, st)) != cudaSuccess ||
        (e = cudaEventRecord(g->stage_done[s], st)) != cudaSuccess)
      return fail(VBQ_ERR_CUDA, std::string("vbq_gguf_upload: copy: ") + cudaGetErrorString(e));
  }
  // the staging buffers are reused by the next upload: wait until both have been read
  for (int k = 0; k < 2; ++k)
    if ((e = cudaEventSynchronize(g->stage_done[k])) != cudaSuccess)
      return fail(VBQ_ERR_CUDA, std::string("vbq_gguf_upload: ") + cudaGetErrorString(e));
  return VBQ_OK;
}

}  // extern "C"
