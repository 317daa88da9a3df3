// ref_gguf_shim.cpp -- TEST INFRASTRUCTURE ONLY: extern "C" access to the reference's own
// GGUF reader (vibeblade::GGUFFile, cpp/include/gguf.h, cpp/src/gguf.cpp), so the tests
// can read the same files with it and with vibeblade_b200's reader and compare.  Built by
// oracle/build.py together with the reference's gguf.cpp into oracle/_ref/libvbref_gguf.so;
// nothing in the product links it.  Exceptions become a NULL handle / -1 and a message.
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "gguf.h"

namespace {
thread_local std::string g_msg;
void put(char* buf, int64_t cap, const std::string& s) {
  if (!buf || cap <= 0) return;
  const size_t n = s.size() < (size_t)(cap - 1) ? s.size() : (size_t)(cap - 1);
  std::memcpy(buf, s.data(), n);
  buf[n] = 0;
}
vibeblade::GGUFFile* F(void* h) { return static_cast<vibeblade::GGUFFile*>(h); }
}  // namespace

extern "C" {

const char* vbr_gguf_error(void) { return g_msg.c_str(); }

void* vbr_gguf_open(const char* path) {
  try {
    return new vibeblade::GGUFFile(path);
  } catch (const std::exception& e) {
    g_msg = e.what();
    return nullptr;
  }
}

void vbr_gguf_close(void* h) { delete F(h); }
int64_t vbr_gguf_version(void* h) { return F(h)->version(); }
int64_t vbr_gguf_n_tensors(void* h) { return (int64_t)F(h)->tensors().size(); }

// tensor i of the table: name into buf, the rest through the pointers
int vbr_gguf_tensor(void* h, int64_t i, char* name, int64_t cap, int32_t* n_dims, int64_t* dims,
                    int32_t* type, uint64_t* offset, uint64_t* size) {
  const auto& ts = F(h)->tensors();
  if (i < 0 || (size_t)i >= ts.size()) return -1;
  const auto& t = ts[(size_t)i];
  put(name, cap, t.name);
  *n_dims = t.n_dims;
  for (int d = 0; d < 4; ++d) dims[d] = t.dims[d];
  *type = (int32_t)t.type;
  *offset = t.offset;
  *size = t.size;
  return 0;
}

// tensor_data(name): 1 and the address, 0 when absent, -1 and a message when it throws
int vbr_gguf_tensor_data(void* h, const char* name, const void** data) {
  try {
    *data = F(h)->tensor_data(name);
    return *data ? 1 : 0;
  } catch (const std::exception& e) {
    g_msg = e.what();
    return -1;
  }
}

int vbr_gguf_has_tensor(void* h, const char* name) { return F(h)->tensor_info(name) != nullptr; }
int64_t vbr_gguf_meta_int(void* h, const char* key, int64_t dflt) { return F(h)->meta_int(key, dflt); }
double vbr_gguf_meta_float(void* h, const char* key, double dflt) { return F(h)->meta_float(key, (float)dflt); }
int vbr_gguf_meta_bool(void* h, const char* key, int dflt) { return F(h)->meta_bool(key, dflt != 0) ? 1 : 0; }
int64_t vbr_gguf_meta_string(void* h, const char* key, char* buf, int64_t cap) {
  const std::string s = F(h)->meta_string(key);
  put(buf, cap, s);
  return (int64_t)s.size();
}
int64_t vbr_gguf_meta_int_array(void* h, const char* key, int64_t* out, int64_t cap) {
  const auto v = F(h)->meta_int_array(key);
  for (int64_t j = 0; j < cap && (size_t)j < v.size(); ++j) out[j] = v[(size_t)j];
  return (int64_t)v.size();
}
int64_t vbr_gguf_meta_float_array(void* h, const char* key, float* out, int64_t cap) {
  const auto v = F(h)->meta_float_array(key);
  for (int64_t j = 0; j < cap && (size_t)j < v.size(); ++j) out[j] = v[(size_t)j];
  return (int64_t)v.size();
}
int64_t vbr_gguf_meta_string_array_len(void* h, const char* key) {
  return (int64_t)F(h)->meta_string_array(key).size();
}
int64_t vbr_gguf_meta_string_at(void* h, const char* key, int64_t j, char* buf, int64_t cap) {
  const auto v = F(h)->meta_string_array(key);
  if (j < 0 || (size_t)j >= v.size()) return -1;
  put(buf, cap, v[(size_t)j]);
  return (int64_t)v[(size_t)j].size();
}

}  // extern "C"
