// gguf.cu — a GGUF v2/v3 tensor-table reader (host code) for loading the
// MoE layers' expert slabs.
//
// Follows the reference's reader (crates/mrml-tensor/src/gguf.rs:80-181):
// little-endian header (magic "GGUF", version 2 or 3, tensor count, metadata
// count), metadata key/value pairs (13 value types, arrays nested), then per
// tensor its name, dimension count, up to 4 dimensions (extra ones skipped),
// GGML type id and data offset; the data section starts at the next multiple
// of `general.alignment` (default 32).  A tensor's size is
// numel / block_elements * block_bytes of its type.  The model loader then
// takes the expert slabs at data_offset + offset (model.rs:638-647) and
// uploads them unchanged (model.rs:726-741).
#include <stdio.h>
#include <string.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/mrml_moe.h"

namespace {

struct Tensor {
  int type = 0, n_dims = 0;
  int64_t dims[4] = {1, 1, 1, 1};
  uint64_t offset = 0, nbytes = 0;
};

struct File {
  std::string path;
  uint32_t version = 0;
  uint64_t data_offset = 0;
  std::map<std::string, Tensor> tensors;
  std::vector<std::string> order;             // tensor names in file order
  std::map<std::string, uint64_t> meta_uint;  // integer metadata that as_u32 accepts
};

// (elements, bytes) per block of the GGML types the reference reads
// (gguf.rs:121-133); false for the others.
bool type_block(int t, uint64_t* elems, uint64_t* bytes) {
  switch (t) {
    case 0: *elems = 1, *bytes = 4; return true;      // F32
    case 1: *elems = 1, *bytes = 2; return true;      // F16
    case 2: *elems = 32, *bytes = 18; return true;    // Q4_0
    case 3: *elems = 32, *bytes = 20; return true;    // Q4_1
    case 8: *elems = 32, *bytes = 34; return true;    // Q8_0
    case 12: *elems = 256, *bytes = 144; return true;  // Q4_K
    case 13: *elems = 256, *bytes = 176; return true;  // Q5_K
    case 14: *elems = 256, *bytes = 210; return true;  // Q6_K
    case 16: *elems = 256, *bytes = 136; return true;  // IQ4_XS
    case 30: *elems = 1, *bytes = 2; return true;     // BF16
    default: return false;
  }
}

struct Reader {
  FILE* f;
  bool ok = true;
  template <typename V>
  V get() {
    V v{};
    if (ok && fread(&v, sizeof(V), 1, f) != 1) ok = false;
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > (1ull << 30)) {
      ok = false;
      return {};
    }
    std::string s(n, '\0');
    if (n && fread(&s[0], 1, n, f) != n) ok = false;
    return s;
  }
  // Reads (and drops) one value of GGUF type `vt`; integer scalars are
  // returned through *u when they are non-negative (the reference's as_u32).
  bool value(uint32_t vt, uint64_t* u, int depth = 0) {
    *u = UINT64_MAX;
    switch (vt) {
      case 0: *u = get<uint8_t>(); break;
      case 1: { const int8_t v = get<int8_t>(); (void)v; break; }
      case 2: *u = get<uint16_t>(); break;
      case 3: { const int16_t v = get<int16_t>(); (void)v; break; }
      case 4: *u = get<uint32_t>(); break;
      case 5: { const int32_t v = get<int32_t>(); if (v >= 0) *u = (uint64_t)v; break; }
      case 6: get<float>(); break;
      case 7: get<uint8_t>(); break;
      case 8: str(); break;
      case 9: {
        if (depth > 8) return false;
        const uint32_t it = get<uint32_t>();
        const uint64_t n = get<uint64_t>();
        uint64_t dummy;
        for (uint64_t i = 0; ok && i < n; ++i)
          if (!value(it, &dummy, depth + 1)) return false;
        *u = UINT64_MAX;
        break;
      }
      case 10: *u = get<uint64_t>(); break;
      case 11: { const int64_t v = get<int64_t>(); if (v >= 0) *u = (uint64_t)v; break; }
      case 12: get<double>(); break;
      default: return false;  // unknown value type
    }
    return ok;
  }
};

int parse(const char* path, File* out) {
  FILE* f = fopen(path, "rb");
  if (!f) return MRML_ERR_INVALID_ARGUMENT;
  Reader r{f};
  int st = MRML_OK;
  do {
    if (r.get<uint32_t>() != 0x46554747u || !r.ok) { st = MRML_ERR_INVALID_ARGUMENT; break; }  // "GGUF"
    out->version = r.get<uint32_t>();
    if (out->version < 2 || out->version > 3) { st = MRML_ERR_UNSUPPORTED; break; }
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > (1ull << 24) || n_kv > (1ull << 24)) { st = MRML_ERR_INVALID_ARGUMENT; break; }
    for (uint64_t i = 0; i < n_kv && st == MRML_OK; ++i) {
      const std::string key = r.str();
      const uint32_t vt = r.get<uint32_t>();
      uint64_t u;
      if (!r.ok || !r.value(vt, &u)) { st = MRML_ERR_INVALID_ARGUMENT; break; }
      if (u != UINT64_MAX) out->meta_uint[key] = u;
    }
    if (st != MRML_OK) break;
    for (uint64_t i = 0; i < n_tensors; ++i) {
      Tensor t;
      const std::string name = r.str();
      const uint32_t nd = r.get<uint32_t>();
      for (uint32_t d = 0; d < nd && r.ok; ++d) {
        const uint64_t v = r.get<uint64_t>();
        if (d < 4) t.dims[d] = (int64_t)v;  // extra dimensions are skipped
      }
      t.n_dims = nd < 4 ? (int)nd : 4;
      t.type = (int)r.get<uint32_t>();
      t.offset = r.get<uint64_t>();
      if (!r.ok) { st = MRML_ERR_INVALID_ARGUMENT; break; }
      uint64_t be, bb;
      if (!type_block(t.type, &be, &bb)) { st = MRML_ERR_UNSUPPORTED; break; }
      uint64_t numel = 1;
      for (int d = 0; d < 4; ++d) numel *= (uint64_t)t.dims[d];
      t.nbytes = numel / be * bb;
      out->tensors[name] = t;
      out->order.push_back(name);
    }
    if (st != MRML_OK) break;
    auto a = out->meta_uint.find("general.alignment");
    const uint64_t align = a != out->meta_uint.end() && a->second > 0 && a->second <= UINT32_MAX ? a->second : 32;
    const long pos = ftell(f);
    if (pos < 0) { st = MRML_ERR_INVALID_ARGUMENT; break; }
    out->data_offset = ((uint64_t)pos + align - 1) / align * align;
    out->path = path;
  } while (false);
  fclose(f);
  return st;
}

const Tensor* find(const void* file, const char* name) {
  if (!file || !name) return nullptr;
  const File* g = static_cast<const File*>(file);
  auto it = g->tensors.find(name);
  return it == g->tensors.end() ? nullptr : &it->second;
}

}  // namespace

extern "C" {

int mrml_moe_gguf_open(const char* path, void** file) {
  if (!path || !file) return MRML_ERR_INVALID_ARGUMENT;
  *file = nullptr;
  File* g = new (std::nothrow) File();
  if (!g) return MRML_ERR_INVALID_ARGUMENT;
  const int st = parse(path, g);
  if (st != MRML_OK) {
    delete g;
    return st;
  }
  *file = g;
  return MRML_OK;
}

int mrml_moe_gguf_close(void* file) {
  delete static_cast<File*>(file);
  return MRML_OK;
}

int mrml_moe_gguf_version(const void* file) { return file ? (int)static_cast<const File*>(file)->version : 0; }

int mrml_moe_gguf_tensor_count(const void* file) {
  return file ? (int)static_cast<const File*>(file)->order.size() : 0;
}

const char* mrml_moe_gguf_tensor_name(const void* file, int i) {
  if (!file) return nullptr;
  const File* g = static_cast<const File*>(file);
  return i >= 0 && i < (int)g->order.size() ? g->order[i].c_str() : nullptr;
}

int mrml_moe_gguf_tensor(const void* file, const char* name, int* ggml_type, int* n_dims, int64_t* dims,
                         uint64_t* file_offset, uint64_t* nbytes) {
  const Tensor* t = find(file, name);
  if (!t) return MRML_ERR_NOT_FOUND;
  if (ggml_type) *ggml_type = t->type;
  if (n_dims) *n_dims = t->n_dims;
  if (dims)
    for (int d = 0; d < 4; ++d) dims[d] = t->dims[d];
  if (file_offset) *file_offset = static_cast<const File*>(file)->data_offset + t->offset;
  if (nbytes) *nbytes = t->nbytes;
  return MRML_OK;
}

int mrml_moe_gguf_meta_u32(const void* file, const char* key, uint32_t* value) {
  if (!file || !key || !value) return MRML_ERR_INVALID_ARGUMENT;
  const File* g = static_cast<const File*>(file);
  auto it = g->meta_uint.find(key);
  if (it == g->meta_uint.end()) return MRML_ERR_NOT_FOUND;
  *value = (uint32_t)it->second;  // as_u32: integer values, truncated like the reference's `as u32`
  return MRML_OK;
}

int mrml_moe_gguf_read(const void* file, const char* name, void* dst, size_t dst_bytes) {
  const Tensor* t = find(file, name);
  if (!t) return MRML_ERR_NOT_FOUND;
  if (!dst || dst_bytes < t->nbytes) return MRML_ERR_INVALID_ARGUMENT;
  const File* g = static_cast<const File*>(file);
  FILE* f = fopen(g->path.c_str(), "rb");
  if (!f) return MRML_ERR_INVALID_ARGUMENT;
  int st = MRML_OK;
  if (fseeko(f, (off_t)(g->data_offset + t->offset), SEEK_SET) != 0 || fread(dst, 1, t->nbytes, f) != t->nbytes)
    st = MRML_ERR_INVALID_ARGUMENT;
  fclose(f);
  return st;
}

}  // extern "C"
