// GGUF container reader (host code). Replaces parse_gguf / get_tensor
// (src/gguf_loader.rs:341-408, 536-584) for the quantized path: the file is
// memory-mapped (no whole-file copy), header, metadata and tensor infos are
// parsed with the reference's rules and error messages, and Q4_0 / Q8_0
// tensors go to the device as their blocks, re-laid-out into the tiled
// format of the GEMV/GEMM kernels without an f32 dequantization.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <string>
#include <vector>

#include "vxb_internal.h"

using namespace vxb;

namespace {

constexpr uint32_t kMagic = 0x46475547u;  // "GGUF"
constexpr uint64_t kDefaultAlignment = 32;

// GGUFValueType (src/gguf_loader.rs:21-36)
enum { T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STRING, T_ARRAY, T_U64, T_I64, T_F64 };

// GGMLQuantType block geometry (src/gguf_loader.rs:61-128): bytes, elements
bool ggml_block(uint32_t t, uint64_t *bytes, uint64_t *elems) {
  switch (t) {
    case 0: *bytes = 4; *elems = 1; return true;      // F32
    case 1: *bytes = 2; *elems = 1; return true;      // F16
    case 2: *bytes = 18; *elems = 32; return true;    // Q4_0
    case 3: *bytes = 20; *elems = 32; return true;    // Q4_1
    case 6: *bytes = 22; *elems = 32; return true;    // Q5_0
    case 7: *bytes = 24; *elems = 32; return true;    // Q5_1
    case 8: *bytes = 34; *elems = 32; return true;    // Q8_0
    case 10: *bytes = 84; *elems = 256; return true;  // Q2_K
    case 11: *bytes = 110; *elems = 256; return true; // Q3_K
    case 12: *bytes = 144; *elems = 256; return true; // Q4_K
    case 13: *bytes = 176; *elems = 256; return true; // Q5_K
    case 14: *bytes = 210; *elems = 256; return true; // Q6_K
    default: return false;
  }
}

struct Meta {
  std::string key;
  uint32_t type = 0;
  int64_t ival = 0;       // integer and bool values
  double fval = 0;        // f32 / f64 values
  std::string sval;       // strings
  uint32_t elem_type = 0; // arrays
  uint64_t count = 0;
};

struct Tensor {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0, nbytes = 0, nelems = 0;
};

struct Reader {
  const uint8_t *p;
  size_t n, pos = 0;
  std::string err;
  bool take(size_t k, const char *what) {
    if (n - pos < k) {
      if (err.empty()) err = std::string("unexpected EOF reading ") + what;
      return false;
    }
    return true;
  }
  bool u8(uint8_t *v) {
    if (!take(1, "u8")) return false;
    *v = p[pos++];
    return true;
  }
  bool u16(uint16_t *v) {
    if (!take(2, "u16")) return false;
    memcpy(v, p + pos, 2);
    pos += 2;
    return true;
  }
  bool u32(uint32_t *v) {
    if (!take(4, "u32")) return false;
    memcpy(v, p + pos, 4);
    pos += 4;
    return true;
  }
  bool u64(uint64_t *v) {
    if (!take(8, "u64")) return false;
    memcpy(v, p + pos, 8);
    pos += 8;
    return true;
  }
  bool str(std::string *s) {
    uint64_t len;
    if (!u64(&len)) return false;
    if (n - pos < len) {
      if (err.empty()) err = "unexpected EOF reading string of length " + std::to_string(len);
      return false;
    }
    if (!valid_utf8(p + pos, (size_t)len)) {
      if (err.empty()) err = "invalid UTF-8 in GGUF string";
      return false;
    }
    s->assign(reinterpret_cast<const char *>(p + pos), (size_t)len);
    pos += len;
    return true;
  }
  // UTF-8 as Rust's str::from_utf8 accepts it (no overlong forms, no
  // surrogates, nothing above U+10FFFF)
  static bool valid_utf8(const uint8_t *s, size_t len) {
    size_t i = 0;
    while (i < len) {
      const uint8_t c = s[i];
      if (c < 0x80) {
        i++;
        continue;
      }
      int k;
      uint32_t cp;
      if ((c >> 5) == 6) {
        k = 1;
        cp = c & 0x1F;
      } else if ((c >> 4) == 14) {
        k = 2;
        cp = c & 0x0F;
      } else if ((c >> 3) == 30) {
        k = 3;
        cp = c & 0x07;
      } else {
        return false;
      }
      if (len - i <= (size_t)k) return false;
      for (int j = 1; j <= k; j++) {
        if ((s[i + j] & 0xC0) != 0x80) return false;
        cp = (cp << 6) | (s[i + j] & 0x3F);
      }
      if ((k == 1 && cp < 0x80) || (k == 2 && (cp < 0x800 || (cp >= 0xD800 && cp <= 0xDFFF))) ||
          (k == 3 && (cp < 0x10000 || cp > 0x10FFFF)))
        return false;
      i += k + 1;
    }
    return true;
  }
  // one value of type t (arrays: elements read and dropped, count kept)
  bool value(uint32_t t, Meta *m, int depth) {
    uint8_t b;
    uint16_t h;
    uint32_t w;
    uint64_t q;
    switch (t) {
      case T_U8: if (!u8(&b)) return false; m->ival = b; return true;
      case T_I8: if (!u8(&b)) return false; m->ival = (int8_t)b; return true;
      case T_U16: if (!u16(&h)) return false; m->ival = h; return true;
      case T_I16: if (!u16(&h)) return false; m->ival = (int16_t)h; return true;
      case T_U32: if (!u32(&w)) return false; m->ival = w; return true;
      case T_I32: if (!u32(&w)) return false; m->ival = (int32_t)w; return true;
      case T_F32: {
        if (!u32(&w)) return false;
        float f;
        memcpy(&f, &w, 4);
        m->fval = f;
        return true;
      }
      case T_BOOL: if (!u8(&b)) return false; m->ival = b != 0; return true;
      case T_STRING: return str(&m->sval);
      case T_ARRAY: {
        uint32_t et;
        if (!u32(&et)) return false;
        if (et > T_F64) {
          if (err.empty()) err = "unknown GGUF value type: " + std::to_string(et);
          return false;
        }
        if (!u64(&q)) return false;
        m->elem_type = et;
        m->count = q;
        Meta scratch;
        for (uint64_t i = 0; i < q; i++)
          if (!value(et, &scratch, depth + 1)) return false;
        return true;
      }
      case T_U64: if (!u64(&q)) return false; m->ival = (int64_t)q; return true;
      case T_I64: if (!u64(&q)) return false; m->ival = (int64_t)q; return true;
      case T_F64: {
        if (!u64(&q)) return false;
        double d;
        memcpy(&d, &q, 8);
        m->fval = d;
        return true;
      }
      default:
        if (err.empty()) err = "unknown GGUF value type: " + std::to_string(t);
        return false;
    }
  }
};

}  // namespace

struct vxb_gguf {
  const uint8_t *data = nullptr;
  size_t size = 0;
  bool mapped = false;
  uint32_t version = 0;
  uint64_t alignment = kDefaultAlignment, data_offset = 0;
  std::vector<Meta> meta;
  std::vector<Tensor> tensors;
};

namespace {

// parse_gguf (src/gguf_loader.rs:341-408)
int parse(vxb_gguf *g) {
  Reader r{g->data, g->size};
  uint32_t magic;
  uint64_t n_tensors, n_kv;
  if (!r.u32(&magic)) return set_error(nullptr, VXB_EFORMAT, "%s", r.err.c_str());
  if (magic != kMagic)
    return set_error(nullptr, VXB_EFORMAT, "invalid GGUF magic: 0x%08X (expected 0x%08X)", magic, kMagic);
  if (!r.u32(&g->version)) return set_error(nullptr, VXB_EFORMAT, "%s", r.err.c_str());
  if (g->version != 2 && g->version != 3)
    return set_error(nullptr, VXB_EFORMAT, "unsupported GGUF version: %u", g->version);
  if (!r.u64(&n_tensors) || !r.u64(&n_kv)) return set_error(nullptr, VXB_EFORMAT, "%s", r.err.c_str());
  for (uint64_t i = 0; i < n_kv; i++) {
    Meta m;
    if (!r.str(&m.key) || !r.u32(&m.type)) return set_error(nullptr, VXB_EFORMAT, "%s", r.err.c_str());
    if (m.type > T_F64) return set_error(nullptr, VXB_EFORMAT, "unknown GGUF value type: %u", m.type);
    if (!r.value(m.type, &m, 0)) return set_error(nullptr, VXB_EFORMAT, "%s", r.err.c_str());
    g->meta.push_back(std::move(m));
  }
  for (const Meta &m : g->meta)
    if (m.key == "general.alignment" && (m.type == T_U32 || m.type == T_U64 || m.type == T_I32) && m.ival > 0)
      g->alignment = (uint64_t)m.ival;
  for (uint64_t i = 0; i < n_tensors; i++) {
    Tensor t;
    uint32_t nd;
    if (!r.str(&t.name) || !r.u32(&nd)) return set_error(nullptr, VXB_EFORMAT, "%s", r.err.c_str());
    t.nelems = 1;
    for (uint32_t k = 0; k < nd; k++) {
      uint64_t dim;
      if (!r.u64(&dim)) return set_error(nullptr, VXB_EFORMAT, "%s", r.err.c_str());
      t.dims.push_back(dim);
      t.nelems *= dim;
    }
    if (!r.u32(&t.type) || !r.u64(&t.offset)) return set_error(nullptr, VXB_EFORMAT, "%s", r.err.c_str());
    uint64_t bb, be;
    if (!ggml_block(t.type, &bb, &be)) return set_error(nullptr, VXB_EFORMAT, "unknown GGML quant type: %u", t.type);
    t.nbytes = (t.nelems + be - 1) / be * bb;  // GGUFTensorInfo::data_size
    g->tensors.push_back(std::move(t));
  }
  g->data_offset = (r.pos + g->alignment - 1) / g->alignment * g->alignment;
  return VXB_OK;
}

const Meta *find_meta(const vxb_gguf *g, const char *key) {
  for (const Meta &m : g->meta)
    if (m.key == key) return &m;
  return nullptr;
}

}  // namespace

VXB_API int vxb_gguf_open_memory(const void *data, size_t nbytes, vxb_gguf **out) {
  if (!data || !out) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_open_memory: null argument");
  *out = nullptr;
  vxb_gguf *g = new vxb_gguf();
  g->data = (const uint8_t *)data;
  g->size = nbytes;
  if (int rc = parse(g)) {
    delete g;
    return rc;
  }
  *out = g;
  return VXB_OK;
}

VXB_API int vxb_gguf_open(const char *path, vxb_gguf **out) {
  if (!path || !out) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_open: null argument");
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_open: cannot open %s", path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    close(fd);
    return set_error(nullptr, VXB_EFORMAT, "unexpected EOF reading u32");
  }
  void *p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_open: mmap of %s failed", path);
  vxb_gguf *g = new vxb_gguf();
  g->data = (const uint8_t *)p;
  g->size = (size_t)st.st_size;
  g->mapped = true;
  if (int rc = parse(g)) {
    munmap(p, g->size);
    delete g;
    return rc;
  }
  *out = g;
  return VXB_OK;
}

VXB_API int vxb_gguf_close(vxb_gguf *g) {
  if (!g) return VXB_OK;
  if (g->mapped) munmap(const_cast<uint8_t *>(g->data), g->size);
  delete g;
  return VXB_OK;
}

VXB_API int vxb_gguf_info(const vxb_gguf *g, uint32_t *version, int64_t *n_tensors, int64_t *n_metadata,
                          uint64_t *data_offset, uint64_t *alignment) {
  if (!g) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_info: null handle");
  if (version) *version = g->version;
  if (n_tensors) *n_tensors = (int64_t)g->tensors.size();
  if (n_metadata) *n_metadata = (int64_t)g->meta.size();
  if (data_offset) *data_offset = g->data_offset;
  if (alignment) *alignment = g->alignment;
  return VXB_OK;
}

VXB_API int vxb_gguf_tensor(const vxb_gguf *g, int64_t i, char *name, size_t name_cap, int *ggml_type, int *n_dims,
                            uint64_t *dims4, uint64_t *offset, uint64_t *nbytes, const void **h_data) {
  if (!g) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_tensor: null handle");
  if (i < 0 || i >= (int64_t)g->tensors.size()) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_tensor: index %lld", (long long)i);
  const Tensor &t = g->tensors[(size_t)i];
  if (name && name_cap) {
    const size_t k = std::min(name_cap - 1, t.name.size());
    memcpy(name, t.name.data(), k);
    name[k] = 0;
  }
  if (ggml_type) *ggml_type = (int)t.type;
  if (n_dims) *n_dims = (int)t.dims.size();
  if (dims4)
    for (int k = 0; k < 4; k++) dims4[k] = k < (int)t.dims.size() ? t.dims[k] : 1;
  if (offset) *offset = t.offset;
  if (nbytes) *nbytes = t.nbytes;
  if (h_data) {
    // get_tensor's bounds check (src/gguf_loader.rs:545-552)
    const uint64_t start = g->data_offset + t.offset, end = start + t.nbytes;
    if (end > g->size)
      return set_error(nullptr, VXB_EFORMAT,
                       "tensor '%s' data extends beyond file (need %llu bytes at offset %llu, file is %zu bytes)",
                       t.name.c_str(), (unsigned long long)t.nbytes, (unsigned long long)start, g->size);
    *h_data = g->data + start;
  }
  return VXB_OK;
}

VXB_API int vxb_gguf_find_tensor(const vxb_gguf *g, const char *name, int64_t *index) {
  if (!g || !name || !index) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_find_tensor: null argument");
  for (size_t i = 0; i < g->tensors.size(); i++)
    if (g->tensors[i].name == name) {
      *index = (int64_t)i;
      return VXB_OK;
    }
  return set_error(nullptr, VXB_EINVAL, "tensor '%s' not found in GGUF file", name);
}

VXB_API int vxb_gguf_meta_int(const vxb_gguf *g, const char *key, int64_t *value) {
  if (!g || !key || !value) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_meta_int: null argument");
  const Meta *m = find_meta(g, key);
  if (!m) return set_error(nullptr, VXB_EINVAL, "metadata key '%s' not found", key);
  if (m->type == T_F32 || m->type == T_F64 || m->type == T_STRING || m->type == T_ARRAY)
    return set_error(nullptr, VXB_EINVAL, "metadata '%s' is not an integer", key);
  *value = m->ival;
  return VXB_OK;
}

VXB_API int vxb_gguf_meta_float(const vxb_gguf *g, const char *key, double *value) {
  if (!g || !key || !value) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_meta_float: null argument");
  const Meta *m = find_meta(g, key);
  if (!m) return set_error(nullptr, VXB_EINVAL, "metadata key '%s' not found", key);
  if (m->type != T_F32 && m->type != T_F64) return set_error(nullptr, VXB_EINVAL, "metadata '%s' is not a float", key);
  *value = m->fval;
  return VXB_OK;
}

VXB_API int vxb_gguf_meta_string(const vxb_gguf *g, const char *key, char *out, size_t cap, size_t *len) {
  if (!g || !key) return set_error(nullptr, VXB_EINVAL, "vxb_gguf_meta_string: null argument");
  const Meta *m = find_meta(g, key);
  if (!m) return set_error(nullptr, VXB_EINVAL, "metadata key '%s' not found", key);
  if (m->type != T_STRING) return set_error(nullptr, VXB_EINVAL, "metadata '%s' is not a string", key);
  if (len) *len = m->sval.size();
  if (out && cap) {
    const size_t k = std::min(cap - 1, m->sval.size());
    memcpy(out, m->sval.data(), k);
    out[k] = 0;
  }
  return VXB_OK;
}

// A Q4_0 / Q8_0 tensor to the device tiled layout: rows N = product of the
// dimensions after the first, K = the first (fastest) dimension, so the
// blocks run along K as stored.
VXB_API int vxb_gguf_upload_tiled(vxb_ctx *ctx, const vxb_gguf *g, int64_t i, void *d_tiled, size_t tiled_bytes,
                                  void *stream) {
  if (!ctx || !g || !d_tiled) return set_error(ctx, VXB_EINVAL, "vxb_gguf_upload_tiled: null argument");
  const void *src = nullptr;
  int type = 0, nd = 0;
  uint64_t dims[4], nbytes = 0;
  if (int rc = vxb_gguf_tensor(g, i, nullptr, 0, &type, &nd, dims, nullptr, &nbytes, &src)) {
    set_error(ctx, rc, "%s", vxb_last_error(nullptr));
    return rc;
  }
  if (type != VXB_Q4_0 && type != VXB_Q8_0)
    return set_error(ctx, VXB_EUNSUPPORTED, "vxb_gguf_upload_tiled: tensor type %d (Q4_0 or Q8_0 only)", type);
  const uint64_t K = dims[0], N = dims[1] * dims[2] * dims[3];
  if (K % 32 || N == 0 || N > 0x7FFFFFFF || K > 0x7FFFFFFF)
    return set_error(ctx, VXB_EINVAL, "vxb_gguf_upload_tiled: shape %llu x %llu", (unsigned long long)N, (unsigned long long)K);
  if (tiled_bytes < vxb_tiled_bytes(type, (int)N, (int)K))
    return set_error(ctx, VXB_EINVAL, "vxb_gguf_upload_tiled: tiled buffer of %zu bytes, need %zu", tiled_bytes,
                     vxb_tiled_bytes(type, (int)N, (int)K));
  if (int rc = use_device(ctx)) return rc;
  void *d_blocks = nullptr;
  if (cudaMalloc(&d_blocks, nbytes) != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, VXB_ENOMEM, "vxb_gguf_upload_tiled: staging of %llu bytes", (unsigned long long)nbytes);
  }
  cudaStream_t st = (cudaStream_t)stream;
  int rc = cudaMemcpyAsync(d_blocks, src, nbytes, cudaMemcpyHostToDevice, st) == cudaSuccess
               ? VXB_OK : set_error(ctx, VXB_ECUDA, "vxb_gguf_upload_tiled: copy");
  if (!rc) rc = vxb_tile_weights(ctx, type, (const uint8_t *)d_blocks, (int)N, (int)K, d_tiled, stream);
  cudaStreamSynchronize(st);
  cudaFree(d_blocks);
  return rc;
}

VXB_API int vxb_gguf_upload(vxb_ctx *ctx, const vxb_gguf *g, int64_t i, void *d_dst, size_t dst_bytes, void *stream) {
  if (!ctx || !g || !d_dst) return set_error(ctx, VXB_EINVAL, "vxb_gguf_upload: null argument");
  const void *src = nullptr;
  uint64_t nbytes = 0;
  if (int rc = vxb_gguf_tensor(g, i, nullptr, 0, nullptr, nullptr, nullptr, nullptr, &nbytes, &src)) {
    set_error(ctx, rc, "%s", vxb_last_error(nullptr));
    return rc;
  }
  if (dst_bytes < nbytes)
    return set_error(ctx, VXB_EINVAL, "vxb_gguf_upload: buffer of %zu bytes, the tensor holds %llu", dst_bytes,
                     (unsigned long long)nbytes);
  if (int rc = use_device(ctx)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  VXB_CUDA_TRY(ctx, cudaMemcpyAsync(d_dst, src, nbytes, cudaMemcpyHostToDevice, st));
  VXB_CUDA_TRY(ctx, cudaStreamSynchronize(st));  // the mapping may be closed right after
  return VXB_OK;
}
