// gguf.cu — GGUF directory reader and expert-tensor loader (host code).
//
// Parsing restates GgufReader::inspect / read_directory
// (har/crates/har-model/src/lib.rs:126-399,507-640): magic "GGUF", version
// 1..3, u64 tensor and metadata counts (each <= 10,000,000), metadata values
// of types 0..12 (arrays of up to 1,000,000 elements, strings of up to 2^30
// bytes), general.alignment (default 32, at least 1), tensor infos of rank
// <= 16, the data section at the first aligned offset after the infos, and
// each tensor's payload = ceil(elements / block) * block_bytes from the
// type tables (the span to the next tensor, or to the end of the file, when
// the type is not in the tables).
//
// Loading follows the expert layout HAR reads (expert_matvec,
// har/crates/har-demo/src/bin/har-native-qwen35moe.rs:626-689, and ExpertIndex,
// har/crates/har-storage/src/gguf.rs:300-403): a `*_exps` tensor has GGML
// dims [K, N, E] and expert e's rows at e*N*row_bytes, which is the library's
// [E][N][K/256] device layout, so the payload is copied byte for byte — read
// from the file in 64 MiB pieces into two pinned buffers that alternate, each
// piece copied to the device on the context's stream while the next is read.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <unordered_map>

#include "har_internal.cuh"

namespace {

constexpr uint64_t MAX_COUNT = 10000000ull;
constexpr uint64_t MAX_ARRAY = 1000000ull;
constexpr uint64_t MAX_STRING = 1ull << 30;
constexpr size_t STAGE_BYTES = 64ull << 20;

// GGML block geometry (tensor_block_size / tensor_type_size,
// har/crates/har-model/src/lib.rs:605-640)
uint64_t type_block(uint32_t t) {
  switch (t) {
    case 0: case 1: case 30: return 1;
    case 2: case 3: case 6: case 7: case 8: return 32;
    case 10: case 11: case 12: case 13: case 14: case 15: case 36: case 39: return 256;
    default: return 0;
  }
}
uint64_t type_size(uint32_t t) {
  switch (t) {
    case 0: return 4;
    case 1: case 30: return 2;
    case 2: return 18;
    case 3: return 20;
    case 6: return 22;
    case 7: return 24;
    case 8: return 34;
    case 10: return 84;
    case 11: return 110;
    case 12: return 144;
    case 13: return 176;
    case 14: return 210;
    case 15: return 292;
    case 36: return 144;
    case 39: return 256;
    default: return 0;
  }
}
uint64_t payload_for(uint32_t t, uint64_t elements) {
  const uint64_t b = type_block(t), s = type_size(t);
  if (!b || !s) return 0;
  return (elements + b - 1) / b * s;
}

struct Meta {
  enum Kind { UINT, INT, FLOAT, BOOL, STRING, ARRAY } kind = UINT;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  uint64_t count = 0;  // arrays
};

// Sequential reader over a file descriptor with bounds checks; every failure
// leaves a message and makes the parse return an error (never throws).
struct Cursor {
  int fd;
  uint64_t size, pos = 0;
  std::string err;
  std::vector<uint8_t> buf;
  uint64_t buf_pos = 0;  // file offset of buf[0]

  bool read(void *dst, uint64_t n) {
    if (!err.empty()) return false;
    if (n > size || pos > size - n) {
      err = "unexpected end of file at byte " + std::to_string(pos);
      return false;
    }
    uint8_t *d = static_cast<uint8_t *>(dst);
    while (n) {
      if (pos >= buf_pos && pos < buf_pos + buf.size()) {
        const uint64_t take = std::min<uint64_t>(n, buf_pos + buf.size() - pos);
        memcpy(d, buf.data() + (pos - buf_pos), take);
        d += take;
        pos += take;
        n -= take;
        continue;
      }
      buf.resize(1 << 20);
      const ssize_t got = pread(fd, buf.data(), buf.size(), (off_t)pos);
      if (got <= 0) {
        err = "read failed at byte " + std::to_string(pos);
        buf.clear();
        return false;
      }
      buf.resize((size_t)got);
      buf_pos = pos;
    }
    return true;
  }
  bool skip(uint64_t n) {
    if (!err.empty()) return false;
    if (n > size || pos > size - n) {
      err = "unexpected end of file at byte " + std::to_string(pos);
      return false;
    }
    pos += n;
    return true;
  }
  template <class T>
  bool get(T &v) { return read(&v, sizeof(T)); }
  bool str(std::string &s) {
    uint64_t n = 0;
    if (!get(n)) return false;
    if (n > MAX_STRING) {
      err = "string of " + std::to_string(n) + " bytes exceeds the bound";
      return false;
    }
    s.resize((size_t)n);
    return read(&s[0], n);
  }
};

bool read_value(Cursor &c, uint32_t type, Meta *m, int depth) {
  uint8_t b8;
  uint16_t b16;
  uint32_t b32;
  uint64_t b64;
  Meta tmp;
  Meta &v = m ? *m : tmp;
  switch (type) {
    case 0: if (!c.get(b8)) return false; v.kind = Meta::UINT; v.u = b8; return true;
    case 1: if (!c.get(b8)) return false; v.kind = Meta::INT; v.i = (int8_t)b8; return true;
    case 2: if (!c.get(b16)) return false; v.kind = Meta::UINT; v.u = b16; return true;
    case 3: if (!c.get(b16)) return false; v.kind = Meta::INT; v.i = (int16_t)b16; return true;
    case 4: if (!c.get(b32)) return false; v.kind = Meta::UINT; v.u = b32; return true;
    case 5: if (!c.get(b32)) return false; v.kind = Meta::INT; v.i = (int32_t)b32; return true;
    case 6: {
      float f;
      if (!c.get(f)) return false;
      v.kind = Meta::FLOAT;
      v.f = f;
      return true;
    }
    case 7: if (!c.get(b8)) return false; v.kind = Meta::BOOL; v.u = b8 != 0; return true;
    case 8: v.kind = Meta::STRING; return c.str(v.s);
    case 9: {
      uint32_t et = 0;
      uint64_t n = 0;
      if (!c.get(et) || !c.get(n)) return false;
      if (n > MAX_ARRAY) {
        c.err = "metadata array of " + std::to_string(n) + " elements exceeds the bound";
        return false;
      }
      if (depth > 8) {
        c.err = "metadata arrays nested too deeply";
        return false;
      }
      v.kind = Meta::ARRAY;
      v.count = n;
      static const uint64_t fixed[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
      if (et <= 12 && fixed[et]) return c.skip(fixed[et] * n);
      for (uint64_t k = 0; k < n; ++k)
        if (!read_value(c, et, nullptr, depth + 1)) return false;
      return true;
    }
    case 10: if (!c.get(b64)) return false; v.kind = Meta::UINT; v.u = b64; return true;
    case 11: if (!c.get(b64)) return false; v.kind = Meta::INT; v.i = (int64_t)b64; return true;
    case 12: {
      double f;
      if (!c.get(f)) return false;
      v.kind = Meta::FLOAT;
      v.f = f;
      return true;
    }
    default:
      c.err = "unsupported GGUF metadata type " + std::to_string(type);
      return false;
  }
}

// A metadata value read as a number the way HAR's metadata_number does
// (har/crates/har-model/src/lib.rs:541-543: the value's text parsed as u64):
// unsigned and non-negative signed integers, integral non-negative floats
// (whose text has no decimal point) and strings of decimal digits.
bool meta_number(const Meta &m, uint64_t *v) {
  switch (m.kind) {
    case Meta::UINT: *v = m.u; return true;
    case Meta::INT: if (m.i < 0) return false; *v = (uint64_t)m.i; return true;
    case Meta::FLOAT:
      if (!(m.f >= 0.0) || m.f >= 18446744073709551616.0 || m.f != (double)(uint64_t)m.f)
        return false;
      *v = (uint64_t)m.f;
      return true;
    case Meta::STRING: {
      size_t i = (!m.s.empty() && m.s[0] == '+') ? 1 : 0;
      if (i == m.s.size()) return false;
      uint64_t x = 0;
      for (; i < m.s.size(); ++i) {
        const char ch = m.s[i];
        if (ch < '0' || ch > '9') return false;
        if (x > (UINT64_MAX - (uint64_t)(ch - '0')) / 10) return false;
        x = x * 10 + (uint64_t)(ch - '0');
      }
      *v = x;
      return true;
    }
    default: return false;
  }
}

void copy_msg(const std::string &m, char *buf, size_t len) {
  if (!buf || !len) return;
  const size_t n = std::min(len - 1, m.size());
  memcpy(buf, m.data(), n);
  buf[n] = 0;
}

}  // namespace

struct har_cuda_gguf {
  int fd = -1;
  uint64_t file_bytes = 0;
  uint32_t version = 0;
  uint64_t tensor_count = 0, metadata_count = 0, alignment = 32, data_offset = 0;
  std::map<std::string, Meta> meta;
  struct Tensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;   // relative to the data section
    uint64_t payload = 0;  // bytes
  };
  std::vector<Tensor> tensors;
  std::unordered_map<std::string, size_t> by_name;
  mutable std::string last_error;  // set by const queries too
  void *stage[2] = {nullptr, nullptr};  // pinned, portable (any device)
};

namespace {

int32_t gerr(const har_cuda_gguf *g, int32_t code, const std::string &m) {
  g->last_error = m;
  return code;
}

const har_cuda_gguf::Tensor *find_tensor(const har_cuda_gguf *g, const char *name) {
  if (!g || !name) return nullptr;
  auto it = g->by_name.find(name);
  return it == g->by_name.end() ? nullptr : &g->tensors[it->second];
}

// Copy `bytes` of the file at `file_off` to device memory `dst` through the
// two pinned stages, on the context's stream; waits for the last copy.
int32_t stream_to_device(har_cuda_ctx *ctx, har_cuda_gguf *g, uint64_t file_off, uint64_t bytes,
                         uint8_t *dst) {
  for (int i = 0; i < 2; ++i) {
    if (!g->stage[i] &&
        cudaHostAlloc(&g->stage[i], STAGE_BYTES, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      g->stage[i] = nullptr;
      return har::set_error(ctx, HAR_CUDA_ERR_OOM, "gguf: pinned staging allocation failed");
    }
  }
  cudaEvent_t done[2] = {nullptr, nullptr};
  for (int i = 0; i < 2; ++i)
    if (cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      if (done[0]) cudaEventDestroy(done[0]);
      return har::set_error(ctx, HAR_CUDA_ERR_CUDA, "gguf: cudaEventCreate failed");
    }
  bool used[2] = {false, false};
  int32_t st = HAR_CUDA_OK;
  uint64_t off = 0;
  for (int k = 0; off < bytes; k ^= 1) {
    const uint64_t n = std::min<uint64_t>(STAGE_BYTES, bytes - off);
    if (used[k] && cudaEventSynchronize(done[k]) != cudaSuccess) {
      st = har::set_error(ctx, HAR_CUDA_ERR_CUDA, "gguf: staging copy failed");
      break;
    }
    uint8_t *h = static_cast<uint8_t *>(g->stage[k]);
    uint64_t got = 0;
    while (got < n) {
      const ssize_t r = pread(g->fd, h + got, (size_t)(n - got), (off_t)(file_off + off + got));
      if (r <= 0) break;
      got += (uint64_t)r;
    }
    if (got != n) {
      st = har::set_error(ctx, HAR_CUDA_ERR_ARG,
                          "gguf: short read at file byte " + std::to_string(file_off + off + got));
      break;
    }
    if (cudaMemcpyAsync(dst + off, h, n, cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess ||
        cudaEventRecord(done[k], ctx->stream) != cudaSuccess) {
      cudaGetLastError();
      st = har::set_error(ctx, HAR_CUDA_ERR_CUDA, "gguf: host-to-device copy failed");
      break;
    }
    used[k] = true;
    off += n;
  }
  // both stages must be idle before they are reused or freed
  for (int i = 0; i < 2; ++i) {
    if (used[i] && cudaEventSynchronize(done[i]) != cudaSuccess && st == HAR_CUDA_OK)
      st = har::set_error(ctx, HAR_CUDA_ERR_CUDA, "gguf: staging copy failed");
    cudaEventDestroy(done[i]);
  }
  return st;
}

}  // namespace

namespace har {

// Weight tensor of a supported block type as [E][N][K/256]: GGML dims [K, N]
// (E = 1) or [K, N, E].
int32_t gguf_load_weights(har_cuda_ctx *ctx, har_cuda_gguf *g, const char *name,
                          har_cuda_weights **out) {
  const har_cuda_gguf::Tensor *t = find_tensor(g, name);
  if (!t) return set_error(ctx, HAR_CUDA_ERR_ARG, std::string("gguf: no tensor ") + (name ? name : "(null)"));
  if (!ggml_block_bytes((int)t->type))
    return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED,
                     "gguf: tensor " + t->name + " has GGML type " + std::to_string(t->type) +
                         " (loadable: 11 Q3_K, 12 Q4_K, 14 Q6_K)");
  if (t->dims.size() != 2 && t->dims.size() != 3)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "gguf: tensor " + t->name + " is not 2-D or 3-D");
  const int64_t K = (int64_t)t->dims[0], N = (int64_t)t->dims[1];
  const int64_t E = t->dims.size() == 3 ? (int64_t)t->dims[2] : 1;
  if (K <= 0 || N <= 0 || E <= 0 || K % QK != 0)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                     "gguf: tensor " + t->name + " has K not a positive multiple of 256");
  const uint64_t bytes = (uint64_t)E * (uint64_t)N * (uint64_t)(K / QK) * (uint64_t)ggml_block_bytes((int)t->type);
  if (t->payload != bytes)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "gguf: tensor " + t->name + " payload mismatch");
  const uint64_t at = g->data_offset + t->offset;
  if (at > g->file_bytes || bytes > g->file_bytes - at)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "gguf: tensor " + t->name + " runs past the file end");
  if (cudaSetDevice(ctx->device) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "gguf: cudaSetDevice failed");
  void *d = nullptr;
  if (cudaMalloc(&d, bytes) != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, HAR_CUDA_ERR_OOM, "gguf: cudaMalloc failed for " + t->name);
  }
  int32_t st = stream_to_device(ctx, g, at, bytes, static_cast<uint8_t *>(d));
  if (st != HAR_CUDA_OK) {
    cudaFree(d);
    return st;
  }
  har_cuda_weights *w = new har_cuda_weights();
  w->dev = static_cast<const uint8_t *>(d);
  w->owned = true;
  w->type = (int32_t)t->type;
  w->E = E;
  w->N = N;
  w->K = K;
  w->row_bytes = K / QK * ggml_block_bytes((int)t->type);
  w->expert_bytes = w->row_bytes * N;
  w->device = ctx->device;
  *out = w;
  return HAR_CUDA_OK;
}

// An F32 tensor of exactly `count` elements into device memory `dst`.
int32_t gguf_load_f32(har_cuda_ctx *ctx, har_cuda_gguf *g, const char *name, float *dst,
                      int64_t count) {
  const har_cuda_gguf::Tensor *t = find_tensor(g, name);
  if (!t) return set_error(ctx, HAR_CUDA_ERR_ARG, std::string("gguf: no tensor ") + (name ? name : "(null)"));
  if (t->type != GGML_F32)
    return set_error(ctx, HAR_CUDA_ERR_UNSUPPORTED, "gguf: tensor " + t->name + " is not F32");
  uint64_t el = 1;
  for (uint64_t d : t->dims) el *= d;
  if (count < 0 || el != (uint64_t)count || t->payload != el * 4)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY,
                     "gguf: tensor " + t->name + " has " + std::to_string(el) + " elements, expected " +
                         std::to_string(count));
  const uint64_t at = g->data_offset + t->offset;
  if (at > g->file_bytes || t->payload > g->file_bytes - at)
    return set_error(ctx, HAR_CUDA_ERR_GEOMETRY, "gguf: tensor " + t->name + " runs past the file end");
  if (cudaSetDevice(ctx->device) != cudaSuccess)
    return set_error(ctx, HAR_CUDA_ERR_CUDA, "gguf: cudaSetDevice failed");
  return stream_to_device(ctx, g, at, t->payload, reinterpret_cast<uint8_t *>(dst));
}

}  // namespace har

using namespace har;

extern "C" {

int32_t har_cuda_gguf_open(const char *path, char *err, size_t err_len, har_cuda_gguf **out) {
  if (!path || !out) {
    copy_msg("gguf_open: null argument", err, err_len);
    return HAR_CUDA_ERR_ARG;
  }
  *out = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) {
    copy_msg(std::string("gguf_open: cannot open ") + path, err, err_len);
    return HAR_CUDA_ERR_ARG;
  }
  struct stat sb;
  if (fstat(fd, &sb) != 0) {
    close(fd);
    copy_msg("gguf_open: fstat failed", err, err_len);
    return HAR_CUDA_ERR_ARG;
  }
  har_cuda_gguf *g = new har_cuda_gguf();
  g->fd = fd;
  g->file_bytes = (uint64_t)sb.st_size;
  Cursor c{fd, g->file_bytes};
  auto fail = [&](int32_t code, const std::string &m) {
    copy_msg("gguf_open: " + m, err, err_len);
    har_cuda_gguf_close(g);
    return code;
  };
  char magic[4];
  if (!c.read(magic, 4)) return fail(HAR_CUDA_ERR_GEOMETRY, c.err);
  if (memcmp(magic, "GGUF", 4) != 0) return fail(HAR_CUDA_ERR_GEOMETRY, "bad magic");
  if (!c.get(g->version) || !c.get(g->tensor_count) || !c.get(g->metadata_count))
    return fail(HAR_CUDA_ERR_GEOMETRY, c.err);
  if (g->version < 1 || g->version > 3)
    return fail(HAR_CUDA_ERR_UNSUPPORTED, "GGUF version " + std::to_string(g->version));
  if (g->tensor_count > MAX_COUNT || g->metadata_count > MAX_COUNT)
    return fail(HAR_CUDA_ERR_GEOMETRY, "count exceeds safety bound");
  for (uint64_t i = 0; i < g->metadata_count; ++i) {
    std::string key;
    uint32_t vt = 0;
    Meta m;
    if (!c.str(key) || !c.get(vt) || !read_value(c, vt, &m, 0))
      return fail(HAR_CUDA_ERR_GEOMETRY, c.err);
    g->meta[key] = m;
  }
  auto al = g->meta.find("general.alignment");
  uint64_t alv = 32;
  if (al != g->meta.end() && !meta_number(al->second, &alv)) alv = 32;
  g->alignment = std::max<uint64_t>(alv, 1);
  g->tensors.reserve((size_t)g->tensor_count);
  for (uint64_t i = 0; i < g->tensor_count; ++i) {
    har_cuda_gguf::Tensor t;
    uint32_t rank = 0;
    if (!c.str(t.name) || !c.get(rank)) return fail(HAR_CUDA_ERR_GEOMETRY, c.err);
    if (rank > 16) return fail(HAR_CUDA_ERR_GEOMETRY, "tensor rank " + std::to_string(rank));
    t.dims.resize(rank);
    for (uint32_t r = 0; r < rank; ++r)
      if (!c.get(t.dims[r])) return fail(HAR_CUDA_ERR_GEOMETRY, c.err);
    if (!c.get(t.type) || !c.get(t.offset)) return fail(HAR_CUDA_ERR_GEOMETRY, c.err);
    g->tensors.push_back(std::move(t));
  }
  const uint64_t pos = c.pos;
  g->data_offset = (pos + g->alignment - 1) / g->alignment * g->alignment;
  if (g->data_offset > g->file_bytes)
    return fail(HAR_CUDA_ERR_GEOMETRY, "data offset " + std::to_string(g->data_offset) +
                                           " is past the end of the file");
  // payload sizes: from the type tables, else the span to the next tensor
  std::vector<std::pair<uint64_t, size_t>> order;
  for (size_t i = 0; i < g->tensors.size(); ++i) order.push_back({g->tensors[i].offset, i});
  std::sort(order.begin(), order.end());
  std::vector<uint64_t> span(g->tensors.size(), 0);
  for (size_t j = 0; j < order.size(); ++j) {
    const size_t i = order[j].second;
    if (j + 1 < order.size())
      span[i] = order[j + 1].first >= order[j].first ? order[j + 1].first - order[j].first : 0;
    else {
      const uint64_t at = g->data_offset + g->tensors[i].offset;
      span[i] = g->file_bytes > at ? g->file_bytes - at : 0;
    }
  }
  for (size_t i = 0; i < g->tensors.size(); ++i) {
    auto &t = g->tensors[i];
    uint64_t el = 1;
    for (uint64_t d : t.dims)
      if (__builtin_mul_overflow(el, d, &el) || el > (1ull << 62))
        return fail(HAR_CUDA_ERR_GEOMETRY, "tensor " + t.name + " has more than 2^62 elements");
    const uint64_t known = payload_for(t.type, el);
    t.payload = known ? known : span[i];
    g->by_name.emplace(t.name, i);
  }
  *out = g;
  copy_msg("", err, err_len);
  return HAR_CUDA_OK;
}

int32_t har_cuda_gguf_close(har_cuda_gguf *g) {
  if (!g) return HAR_CUDA_ERR_ARG;
  for (void *s : g->stage)
    if (s) cudaFreeHost(s);
  if (g->fd >= 0) close(g->fd);
  delete g;
  return HAR_CUDA_OK;
}

int32_t har_cuda_gguf_last_error(const har_cuda_gguf *g, char *buf, size_t len) {
  if (!g || !buf || !len) return HAR_CUDA_ERR_ARG;
  copy_msg(g->last_error, buf, len);
  return HAR_CUDA_OK;
}

int32_t har_cuda_gguf_header(const har_cuda_gguf *g, uint32_t *version, uint64_t *tensor_count,
                             uint64_t *metadata_count, uint64_t *alignment,
                             uint64_t *data_offset) {
  if (!g) return HAR_CUDA_ERR_ARG;
  if (version) *version = g->version;
  if (tensor_count) *tensor_count = g->tensor_count;
  if (metadata_count) *metadata_count = g->metadata_count;
  if (alignment) *alignment = g->alignment;
  if (data_offset) *data_offset = g->data_offset;
  return HAR_CUDA_OK;
}

int32_t har_cuda_gguf_tensor_info(const har_cuda_gguf *g, int64_t index, char *name,
                                  size_t name_len, uint32_t *ggml_type, uint32_t *rank,
                                  uint64_t *dims, uint64_t *file_offset, uint64_t *payload_bytes) {
  if (!g) return HAR_CUDA_ERR_ARG;
  if (index < 0 || (uint64_t)index >= g->tensors.size())
    return gerr(g, HAR_CUDA_ERR_ARG,
                "tensor index " + std::to_string(index) + " out of range");
  const auto &t = g->tensors[(size_t)index];
  copy_msg(t.name, name, name_len);
  if (ggml_type) *ggml_type = t.type;
  if (rank) *rank = (uint32_t)t.dims.size();
  if (dims)
    for (size_t r = 0; r < t.dims.size(); ++r) dims[r] = t.dims[r];
  if (file_offset) *file_offset = g->data_offset + t.offset;
  if (payload_bytes) *payload_bytes = t.payload;
  return HAR_CUDA_OK;
}

int64_t har_cuda_gguf_find(const har_cuda_gguf *g, const char *name) {
  if (!g || !name) return -1;
  auto it = g->by_name.find(name);
  return it == g->by_name.end() ? -1 : (int64_t)it->second;
}

int32_t har_cuda_gguf_meta_u64(const har_cuda_gguf *g, const char *key, uint64_t *value) {
  if (!g || !key || !value) return HAR_CUDA_ERR_ARG;
  auto it = g->meta.find(key);
  if (it == g->meta.end())
    return gerr(g, HAR_CUDA_ERR_ARG, std::string("no metadata key ") + key);
  if (meta_number(it->second, value)) return HAR_CUDA_OK;
  return gerr(g, HAR_CUDA_ERR_ARG,
              std::string("metadata ") + key + " is not a non-negative integer");
}

int32_t har_cuda_gguf_meta_string(const har_cuda_gguf *g, const char *key, char *buf,
                                  size_t len) {
  if (!g || !key || !buf || !len) return HAR_CUDA_ERR_ARG;
  auto it = g->meta.find(key);
  if (it == g->meta.end() || it->second.kind != Meta::STRING)
    return gerr(g, HAR_CUDA_ERR_ARG,
                std::string("no string metadata key ") + key);
  copy_msg(it->second.s, buf, len);
  return HAR_CUDA_OK;
}

int32_t har_cuda_weights_from_gguf(har_cuda_ctx *ctx, har_cuda_gguf *g, const char *name,
                                   har_cuda_weights **out) {
  if (!ctx || !out) return HAR_CUDA_ERR_ARG;
  *out = nullptr;
  if (!g) return set_error(ctx, HAR_CUDA_ERR_ARG, "weights_from_gguf: gguf is null");
  return gguf_load_weights(ctx, g, name, out);
}

int32_t har_cuda_gguf_read_f32(har_cuda_ctx *ctx, har_cuda_gguf *g, const char *name,
                               float *dst_dev, int64_t count) {
  if (!ctx) return HAR_CUDA_ERR_ARG;
  if (!g || !dst_dev) return set_error(ctx, HAR_CUDA_ERR_ARG, "gguf_read_f32: null argument");
  return gguf_load_f32(ctx, g, name, dst_dev, count);
}

int32_t har_cuda_moe_layer_from_gguf(har_cuda_ctx *ctx, har_cuda_gguf *g, int32_t layer,
                                     har_cuda_moe_layer **out) {
  if (!ctx || !out) return HAR_CUDA_ERR_ARG;
  *out = nullptr;
  if (!g) return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_layer_from_gguf: gguf is null");
  if (layer < 0) return set_error(ctx, HAR_CUDA_ERR_ARG, "moe_layer_from_gguf: negative layer");
  const std::string p = "blk." + std::to_string(layer) + ".";
  std::vector<har_cuda_weights *> w(6, nullptr);
  static const char *names[6] = {"ffn_gate_exps.weight",  "ffn_up_exps.weight",
                                 "ffn_down_exps.weight",  "ffn_gate_shexp.weight",
                                 "ffn_up_shexp.weight",   "ffn_down_shexp.weight"};
  auto cleanup = [&](void *buf) {
    for (auto *x : w)
      if (x) har_cuda_weights_free(x);
    if (buf) cudaFree(buf);
  };
  const bool shared = find_tensor(g, (p + names[3]).c_str()) != nullptr;
  for (int i = 0; i < (shared ? 6 : 3); ++i) {
    const int32_t st = gguf_load_weights(ctx, g, (p + names[i]).c_str(), &w[i]);
    if (st != HAR_CUDA_OK) {
      cleanup(nullptr);
      return st;
    }
  }
  const int64_t E = w[0]->E, H = w[0]->K;
  // f32 rows the layer owns: the router [E][H] (ffn_gate_inp: GGML dims [H, E])
  // and the shared-expert gate row [H] (ffn_gate_inp_shexp)
  const bool has_router = find_tensor(g, (p + "ffn_gate_inp.weight").c_str()) != nullptr;
  const bool has_sgate = shared && find_tensor(g, (p + "ffn_gate_inp_shexp.weight").c_str());
  void *buf = nullptr;
  const size_t fl = (size_t)((has_router ? E * H : 0) + (has_sgate ? H : 0));
  if (fl) {
    if (cudaMalloc(&buf, fl * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      cleanup(nullptr);
      return set_error(ctx, HAR_CUDA_ERR_OOM, "moe_layer_from_gguf: cudaMalloc failed");
    }
  }
  float *router = has_router ? static_cast<float *>(buf) : nullptr;
  float *sgate = has_sgate ? static_cast<float *>(buf) + (has_router ? E * H : 0) : nullptr;
  int32_t st = HAR_CUDA_OK;
  if (router) st = gguf_load_f32(ctx, g, (p + "ffn_gate_inp.weight").c_str(), router, E * H);
  if (st == HAR_CUDA_OK && sgate)
    st = gguf_load_f32(ctx, g, (p + "ffn_gate_inp_shexp.weight").c_str(), sgate, H);
  har_cuda_moe_layer *l = nullptr;
  if (st == HAR_CUDA_OK)
    st = har_cuda_moe_layer_create(ctx, w[0], w[1], w[2], w[3], w[4], w[5], sgate, &l);
  if (st != HAR_CUDA_OK) {
    cleanup(buf);
    return st;
  }
  l->owned = w;
  l->owned_dev = buf;
  l->router = router;
  *out = l;
  return HAR_CUDA_OK;
}

}  // extern "C"
