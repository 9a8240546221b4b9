// loader.cu — safetensors checkpoint reader and the decoder's W8 checkpoint
// loader (host code).
//
// Reference: crates/rxla-safetensors/src/lib.rs
//   SafeTensors::new          :147-177  8-byte little-endian header length
//                                       (at most 100 MB), JSON header, payload
//                                       length must equal the file's rest
//   names / info / metadata   :179-208  tensor table, "__metadata__" strings,
//                                       require_metadata (exact string match)
//   read_u8 / read_f32 / ...  :299-540  exact payload bytes of one tensor
//   upload_u8                 :664-700  U8 quantized storage uploaded as is
// The header validation restates the upstream `safetensors` crate 0.8.0 (a
// Cargo dependency of rxla-safetensors, not vendored): tensors sorted by
// offset tile the payload without gaps or overlaps, and each tensor's byte
// range equals its element count times its dtype size.
//
// The W8 checkpoint format is rxla's "rxla-qwen3.5-w8-v1"
// (benchmarks/quantize_qwen3_5_w8.py:17-56): every 2-D weight is U8
// (q + 128, symmetric per group) with an F32 "<name>.scale" [rows, cols / G],
// other tensors F32; metadata "format" and "group_size".
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "internal.cuh"

namespace rxla {
namespace st {

struct Tensor {
  std::string name;
  int32_t dtype;  // RXLA_B200_* or -1 (a dtype the boundary has no code for)
  int32_t elem;   // bytes per element
  std::vector<int64_t> shape;
  int64_t begin, end;  // payload byte range
};

// Minimal JSON reader for the safetensors header: objects, arrays, strings
// (with escapes), non-negative integers.  Anything else is an error.
struct Json {
  const char* p;
  const char* e;
  std::string err;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool lit(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return fail_("expected a string");
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= e) return fail_("bad escape");
        const char x = *p++;
        switch (x) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (e - p < 4) return fail_("bad \\u escape");
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              const char h = *p++;
              v <<= 4;
              if (h >= '0' && h <= '9') v |= (unsigned)(h - '0');
              else if (h >= 'a' && h <= 'f') v |= (unsigned)(h - 'a' + 10);
              else if (h >= 'A' && h <= 'F') v |= (unsigned)(h - 'A' + 10);
              else return fail_("bad \\u escape");
            }
            // UTF-8 of the code unit (surrogate pairs are kept as two units)
            if (v < 0x80) {
              out += (char)v;
            } else if (v < 0x800) {
              out += (char)(0xc0 | (v >> 6));
              out += (char)(0x80 | (v & 0x3f));
            } else {
              out += (char)(0xe0 | (v >> 12));
              out += (char)(0x80 | ((v >> 6) & 0x3f));
              out += (char)(0x80 | (v & 0x3f));
            }
            break;
          }
          default: return fail_("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (p >= e) return fail_("unterminated string");
    ++p;
    return true;
  }
  bool uint(int64_t& v) {
    ws();
    if (p >= e || *p < '0' || *p > '9') return fail_("expected a non-negative integer");
    v = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      if (v > (INT64_MAX - 9) / 10) return fail_("integer overflow");
      v = v * 10 + (*p++ - '0');
    }
    return true;
  }
  bool uints(std::vector<int64_t>& out) {
    out.clear();
    if (!lit('[')) return fail_("expected an array");
    if (lit(']')) return true;
    do {
      int64_t v;
      if (!uint(v)) return false;
      out.push_back(v);
    } while (lit(','));
    if (!lit(']')) return fail_("expected ]");
    return true;
  }
  bool fail_(const char* m) {
    if (err.empty()) err = m;
    return false;
  }
};

static bool dtype_of(const std::string& s, int32_t& code, int32_t& elem) {
  static const struct {
    const char* name;
    int32_t code, elem;
  } kTypes[] = {{"F32", RXLA_B200_F32, 4}, {"BF16", RXLA_B200_BF16, 2}, {"U8", RXLA_B200_U8, 1},
                {"I32", RXLA_B200_I32, 4}, {"F16", RXLA_B200_F16, 2},   {"F64", -1, 8},
                {"I64", -1, 8},            {"U64", -1, 8},              {"U32", -1, 4},
                {"I16", -1, 2},            {"U16", -1, 2},              {"I8", -1, 1},
                {"BOOL", -1, 1},           {"F8_E4M3", -1, 1},          {"F8_E5M2", -1, 1}};
  for (auto& t : kTypes)
    if (s == t.name) {
      code = t.code;
      elem = t.elem;
      return true;
    }
  return false;
}

}  // namespace st
}  // namespace rxla

struct rxla_b200_safetensors {
  int fd = -1;
  int64_t data_start = 0;
  std::vector<rxla::st::Tensor> tensors;  // header order
  std::map<std::string, int32_t> index;
  std::map<std::string, std::string> metadata;
};

using namespace rxla;

extern "C" int32_t rxla_b200_safetensors_close(rxla_b200_safetensors* f) {
  if (!f) return RXLA_B200_OK;
  if (f->fd >= 0) close(f->fd);
  delete f;
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_safetensors_open(const char* path, rxla_b200_safetensors** out) {
  RXLA_REQUIRE(path && out, "safetensors_open: null argument");
  *out = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(RXLA_B200_NOT_FOUND, std::string("safetensors_open: cannot open ") + path);
  auto* f = new rxla_b200_safetensors();
  f->fd = fd;
  auto bad = [&](const std::string& m) {
    rxla_b200_safetensors_close(f);
    return fail(RXLA_B200_INVALID_ARGUMENT, "safetensors_open: " + m);
  };
  struct stat sb;
  if (fstat(fd, &sb) != 0) return bad("cannot stat the file");
  const int64_t file_len = sb.st_size;
  uint8_t prefix[8];
  if (file_len < 8 || pread(fd, prefix, 8, 0) != 8) return bad("truncated header");
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | prefix[i];
  if (hlen > 100000000ull) return bad("header exceeds 100 MB limit");
  if ((int64_t)hlen + 8 > file_len) return bad("truncated header");
  std::string header((size_t)hlen, '\0');
  if (hlen && pread(fd, &header[0], hlen, 8) != (ssize_t)hlen) return bad("truncated header");
  f->data_start = 8 + (int64_t)hlen;

  st::Json j{header.data(), header.data() + header.size(), {}};
  if (!j.lit('{')) return bad("header is not a JSON object");
  if (!j.lit('}')) {
    do {
      std::string key;
      if (!j.str(key) || !j.lit(':')) return bad("header: " + (j.err.empty() ? "expected :" : j.err));
      if (key == "__metadata__") {
        if (!j.lit('{')) return bad("__metadata__ must be an object of strings");
        if (!j.lit('}')) {
          do {
            std::string k, v;
            if (!j.str(k) || !j.lit(':') || !j.str(v))
              return bad("__metadata__ must be an object of strings");
            f->metadata[k] = v;
          } while (j.lit(','));
          if (!j.lit('}')) return bad("__metadata__: expected }");
        }
        continue;
      }
      st::Tensor t{key, 0, 0, {}, -1, -1};
      bool have_dtype = false, have_shape = false, have_off = false;
      if (!j.lit('{')) return bad("tensor " + key + ": expected an object");
      if (!j.lit('}')) {
        do {
          std::string field;
          if (!j.str(field) || !j.lit(':')) return bad("tensor " + key + ": malformed entry");
          if (field == "dtype") {
            std::string dt;
            if (!j.str(dt)) return bad("tensor " + key + ": dtype must be a string");
            if (!st::dtype_of(dt, t.dtype, t.elem)) return bad("tensor " + key + ": unknown dtype " + dt);
            have_dtype = true;
          } else if (field == "shape") {
            if (!j.uints(t.shape)) return bad("tensor " + key + ": bad shape");
            have_shape = true;
          } else if (field == "data_offsets") {
            std::vector<int64_t> o;
            if (!j.uints(o) || o.size() != 2) return bad("tensor " + key + ": bad data_offsets");
            t.begin = o[0];
            t.end = o[1];
            have_off = true;
          } else {
            return bad("tensor " + key + ": unknown field " + field);
          }
        } while (j.lit(','));
        if (!j.lit('}')) return bad("tensor " + key + ": expected }");
      }
      if (!have_dtype || !have_shape || !have_off) return bad("tensor " + key + ": incomplete entry");
      if (f->index.count(key)) return bad("duplicate tensor " + key);
      f->index[key] = (int32_t)f->tensors.size();
      f->tensors.push_back(std::move(t));
    } while (j.lit(','));
    if (!j.lit('}')) return bad("header: expected }");
  }
  j.ws();
  if (j.p != j.e) return bad("trailing bytes after the header object");

  // offsets tile the payload: sorted by start, each start = previous end,
  // each length = elements * dtype size, the last end = payload length
  std::vector<const st::Tensor*> order;
  for (auto& t : f->tensors) order.push_back(&t);
  std::sort(order.begin(), order.end(), [](const st::Tensor* a, const st::Tensor* b) {
    return a->begin != b->begin ? a->begin < b->begin : a->end < b->end;
  });
  int64_t pos = 0;
  for (const st::Tensor* t : order) {
    int64_t n = 1;
    for (int64_t dim : t->shape) {
      if (dim != 0 && n > INT64_MAX / dim) return bad("tensor " + t->name + ": shape overflow");
      n *= dim;
    }
    if (n > INT64_MAX / t->elem) return bad("tensor " + t->name + ": shape overflow");
    if (t->begin != pos || t->end < t->begin)
      return bad("tensor " + t->name + ": data_offsets leave a gap or overlap");
    if (t->end - t->begin != n * t->elem)
      return bad("tensor " + t->name + ": byte range does not match shape and dtype");
    pos = t->end;
  }
  if (f->data_start + pos != file_len) return bad("payload length does not match metadata");
  *out = f;
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_safetensors_count(const rxla_b200_safetensors* f, int32_t* count) {
  RXLA_REQUIRE(f && count, "safetensors_count: null argument");
  *count = (int32_t)f->tensors.size();
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_safetensors_info(const rxla_b200_safetensors* f, int32_t index,
                                              const char** name, int32_t* dtype, int32_t* ndim,
                                              int64_t* shape, int64_t* bytes) {
  RXLA_REQUIRE(f, "safetensors_info: null reader");
  RXLA_REQUIRE(index >= 0 && index < (int32_t)f->tensors.size(),
               "safetensors_info: index out of range");
  const st::Tensor& t = f->tensors[(size_t)index];
  RXLA_REQUIRE(t.shape.size() <= 8, "safetensors_info: more than 8 dimensions");
  if (name) *name = t.name.c_str();
  if (dtype) *dtype = t.dtype;
  if (ndim) *ndim = (int32_t)t.shape.size();
  if (shape)
    for (size_t i = 0; i < t.shape.size(); ++i) shape[i] = t.shape[i];
  if (bytes) *bytes = t.end - t.begin;
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_safetensors_find(const rxla_b200_safetensors* f, const char* name,
                                              int32_t* index) {
  RXLA_REQUIRE(f && name && index, "safetensors_find: null argument");
  auto it = f->index.find(name);
  if (it == f->index.end())
    return fail(RXLA_B200_NOT_FOUND, std::string("safetensors: missing tensor ") + name);
  *index = it->second;
  return RXLA_B200_OK;
}

extern "C" int32_t rxla_b200_safetensors_metadata(const rxla_b200_safetensors* f, const char* key,
                                                  const char** value) {
  RXLA_REQUIRE(f && key && value, "safetensors_metadata: null argument");
  auto it = f->metadata.find(key);
  if (it == f->metadata.end())
    return fail(RXLA_B200_NOT_FOUND, std::string("safetensors: no metadata ") + key);
  *value = it->second.c_str();
  return RXLA_B200_OK;
}

namespace rxla {
namespace st {

// A tensor seen as [rows, cols]: 0-D and 1-D tensors are one row, higher
// ranks keep their first dimension as rows.
static void as_matrix(const Tensor& t, int64_t& rows, int64_t& cols) {
  rows = t.shape.size() >= 2 ? t.shape[0] : 1;
  cols = 1;
  for (size_t i = t.shape.size() >= 2 ? 1 : 0; i < t.shape.size(); ++i) cols *= t.shape[i];
}

static int32_t read_block(const rxla_b200_safetensors* f, const Tensor& t, int64_t row0,
                          int64_t rows, int64_t col0, int64_t cols, uint8_t* dst) {
  int64_t R, C;
  as_matrix(t, R, C);
  // overflow-safe: rows <= R and row0 <= R - rows (never forms row0 + rows)
  RXLA_REQUIRE(row0 >= 0 && rows >= 0 && col0 >= 0 && cols >= 0 && rows <= R &&
                   row0 <= R - rows && cols <= C && col0 <= C - cols,
               "safetensors_read: block outside tensor " + t.name);
  const int64_t rb = C * t.elem, cb = cols * t.elem;
  auto pread_all = [&](uint8_t* d, int64_t n, int64_t off) -> bool {
    while (n > 0) {
      const ssize_t r = pread(f->fd, d, (size_t)std::min<int64_t>(n, 1 << 30), off);
      if (r <= 0) return false;
      d += r;
      n -= r;
      off += r;
    }
    return true;
  };
  const int64_t base = f->data_start + t.begin;
  if (cols == C) {  // whole rows: one read
    if (!pread_all(dst, rows * rb, base + row0 * rb))
      return fail(RXLA_B200_UNAVAILABLE, "safetensors_read: read failed for " + t.name);
    return RXLA_B200_OK;
  }
  for (int64_t r = 0; r < rows; ++r)
    if (!pread_all(dst + r * cb, cb, base + (row0 + r) * rb + col0 * t.elem))
      return fail(RXLA_B200_UNAVAILABLE, "safetensors_read: read failed for " + t.name);
  return RXLA_B200_OK;
}

}  // namespace st
}  // namespace rxla

extern "C" int32_t rxla_b200_safetensors_read(const rxla_b200_safetensors* f, int32_t index,
                                              int64_t row0, int64_t rows, int64_t col0,
                                              int64_t cols, void* dst, int64_t dst_bytes) {
  RXLA_REQUIRE(f && (dst || dst_bytes == 0), "safetensors_read: null argument");
  RXLA_REQUIRE(index >= 0 && index < (int32_t)f->tensors.size(),
               "safetensors_read: index out of range");
  const st::Tensor& t = f->tensors[(size_t)index];
  // checked product: rows * cols * elem must not wrap before it is compared
  int64_t want = 0;
  RXLA_REQUIRE(rows >= 0 && cols >= 0 && !__builtin_mul_overflow(rows, cols, &want) &&
                   !__builtin_mul_overflow(want, (int64_t)t.elem, &want) && dst_bytes == want,
               "safetensors_read: destination must hold exactly rows * cols elements");
  return st::read_block(f, t, row0, rows, col0, cols, static_cast<uint8_t*>(dst));
}

namespace rxla {
namespace dec {

// The rows and columns of a full (tp = 1) tensor that this rank's parameter
// holds: column-parallel q/k/v and gate/up by output rows, row-parallel
// o_proj / down_proj by input columns (per-channel scales whole), the rest
// whole.  The same rules as the Python shard_parameter.
static void shard_block(const std::string& n, int64_t R, int64_t C, const rxla_b200_decoder* d,
                        int64_t& r0, int64_t& nr, int64_t& c0, int64_t& nc) {
  const int tp = d->cfg.tp_size, rank = d->cfg.tp_rank;
  r0 = 0;
  nr = R;
  c0 = 0;
  nc = C;
  if (tp <= 1) return;
  auto ends = [&](const char* s) {
    const size_t l = strlen(s);
    return n.size() >= l && n.compare(n.size() - l, l, s) == 0;
  };
  const int64_t D = d->cfg.head_dim;
  if (ends("q_proj.weight") || ends("q_proj.scale")) {
    nr = (int64_t)d->hq * D;
    r0 = rank * nr;
  } else if (ends("k_proj.weight") || ends("k_proj.scale") || ends("v_proj.weight") ||
             ends("v_proj.scale")) {
    nr = (int64_t)d->hkv * D;
    r0 = rank * nr;
  } else if (ends("gate_proj.weight") || ends("gate_proj.scale") || ends("up_proj.weight") ||
             ends("up_proj.scale")) {
    nr = d->inter;
    r0 = rank * nr;
  } else if (ends("o_proj.weight") || ends("down_proj.weight") ||
             ((ends("o_proj.scale") || ends("down_proj.scale")) && C > 1)) {
    nc = C / tp;
    c0 = rank * nc;
  }
}

}  // namespace dec
}  // namespace rxla

extern "C" int32_t rxla_b200_decoder_load_safetensors(rxla_b200_decoder* d, const char* path,
                                                      const char* prefix, int32_t* loaded,
                                                      int32_t* skipped) {
  RXLA_REQUIRE(d && path, "decoder_load_safetensors: null argument");
  rxla_b200_safetensors* f = nullptr;
  int32_t st = rxla_b200_safetensors_open(path, &f);
  if (st) return st;
  struct Closer {
    rxla_b200_safetensors* f;
    ~Closer() { rxla_b200_safetensors_close(f); }
  } closer{f};
  // a checkpoint that states its group size must match the decoder's
  // (per-channel decoders, group_size 0, are checked by the scale sizes)
  auto gs = f->metadata.find("group_size");
  if (gs != f->metadata.end() && d->cfg.group_size > 0)
    RXLA_REQUIRE(atol(gs->second.c_str()) == d->cfg.group_size,
                 "decoder_load_safetensors: checkpoint group_size " + gs->second +
                     " differs from the decoder's " + std::to_string(d->cfg.group_size));
  const std::string pre = prefix ? prefix : "";
  std::map<std::string, int64_t> covered;  // bytes written per decoder parameter
  std::vector<uint8_t> host;
  int32_t n_loaded = 0, n_skipped = 0;
  RXLA_CUDA_CHECK(cudaSetDevice(d->device));
  for (const st::Tensor& t : f->tensors) {
    if (t.name.compare(0, pre.size(), pre) != 0) {
      ++n_skipped;
      continue;
    }
    const std::string name = t.name.substr(pre.size());
    void* ptr = nullptr;
    int64_t bytes = 0;
    int32_t dt = 0;
    if (rxla_b200_decoder_parameter(d, name.c_str(), &ptr, &bytes, &dt) != RXLA_B200_OK) {
      ++n_skipped;
      continue;
    }
    RXLA_REQUIRE(t.dtype == dt, "decoder_load_safetensors: " + t.name +
                                    " has the wrong dtype for parameter " + name);
    int64_t R, C, r0, nr, c0, nc;
    st::as_matrix(t, R, C);
    dec::shard_block(name, R, C, d, r0, nr, c0, nc);
    RXLA_REQUIRE(nr * nc * t.elem == bytes,
                 "decoder_load_safetensors: " + t.name + " holds " +
                     std::to_string(nr * nc * t.elem) + " bytes for this rank, parameter " +
                     name + " holds " + std::to_string(bytes));
    host.resize((size_t)bytes);
    st = st::read_block(f, t, r0, nr, c0, nc, host.data());
    if (st) return st;
    RXLA_CUDA_CHECK(cudaMemcpy(ptr, host.data(), (size_t)bytes, cudaMemcpyHostToDevice));
    for (auto& p : d->params)
      if (static_cast<uint8_t*>(ptr) >= static_cast<uint8_t*>(p.ptr) &&
          static_cast<uint8_t*>(ptr) < static_cast<uint8_t*>(p.ptr) + p.bytes)
        covered[p.name] += bytes;
    ++n_loaded;
  }
  for (auto& p : d->params)
    if (covered[p.name] != p.bytes)
      return fail(RXLA_B200_NOT_FOUND,
                  "decoder_load_safetensors: the checkpoint does not fill parameter " + p.name +
                      " (" + std::to_string(covered[p.name]) + " of " + std::to_string(p.bytes) +
                      " bytes)");
  if (loaded) *loaded = n_loaded;
  if (skipped) *skipped = n_skipped;
  return RXLA_B200_OK;
}
