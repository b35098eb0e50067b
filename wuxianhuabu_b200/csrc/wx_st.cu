// wx_st.cu — safetensors checkpoint reader (host side): the lazy, memory-mapped
// container of the reference (H3Weights, model/minimax h3/H3Common.swift:180-261,
// over MappedSafetensors) with its quantized-triple lookup that accepts both
// naming variants (`prefix.scales/.biases` and `prefix.weight.scales/.weight.biases`,
// H3Common.swift:243-258) and MfLinear.load's geometry rules (bits = 32*w_cols/in,
// group = in/s_cols, H3Common.swift:311-338).
//
// File layout (safetensors): u64 little-endian header length N, N bytes of JSON
// {"name": {"dtype": "BF16", "shape": [..], "data_offsets": [begin, end]}, ...,
//  "__metadata__": {...}}, then the data block; offsets are relative to it.
// The file is mapped read-only; tensors are copied to device memory on demand.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "wx_internal.h"

struct wx_st_file {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t size = 0;
  size_t data0 = 0;  // start of the data block
  std::vector<std::string> names;
  std::vector<wx_st_info> infos;
  std::unordered_map<std::string, size_t> index;
};

namespace wx {
namespace {

// Minimal JSON reader for the safetensors header (objects, arrays, strings,
// numbers, literals); values the reader does not need are skipped.
struct Json {
  const char* p;
  const char* e;
  bool ok = true;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return ok = false;
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\') {
        if (++p >= e) return ok = false;
        switch (*p) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {  // keep the escape verbatim: names are compared byte-wise
            if (e - p < 5) return ok = false;
            out.append("\\u");
            out.append(p + 1, 4);
            p += 4;
            break;
          }
          default: out += *p;
        }
        ++p;
      } else {
        out += *p++;
      }
    }
    if (p >= e) return ok = false;
    ++p;
    return true;
  }
  bool num(int64_t& v) {
    ws();
    const char* s = p;
    if (p < e && (*p == '-' || *p == '+')) ++p;
    while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '-' || *p == '+'))
      ++p;
    if (p == s) return ok = false;
    v = strtoll(std::string(s, p).c_str(), nullptr, 10);
    return true;
  }
  bool skip() {  // any value
    ws();
    if (p >= e) return ok = false;
    if (*p == '"') {
      std::string t;
      return str(t);
    }
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      const bool obj = *p == '{';
      ++p;
      if (eat(close)) return true;
      do {
        if (obj) {
          std::string k;
          if (!str(k) || !eat(':')) return ok = false;
        }
        if (!skip()) return false;
      } while (eat(','));
      return eat(close) || (ok = false);
    }
    if (*p == 't' || *p == 'f' || *p == 'n') {
      while (p < e && *p >= 'a' && *p <= 'z') ++p;
      return true;
    }
    int64_t v;
    return num(v);
  }
};

size_t dtype_size(const char* d) {
  static const struct {
    const char* n;
    size_t s;
  } t[] = {{"F64", 8}, {"I64", 8}, {"U64", 8}, {"F32", 4}, {"I32", 4}, {"U32", 4}, {"F16", 2}, {"BF16", 2},
           {"I16", 2}, {"U16", 2}, {"I8", 1}, {"U8", 1}, {"BOOL", 1}, {"F8_E4M3", 1}, {"F8_E5M2", 1}};
  for (const auto& x : t)
    if (!strcmp(x.n, d)) return x.s;
  return 0;
}

int parse_header(wx_st_file* f, const char* hdr, size_t n, std::string& err) {
  Json j{hdr, hdr + n};
  if (!j.eat('{')) {
    err = "header is not a JSON object";
    return WX_ERR_INVALID;
  }
  if (j.eat('}')) return WX_OK;
  do {
    std::string name;
    if (!j.str(name) || !j.eat(':')) {
      err = "malformed header key";
      return WX_ERR_INVALID;
    }
    if (name == "__metadata__") {
      if (!j.skip()) {
        err = "malformed __metadata__";
        return WX_ERR_INVALID;
      }
      continue;
    }
    wx_st_info info{};
    bool have_dtype = false, have_shape = false, have_off = false;
    int64_t off0 = 0, off1 = 0;
    if (!j.eat('{')) {
      err = "tensor entry is not an object: " + name;
      return WX_ERR_INVALID;
    }
    if (!j.eat('}')) {
      do {
        std::string k;
        if (!j.str(k) || !j.eat(':')) {
          err = "malformed entry of " + name;
          return WX_ERR_INVALID;
        }
        if (k == "dtype") {
          std::string d;
          if (!j.str(d) || d.size() >= sizeof(info.dtype)) {
            err = "bad dtype of " + name;
            return WX_ERR_INVALID;
          }
          memcpy(info.dtype, d.c_str(), d.size() + 1);
          have_dtype = true;
        } else if (k == "shape") {
          if (!j.eat('[')) {
            err = "bad shape of " + name;
            return WX_ERR_INVALID;
          }
          info.ndim = 0;
          if (!j.eat(']')) {
            do {
              int64_t v;
              if (info.ndim >= 8 || !j.num(v) || v < 0) {
                err = "bad shape of " + name;
                return WX_ERR_INVALID;
              }
              info.shape[info.ndim++] = v;
            } while (j.eat(','));
            if (!j.eat(']')) {
              err = "bad shape of " + name;
              return WX_ERR_INVALID;
            }
          }
          have_shape = true;
        } else if (k == "data_offsets") {
          if (!j.eat('[') || !j.num(off0) || !j.eat(',') || !j.num(off1) || !j.eat(']')) {
            err = "bad data_offsets of " + name;
            return WX_ERR_INVALID;
          }
          have_off = true;
        } else if (!j.skip()) {
          err = "malformed entry of " + name;
          return WX_ERR_INVALID;
        }
      } while (j.eat(','));
      if (!j.eat('}')) {
        err = "malformed entry of " + name;
        return WX_ERR_INVALID;
      }
    }
    if (!have_dtype || !have_shape || !have_off) {
      err = "incomplete entry " + name;
      return WX_ERR_INVALID;
    }
    const size_t es = dtype_size(info.dtype);
    uint64_t count = 1;
    for (int d = 0; d < info.ndim; ++d) count *= (uint64_t)info.shape[d];
    if (off0 < 0 || off1 < off0 || f->data0 + (uint64_t)off1 > f->size || (es && count * es != (uint64_t)(off1 - off0))) {
      err = "data_offsets out of range or inconsistent with dtype/shape: " + name;
      return WX_ERR_INVALID;
    }
    info.offset = f->data0 + (uint64_t)off0;
    info.nbytes = (uint64_t)(off1 - off0);
    info.host = f->map + info.offset;
    f->index[name] = f->infos.size();
    f->names.push_back(name);
    f->infos.push_back(info);
  } while (j.eat(','));
  if (!j.eat('}') || !j.ok) {
    err = "malformed header";
    return WX_ERR_INVALID;
  }
  return WX_OK;
}

thread_local std::string g_st_err;

}  // namespace
}  // namespace wx

using namespace wx;

extern "C" {

const char* wx_st_last_error(void) { return g_st_err.c_str(); }

int wx_st_open(const char* path, wx_st_file** out) {
  if (!path || !out) return WX_ERR_INVALID;
  *out = nullptr;
  auto* f = new wx_st_file();
  auto fail = [&](int st, const std::string& msg) {
    g_st_err = std::string(path) + ": " + msg;
    if (f->map) munmap(const_cast<uint8_t*>(f->map), f->size);
    if (f->fd >= 0) close(f->fd);
    delete f;
    return st;
  };
  f->fd = open(path, O_RDONLY);
  if (f->fd < 0) return fail(WX_ERR_INVALID, "cannot open");
  struct stat sb;
  if (fstat(f->fd, &sb) != 0 || sb.st_size < 8) return fail(WX_ERR_INVALID, "not a safetensors file (too short)");
  f->size = (size_t)sb.st_size;
  void* m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
  if (m == MAP_FAILED) return fail(WX_ERR_INVALID, "mmap failed");
  f->map = static_cast<const uint8_t*>(m);
  uint64_t n = 0;
  memcpy(&n, f->map, 8);  // little-endian u64 (host order on x86-64 / aarch64)
  if (n == 0 || n > f->size - 8 || n > (uint64_t)100 << 20) return fail(WX_ERR_INVALID, "bad header length");
  f->data0 = 8 + (size_t)n;
  std::string err;
  const int st = parse_header(f, reinterpret_cast<const char*>(f->map + 8), (size_t)n, err);
  if (st) return fail(st, err);
  *out = f;
  return WX_OK;
}

int wx_st_close(wx_st_file* f) {
  if (!f) return WX_OK;
  if (f->map) munmap(const_cast<uint8_t*>(f->map), f->size);
  if (f->fd >= 0) close(f->fd);
  delete f;
  return WX_OK;
}

int64_t wx_st_count(const wx_st_file* f) { return f ? (int64_t)f->names.size() : 0; }

const char* wx_st_name(const wx_st_file* f, int64_t i) {
  if (!f || i < 0 || i >= (int64_t)f->names.size()) return nullptr;
  return f->names[(size_t)i].c_str();
}

int wx_st_find(const wx_st_file* f, const char* name, wx_st_info* out) {
  if (!f || !name || !out) return WX_ERR_INVALID;
  auto it = f->index.find(name);
  if (it == f->index.end()) return WX_ERR_INVALID;
  *out = f->infos[it->second];
  return WX_OK;
}

int wx_st_upload(wx_ctx* ctx, const wx_st_file* f, const char* name, void* dst, uint64_t dst_bytes) {
  WX_CHECK_ARG(ctx, ctx && f && name && dst);
  wx_st_info info;
  if (wx_st_find(f, name, &info) != WX_OK) return set_error(ctx, WX_ERR_INVALID, "no tensor %s in the file", name);
  if (info.nbytes > dst_bytes)
    return set_error(ctx, WX_ERR_INVALID, "%s needs %llu bytes, destination has %llu", name,
                     (unsigned long long)info.nbytes, (unsigned long long)dst_bytes);
  // pageable source: the copy is staged by the driver and complete when this returns
  cudaError_t e = cudaMemcpyAsync(dst, info.host, info.nbytes, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return set_error(ctx, WX_ERR_CUDA, "upload of %s: %s", name, cudaGetErrorString(e));
  return WX_OK;
}

int wx_st_find_qlinear(const wx_st_file* f, const char* prefix, int64_t in_features, wx_st_info* wq,
                       wx_st_info* scales, wx_st_info* biases, wx_st_info* bias, int32_t* bits, int32_t* group) {
  if (!f || !prefix || in_features <= 0 || !wq || !scales || !biases || !bias || !bits || !group) {
    g_st_err = "wx_st_find_qlinear: invalid arguments";
    return WX_ERR_INVALID;
  }
  const std::string p(prefix);
  if (wx_st_find(f, (p + ".weight").c_str(), wq) != WX_OK) {
    g_st_err = "missing weight: " + p + ".weight";
    return WX_ERR_INVALID;
  }
  // mlx-serve naming first, then the comfy / HF spelling (H3Common.swift:250-257)
  if (!(wx_st_find(f, (p + ".scales").c_str(), scales) == WX_OK &&
        wx_st_find(f, (p + ".biases").c_str(), biases) == WX_OK) &&
      !(wx_st_find(f, (p + ".weight.scales").c_str(), scales) == WX_OK &&
        wx_st_find(f, (p + ".weight.biases").c_str(), biases) == WX_OK)) {
    g_st_err = "not a quantized linear (no scales/biases): " + p;
    return WX_ERR_INVALID;
  }
  if (wq->ndim != 2 || scales->ndim != 2 || biases->ndim != 2 || strcmp(wq->dtype, "U32") ||
      scales->shape[0] != wq->shape[0] || biases->shape[0] != wq->shape[0] || scales->shape[1] != biases->shape[1] ||
      scales->shape[1] <= 0 || in_features % scales->shape[1] != 0 || (32 * wq->shape[1]) % in_features != 0) {
    g_st_err = "inconsistent quantized triple: " + p;
    return WX_ERR_INVALID;
  }
  *bits = (int32_t)(32 * wq->shape[1] / in_features);
  *group = (int32_t)(in_features / scales->shape[1]);
  if (wx_st_find(f, (p + ".bias").c_str(), bias) != WX_OK) memset(bias, 0, sizeof(*bias));
  return WX_OK;
}

}  // extern "C"
