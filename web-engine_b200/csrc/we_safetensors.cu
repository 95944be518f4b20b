// .safetensors reader of the weight loader (src/weights/safetensors.ts:1-70, src/model/weights.ts:26-50): the
// header is parsed and checked here, in native code, with the reference's checks and messages (the file is
// untrusted: every offset and size is validated before use); the data region is mapped read-only and a
// tensor goes to HBM through a pair of pinned staging chunks with asynchronous copies on the context's stream,
// so reading the next chunk from the page cache overlaps the DMA of the previous one.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/we_b200.h"

int we_ctx_fail(we_ctx* ctx, int code, const std::string& msg);
cudaStream_t we_ctx_stream(we_ctx* ctx);

namespace {

constexpr uint64_t kMaxHeader = 100000000;  // the Python library's limit (safetensors.ts:13)
constexpr size_t kChunk = 32u << 20;        // pinned staging chunk of an upload

// bytes per element (safetensors.ts:8-11)
int dtype_bytes(const std::string& d) {
  static const std::map<std::string, int> t = {{"F64", 8}, {"F32", 4},    {"F16", 2},     {"BF16", 2}, {"F8_E4M3", 1},
                                               {"F8_E5M2", 1}, {"I64", 8}, {"I32", 4}, {"I16", 2}, {"I8", 1},
                                               {"U64", 8}, {"U32", 4},     {"U16", 2},     {"U8", 1},   {"BOOL", 1}};
  auto it = t.find(d);
  return it == t.end() ? 0 : it->second;
}

// ---- a small JSON reader: objects keep their key order, numbers are doubles (as JSON.parse reads them) ----
struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
};

struct Parser {
  const char* p;
  const char* end;
  int depth = 0;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
  }
  bool lit(const char* s) {
    size_t n = std::strlen(s);
    if ((size_t)(end - p) < n || std::memcmp(p, s, n) != 0) return false;
    p += n;
    return true;
  }
  static void put_utf8(std::string& o, uint32_t c) {
    if (c < 0x80) o += (char)c;
    else if (c < 0x800) { o += (char)(0xC0 | (c >> 6)); o += (char)(0x80 | (c & 0x3F)); }
    else if (c < 0x10000) { o += (char)(0xE0 | (c >> 12)); o += (char)(0x80 | ((c >> 6) & 0x3F)); o += (char)(0x80 | (c & 0x3F)); }
    else { o += (char)(0xF0 | (c >> 18)); o += (char)(0x80 | ((c >> 12) & 0x3F)); o += (char)(0x80 | ((c >> 6) & 0x3F)); o += (char)(0x80 | (c & 0x3F)); }
  }
  bool hex4(uint32_t& v) {
    if (end - p < 4) return false;
    v = 0;
    for (int i = 0; i < 4; i++) {
      char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return false;
    }
    return true;
  }
  bool string(std::string& o) {
    if (p >= end || *p != '"') return false;
    p++;
    while (p < end && *p != '"') {
      unsigned char c = (unsigned char)*p++;
      if (c < 0x20) return false;
      if (c != '\\') { o += (char)c; continue; }
      if (p >= end) return false;
      char e = *p++;
      switch (e) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t v;
          if (!hex4(v)) return false;
          if (v >= 0xD800 && v < 0xDC00 && end - p >= 6 && p[0] == '\\' && p[1] == 'u') {
            const char* save = p;
            p += 2;
            uint32_t lo;
            if (hex4(lo) && lo >= 0xDC00 && lo < 0xE000) v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
            else p = save;
          }
          put_utf8(o, v);
          break;
        }
        default: return false;
      }
    }
    if (p >= end) return false;
    p++;
    return true;
  }
  bool number(double& v) {
    const char* s = p;
    if (p < end && *p == '-') p++;
    if (p >= end) return false;
    if (*p == '0') p++;
    else if (*p >= '1' && *p <= '9') while (p < end && *p >= '0' && *p <= '9') p++;
    else return false;
    if (p < end && *p == '.') {
      p++;
      if (p >= end || *p < '0' || *p > '9') return false;
      while (p < end && *p >= '0' && *p <= '9') p++;
    }
    if (p < end && (*p == 'e' || *p == 'E')) {
      p++;
      if (p < end && (*p == '+' || *p == '-')) p++;
      if (p >= end || *p < '0' || *p > '9') return false;
      while (p < end && *p >= '0' && *p <= '9') p++;
    }
    v = std::strtod(std::string(s, p).c_str(), nullptr);
    return true;
  }
  bool value(Json& j) {
    if (++depth > 128) return false;  // hostile nesting
    ws();
    bool r = false;
    if (p >= end) r = false;
    else if (*p == '{') {
      j.kind = Json::OBJ;
      p++;
      ws();
      if (p < end && *p == '}') { p++; r = true; }
      else {
        std::unordered_map<std::string, size_t> seen;
        for (;;) {
          ws();
          std::string k;
          if (!string(k)) break;
          ws();
          if (p >= end || *p != ':') break;
          p++;
          Json v;
          if (!value(v)) break;
          // a repeated key keeps its first position and takes the last value, as JSON.parse does
          auto it = seen.find(k);
          if (it != seen.end()) {
            j.obj[it->second].second = std::move(v);
          } else {
            seen.emplace(k, j.obj.size());
            j.obj.emplace_back(std::move(k), std::move(v));
          }
          ws();
          if (p < end && *p == ',') { p++; continue; }
          if (p < end && *p == '}') { p++; r = true; }
          break;
        }
      }
    } else if (*p == '[') {
      j.kind = Json::ARR;
      p++;
      ws();
      if (p < end && *p == ']') { p++; r = true; }
      else {
        for (;;) {
          Json v;
          if (!value(v)) break;
          j.arr.push_back(std::move(v));
          ws();
          if (p < end && *p == ',') { p++; continue; }
          if (p < end && *p == ']') { p++; r = true; }
          break;
        }
      }
    } else if (*p == '"') {
      j.kind = Json::STR;
      r = string(j.str);
    } else if (lit("true")) { j.kind = Json::BOOL; j.b = true; r = true; }
    else if (lit("false")) { j.kind = Json::BOOL; r = true; }
    else if (lit("null")) { j.kind = Json::NUL; r = true; }
    else { j.kind = Json::NUM; r = number(j.num); }
    depth--;
    return r;
  }
};

// Number.isSafeInteger(n) && n >= 0 (safetensors.ts:25)
bool is_count(const Json& j, int64_t& v) {
  if (j.kind != Json::NUM || !std::isfinite(j.num) || j.num < 0 || j.num > 9007199254740991.0 ||
      std::floor(j.num) != j.num)
    return false;
  v = (int64_t)j.num;
  return true;
}

// String(value) of the reference's message for a non-string dtype
std::string js_string(const Json* j) {
  if (!j) return "undefined";
  switch (j->kind) {
    case Json::NUL: return "null";
    case Json::BOOL: return j->b ? "true" : "false";
    case Json::NUM: {
      char buf[64];
      std::snprintf(buf, sizeof buf, "%.17g", j->num);
      return buf;
    }
    case Json::STR: return j->str;
    case Json::ARR: return "[array]";
    default: return "[object Object]";
  }
}

}  // namespace

struct we_st {
  int fd = -1;
  uint8_t* map = nullptr;
  size_t file_size = 0;
  struct Tensor {
    std::string name, dtype;
    std::vector<int64_t> shape;
    int64_t offset, size;
  };
  std::vector<Tensor> tensors;  // header order
  std::map<std::string, size_t> index;
  std::vector<std::pair<std::string, std::string>> metadata;
  // upload staging: two pinned chunks and the events of their last copies
  void* stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  int device = -1;
};

namespace {

int st_fail(char* err, size_t n, int code, const std::string& msg) {
  if (err && n) {
    std::strncpy(err, msg.c_str(), n - 1);
    err[n - 1] = 0;
  }
  return code;
}

void st_free(we_st* st) {
  if (!st) return;
  for (int i = 0; i < 2; i++) {
    if (st->done[i]) {
      cudaEventSynchronize(st->done[i]);
      cudaEventDestroy(st->done[i]);
    }
    if (st->stage[i]) cudaFreeHost(st->stage[i]);
  }
  if (st->map) munmap(st->map, st->file_size);
  if (st->fd >= 0) close(st->fd);
  delete st;
}

void fill(const we_st::Tensor& t, we_st_tensor* o) {
  o->name = t.name.c_str();
  o->dtype = t.dtype.c_str();
  o->ndim = (int32_t)t.shape.size();
  for (int i = 0; i < 8; i++) o->shape[i] = i < (int)t.shape.size() ? t.shape[i] : 0;
  o->offset = t.offset;
  o->size = t.size;
}

}  // namespace

extern "C" {

int we_st_open(const char* path, we_st** out, char* err, size_t err_len) {
  if (!path || !out) return st_fail(err, err_len, WE_EINVAL, "we_st_open: missing argument");
  *out = nullptr;
  std::unique_ptr<we_st, void (*)(we_st*)> st(new we_st(), st_free);
  st->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (st->fd < 0) return st_fail(err, err_len, WE_EIO, std::string("cannot open ") + path + ": " + std::strerror(errno));
  struct stat sb;
  if (fstat(st->fd, &sb) != 0) return st_fail(err, err_len, WE_EIO, std::string("cannot stat ") + path);
  st->file_size = (size_t)sb.st_size;
  if (st->file_size < 8) return st_fail(err, err_len, WE_EINVAL, "File is too small to be a .safetensors file");
  if (st->file_size > 0) {
    void* m = mmap(nullptr, st->file_size, PROT_READ, MAP_PRIVATE, st->fd, 0);
    if (m == MAP_FAILED) return st_fail(err, err_len, WE_EIO, std::string("cannot map ") + path);
    st->map = static_cast<uint8_t*>(m);
  }
  uint64_t hsize = 0;
  for (int i = 7; i >= 0; i--) hsize = (hsize << 8) | st->map[i];  // little-endian u64
  if (hsize > kMaxHeader || 8 + hsize > st->file_size)
    return st_fail(err, err_len, WE_EINVAL, "Bad header size: " + std::to_string(hsize));
  Json header;
  Parser ps{reinterpret_cast<const char*>(st->map + 8), reinterpret_cast<const char*>(st->map + 8 + hsize)};
  bool parsed = ps.value(header);
  ps.ws();
  if (!parsed || ps.p != ps.end) return st_fail(err, err_len, WE_EINVAL, "Header is not valid JSON");
  if (header.kind != Json::OBJ) return st_fail(err, err_len, WE_EINVAL, "Header is not an object");
  const int64_t start = 8 + (int64_t)hsize;
  const int64_t data_size = (int64_t)st->file_size - start;
  for (auto& kv : header.obj) {
    const std::string& name = kv.first;
    const Json& e = kv.second;
    if (name == "__metadata__") {
      if (e.kind == Json::OBJ)
        for (auto& m : e.obj)
          if (m.second.kind == Json::STR) st->metadata.emplace_back(m.first, m.second.str);
      continue;
    }
    auto field = [&](const char* f) -> const Json* {
      if (e.kind != Json::OBJ) return nullptr;
      for (auto& x : e.obj)
        if (x.first == f) return &x.second;
      return nullptr;
    };
    const Json* dt = field("dtype");
    if (!dt || dt->kind != Json::STR || !dtype_bytes(dt->str))
      return st_fail(err, err_len, WE_EINVAL, name + ": unknown dtype " + js_string(dt));
    const Json* sh = field("shape");
    std::vector<int64_t> shape;
    bool shape_ok = sh && sh->kind == Json::ARR;
    if (shape_ok)
      for (auto& d : sh->arr) {
        int64_t v;
        if (!is_count(d, v)) { shape_ok = false; break; }
        shape.push_back(v);
      }
    if (!shape_ok) return st_fail(err, err_len, WE_EINVAL, name + ": bad shape");
    const Json* off = field("data_offsets");
    int64_t begin = 0, fin = 0;
    if (!off || off->kind != Json::ARR || off->arr.size() != 2 || !is_count(off->arr[0], begin) ||
        !is_count(off->arr[1], fin))
      return st_fail(err, err_len, WE_EINVAL, name + ": bad data_offsets");
    // the element count in float64, as the reference's reduce computes it
    double expected = dtype_bytes(dt->str);
    for (int64_t d : shape) expected *= (double)d;
    if ((double)(fin - begin) != expected) {
      char buf[64];
      std::snprintf(buf, sizeof buf, "%.17g", expected);
      return st_fail(err, err_len, WE_EINVAL,
                     name + ": has " + std::to_string(fin - begin) + " bytes, its shape needs " + buf + " bytes");
    }
    if (fin > data_size) return st_fail(err, err_len, WE_EINVAL, name + ": data goes past the end of the file");
    if (st->index.count(name)) {  // unreachable: repeated keys were merged while parsing
      continue;
    }
    st->index[name] = st->tensors.size();
    st->tensors.push_back({name, dt->str, shape, start + begin, fin - begin});
  }
  std::vector<const we_st::Tensor*> sorted;
  for (auto& t : st->tensors) sorted.push_back(&t);
  std::stable_sort(sorted.begin(), sorted.end(), [](auto a, auto b) { return a->offset < b->offset; });
  for (size_t i = 1; i < sorted.size(); i++)
    if (sorted[i]->offset < sorted[i - 1]->offset + sorted[i - 1]->size)
      return st_fail(err, err_len, WE_EINVAL, sorted[i - 1]->name + " and " + sorted[i]->name + " overlap");
  *out = st.release();
  return WE_OK;
}

int64_t we_st_count(const we_st* st) { return st ? (int64_t)st->tensors.size() : 0; }

int we_st_tensor_at(const we_st* st, int64_t i, we_st_tensor* out) {
  if (!st || !out || i < 0 || i >= (int64_t)st->tensors.size()) return WE_EINVAL;
  fill(st->tensors[(size_t)i], out);
  return WE_OK;
}

int we_st_find(const we_st* st, const char* name, we_st_tensor* out) {
  if (!st || !name || !out) return WE_EINVAL;
  auto it = st->index.find(name);
  if (it == st->index.end()) return WE_EINVAL;
  fill(st->tensors[it->second], out);
  return WE_OK;
}

int64_t we_st_metadata_count(const we_st* st) { return st ? (int64_t)st->metadata.size() : 0; }

int we_st_metadata_at(const we_st* st, int64_t i, const char** key, const char** value) {
  if (!st || !key || !value || i < 0 || i >= (int64_t)st->metadata.size()) return WE_EINVAL;
  *key = st->metadata[(size_t)i].first.c_str();
  *value = st->metadata[(size_t)i].second.c_str();
  return WE_OK;
}

int we_st_read(const we_st* st, const char* name, void* dst, int64_t limit) {
  if (!st || !name || (!dst && limit != 0)) return WE_EINVAL;
  auto it = st->index.find(name);
  if (it == st->index.end()) return WE_EINVAL;
  const auto& t = st->tensors[it->second];
  const int64_t n = limit < 0 ? t.size : std::min(limit, t.size);
  if (n > 0) std::memcpy(dst, st->map + t.offset, (size_t)n);
  return WE_OK;
}

int we_st_upload(we_ctx* ctx, we_st* st, const char* name, void* device_dst) {
  if (!ctx) return WE_EINVAL;
  if (!st || !name || !device_dst) return we_ctx_fail(ctx, WE_EINVAL, "we_st_upload: missing argument");
  auto it = st->index.find(name);
  if (it == st->index.end()) return we_ctx_fail(ctx, WE_EINVAL, std::string("Missing tensor ") + name);
  const auto& t = st->tensors[it->second];
  cudaStream_t stream = we_ctx_stream(ctx);
  int dev = 0;
  cudaGetDevice(&dev);
  if (st->device != dev) {  // staging belongs to one device
    for (int i = 0; i < 2; i++) {
      if (st->done[i]) { cudaEventSynchronize(st->done[i]); cudaEventDestroy(st->done[i]); st->done[i] = nullptr; }
      if (st->stage[i]) { cudaFreeHost(st->stage[i]); st->stage[i] = nullptr; }
    }
    st->device = dev;
  }
  for (int i = 0; i < 2; i++) {
    if (!st->stage[i]) {
      cudaError_t e = cudaHostAlloc(&st->stage[i], kChunk, cudaHostAllocDefault);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&st->done[i], cudaEventDisableTiming);
      if (e != cudaSuccess) return we_ctx_fail(ctx, WE_ECUDA, std::string("upload staging: ") + cudaGetErrorString(e));
    }
  }
  int64_t pos = 0;
  int k = 0;
  while (pos < t.size) {
    const size_t n = (size_t)std::min<int64_t>((int64_t)kChunk, t.size - pos);
    cudaError_t e = cudaEventSynchronize(st->done[k]);  // the chunk's previous copy has left it
    if (e == cudaSuccess) {
      std::memcpy(st->stage[k], st->map + t.offset + pos, n);
      e = cudaMemcpyAsync(static_cast<uint8_t*>(device_dst) + pos, st->stage[k], n, cudaMemcpyHostToDevice, stream);
    }
    if (e == cudaSuccess) e = cudaEventRecord(st->done[k], stream);
    if (e != cudaSuccess) return we_ctx_fail(ctx, WE_ECUDA, std::string("upload: ") + cudaGetErrorString(e));
    pos += (int64_t)n;
    k ^= 1;
  }
  return WE_OK;
}

void we_st_close(we_st* st) { st_free(st); }

}  // extern "C"
