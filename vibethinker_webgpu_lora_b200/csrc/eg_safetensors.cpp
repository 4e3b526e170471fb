// eg_safetensors.cpp -- streaming safetensors model loader (host, C++).
//
// The reference's loader (src/qwgpu/safetensors_loader.js:83-126) reads
// model.safetensors.index.json when present (else one model.safetensors),
// then, shard by shard, parses the header (u64 little-endian length + JSON),
// and for each tensor fetches its byte range, decodes BF16 / F16 / F32 to
// f32 (:20-54), hands it to ModelUploader.visit (model_uploader.js:39-63:
// schema check, quantise, upload) and drops it.  Here each shard is
// memory-mapped, each tensor is decoded into one reusable f32 buffer (OpenMP
// over elements) and passed to eg_upload_tensor, which applies the schema
// (unknown names skipped, shape errors, duplicates), the bit-exact
// quantisers and the device upload.  Peak host memory is one decoded tensor
// plus its quantised copy.
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "eg_host.h"
#include "emberglass.h"

namespace eg {
namespace {

// ---------------------------------------------------------------- JSON
// A small JSON reader, enough for safetensors headers and index files.
struct JVal {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const char* k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JParser {
  const char* p;
  const char* end;
  std::string err;
  int depth = 0;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
  }
  bool fail(const char* m) {
    if (err.empty()) err = m;
    return false;
  }
  bool str(std::string& out) {
    if (p >= end || *p != '"') return fail("expected a string");
    p++;
    while (p < end && *p != '"') {
      char c = *p++;
      if (c != '\\') {
        out.push_back(c);
        continue;
      }
      if (p >= end) return fail("bad escape");
      c = *p++;
      switch (c) {
        case '"': case '\\': case '/': out.push_back(c); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          if (end - p < 4) return fail("bad \\u escape");
          unsigned cp = 0;
          for (int i = 0; i < 4; i++) {
            const char h = *p++;
            cp <<= 4;
            if (h >= '0' && h <= '9') cp |= h - '0';
            else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
            else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
            else return fail("bad \\u escape");
          }
          if (cp < 0x80) {
            out.push_back((char)cp);
          } else if (cp < 0x800) {
            out.push_back((char)(0xC0 | (cp >> 6)));
            out.push_back((char)(0x80 | (cp & 0x3F)));
          } else {
            out.push_back((char)(0xE0 | (cp >> 12)));
            out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            out.push_back((char)(0x80 | (cp & 0x3F)));
          }
          break;
        }
        default: return fail("bad escape");
      }
    }
    if (p >= end) return fail("unterminated string");
    p++;
    return true;
  }
  bool val(JVal& v) {
    if (++depth > 64) return fail("JSON nested too deeply");
    ws();
    if (p >= end) return fail("unexpected end of JSON");
    bool ok = true;
    if (*p == '{') {
      v.kind = JVal::OBJ;
      p++;
      ws();
      if (p < end && *p == '}') {
        p++;
      } else {
        for (;;) {
          ws();
          std::string k;
          if (!str(k)) return false;
          ws();
          if (p >= end || *p != ':') return fail("expected ':'");
          p++;
          v.obj.emplace_back(std::move(k), JVal());
          if (!val(v.obj.back().second)) return false;
          ws();
          if (p < end && *p == ',') { p++; continue; }
          if (p < end && *p == '}') { p++; break; }
          return fail("expected ',' or '}'");
        }
      }
    } else if (*p == '[') {
      v.kind = JVal::ARR;
      p++;
      ws();
      if (p < end && *p == ']') {
        p++;
      } else {
        for (;;) {
          v.arr.emplace_back();
          if (!val(v.arr.back())) return false;
          ws();
          if (p < end && *p == ',') { p++; continue; }
          if (p < end && *p == ']') { p++; break; }
          return fail("expected ',' or ']'");
        }
      }
    } else if (*p == '"') {
      v.kind = JVal::STR;
      ok = str(v.str);
    } else if (end - p >= 4 && !strncmp(p, "true", 4)) {
      v.kind = JVal::BOOL;
      v.b = true;
      p += 4;
    } else if (end - p >= 5 && !strncmp(p, "false", 5)) {
      v.kind = JVal::BOOL;
      p += 5;
    } else if (end - p >= 4 && !strncmp(p, "null", 4)) {
      p += 4;
    } else {
      const char* s = p;
      if (p < end && (*p == '-' || *p == '+')) p++;
      while (p < end && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' ||
                         *p == '-' || *p == '+'))
        p++;
      if (p == s) return fail("unexpected character in JSON");
      v.kind = JVal::NUM;
      v.num = strtod(std::string(s, p).c_str(), nullptr);
    }
    depth--;
    return ok;
  }
};

bool parse_json(const char* s, size_t n, JVal& out, std::string& err) {
  JParser ps{s, s + n, {}, 0};
  if (!ps.val(out)) {
    err = ps.err;
    return false;
  }
  ps.ws();
  if (ps.p != ps.end) {
    err = "trailing characters after JSON";
    return false;
  }
  return true;
}

// ---------------------------------------------------------------- files
struct Mapped {
  const unsigned char* p = nullptr;
  size_t n = 0;
  ~Mapped() {
    if (p) munmap((void*)p, n);
  }
};

eg_status map_file(const std::string& path, Mapped& m) {
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return fail(EG_ERR_ARG, "cannot open %s", path.c_str());
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 8) {
    close(fd);
    return fail(EG_ERR_ARG, "%s: not a safetensors file (size)", path.c_str());
  }
  void* p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return fail(EG_ERR_ARG, "cannot map %s", path.c_str());
  m.p = (const unsigned char*)p;
  m.n = (size_t)st.st_size;
  return EG_OK;
}

bool read_text(const std::string& path, std::string& out) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  char buf[65536];
  size_t k;
  while ((k = fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, k);
  fclose(f);
  return true;
}

struct TensorRef {
  std::string name, dtype;
  std::vector<int64_t> shape;
  size_t begin = 0, end = 0;  // byte offsets into the shard's data section
  int64_t numel = 1;
};

struct Shard {
  std::string path;
  Mapped m;
  size_t data_start = 0;
  std::vector<TensorRef> tensors;  // header order
};

int elem_bytes(const std::string& dt) {
  if (dt == "BF16" || dt == "F16" || dt == "FP16") return 2;
  if (dt == "F32" || dt == "FP32") return 4;
  return 0;
}

// The header (u64 LE length + JSON), validated against the file size.
eg_status open_shard(const std::string& path, Shard& sh) {
  sh.path = path;
  eg_status s = map_file(path, sh.m);
  if (s) return s;
  uint64_t hl = 0;
  memcpy(&hl, sh.m.p, 8);  // little-endian hosts only (x86-64 / aarch64)
  if (hl > sh.m.n - 8) return fail(EG_ERR_ARG, "%s: header length %llu exceeds the file", path.c_str(),
                                   (unsigned long long)hl);
  JVal hdr;
  std::string err;
  if (!parse_json((const char*)sh.m.p + 8, (size_t)hl, hdr, err) || hdr.kind != JVal::OBJ)
    return fail(EG_ERR_ARG, "%s: bad header JSON (%s)", path.c_str(), err.c_str());
  sh.data_start = 8 + (size_t)hl;
  const size_t data_n = sh.m.n - sh.data_start;
  for (auto& kv : hdr.obj) {
    if (kv.first == "__metadata__") continue;
    const JVal& t = kv.second;
    const JVal *dt = t.get("dtype"), *shp = t.get("shape"), *off = t.get("data_offsets");
    if (!dt || dt->kind != JVal::STR || !shp || shp->kind != JVal::ARR || !off ||
        off->kind != JVal::ARR || off->arr.size() != 2)
      return fail(EG_ERR_ARG, "%s: bad header entry for %s", path.c_str(), kv.first.c_str());
    TensorRef r;
    r.name = kv.first;
    r.dtype = dt->str;
    for (auto& c : r.dtype) c = (char)toupper((unsigned char)c);
    if (shp->arr.size() > 8) return fail(EG_ERR_ARG, "%s: %s has more than 8 dims", path.c_str(), kv.first.c_str());
    for (auto& d : shp->arr) {
      if (d.kind != JVal::NUM || d.num < 0 || d.num > 1e15)
        return fail(EG_ERR_ARG, "%s: bad shape of %s", path.c_str(), kv.first.c_str());
      r.shape.push_back((int64_t)d.num);
      if (r.shape.back() && r.numel > ((int64_t)1 << 50) / r.shape.back())
        return fail(EG_ERR_ARG, "%s: %s is too large", path.c_str(), kv.first.c_str());
      r.numel *= r.shape.back();
    }
    if (off->arr[0].kind != JVal::NUM || off->arr[1].kind != JVal::NUM)
      return fail(EG_ERR_ARG, "%s: bad data_offsets of %s", path.c_str(), kv.first.c_str());
    r.begin = (size_t)off->arr[0].num;
    r.end = (size_t)off->arr[1].num;
    if (r.end < r.begin || r.end > data_n)
      return fail(EG_ERR_ARG, "%s: data_offsets of %s outside the file", path.c_str(), kv.first.c_str());
    const int eb = elem_bytes(r.dtype);
    if (eb && (size_t)r.numel * eb != r.end - r.begin)
      return fail(EG_ERR_ARG, "%s: %s has %lld elements but %zu bytes", path.c_str(), kv.first.c_str(),
                  (long long)r.numel, r.end - r.begin);
    sh.tensors.push_back(std::move(r));
  }
  return EG_OK;
}

// Decode to f32 (safetensors_loader.js:20-54): BF16 = the upper 16 bits of
// an f32; F16 exact (subnormals, inf, NaN); F32 copied.
eg_status decode(const Shard& sh, const TensorRef& r, float* out) {
  const unsigned char* src = sh.m.p + sh.data_start + r.begin;
  const int64_t n = r.numel;
  if (r.dtype == "BF16") {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
      uint16_t h;
      memcpy(&h, src + 2 * i, 2);
      const uint32_t u = (uint32_t)h << 16;
      memcpy(out + i, &u, 4);
    }
  } else if (r.dtype == "F16" || r.dtype == "FP16") {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
      uint16_t h;
      memcpy(&h, src + 2 * i, 2);
      const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1F, f = h & 0x3FF;
      uint32_t u;
      if (e == 0x1F) {
        u = s | 0x7F800000u | (f << 13);  // inf / NaN (payload kept)
      } else if (e != 0) {
        u = s | ((e + 112) << 23) | (f << 13);  // rebias 15 -> 127
      } else if (f == 0) {
        u = s;  // +-0
      } else {  // subnormal: f * 2^-24, normalised
        int k = 0;
        uint32_t m = f;
        while (!(m & 0x400)) {
          m <<= 1;
          k++;
        }
        u = s | ((uint32_t)(113 - k) << 23) | ((m & 0x3FF) << 13);
      }
      memcpy(out + i, &u, 4);
    }
  } else if (r.dtype == "F32" || r.dtype == "FP32") {
    memcpy(out, src, (size_t)n * 4);
  } else {
    return fail(EG_ERR_ARG, "unsupported dtype %s for %s", r.dtype.c_str(), r.name.c_str());
  }
  return EG_OK;
}

// Shards of a model: `path` is a .safetensors file, or a directory holding
// model.safetensors.index.json (weight_map -> shard files) or
// model.safetensors (loadIndex, safetensors_loader.js:56-63).
eg_status shard_paths(const std::string& path, std::vector<std::string>& out) {
  struct stat st;
  if (stat(path.c_str(), &st) != 0) return fail(EG_ERR_ARG, "no such file or directory: %s", path.c_str());
  if (!S_ISDIR(st.st_mode)) {
    out.push_back(path);
    return EG_OK;
  }
  std::string idx;
  if (read_text(path + "/model.safetensors.index.json", idx)) {
    JVal j;
    std::string err;
    if (!parse_json(idx.data(), idx.size(), j, err))
      return fail(EG_ERR_ARG, "model.safetensors.index.json: %s", err.c_str());
    const JVal* wm = j.get("weight_map");
    if (wm && wm->kind == JVal::OBJ) {
      for (auto& kv : wm->obj) {
        if (kv.second.kind != JVal::STR) continue;
        bool have = false;
        for (auto& o : out) have |= o == path + "/" + kv.second.str;
        if (!have) out.push_back(path + "/" + kv.second.str);
      }
    }
    if (!out.empty()) return EG_OK;
  }
  out.push_back(path + "/model.safetensors");
  return EG_OK;
}

}  // namespace
}  // namespace eg

using namespace eg;

EG_API eg_status eg_safetensors_tensor(const char* path, const char* name, float* out,
                                       int64_t capacity, int64_t* shape, int* ndim) {
  if (!path || !name) return fail(EG_ERR_ARG, "safetensors_tensor: null argument");
  std::vector<std::string> shards;
  eg_status s = shard_paths(path, shards);
  if (s) return s;
  for (auto& sp : shards) {
    Shard sh;
    if ((s = open_shard(sp, sh))) return s;
    for (auto& r : sh.tensors) {
      if (r.name != name) continue;
      if (ndim) *ndim = (int)r.shape.size();
      if (shape)
        for (size_t i = 0; i < r.shape.size() && i < 8; i++) shape[i] = r.shape[i];
      if (!out) return EG_OK;  // shape query
      if (r.numel > capacity)
        return fail(EG_ERR_ARG, "%s has %lld elements, buffer holds %lld", name, (long long)r.numel,
                    (long long)capacity);
      return decode(sh, r, out);
    }
  }
  return fail(EG_ERR_ARG, "tensor %s not found in %s", name, path);
}

EG_API eg_status eg_load_safetensors(eg_rt* rt, const char* path, int* n_uploaded) {
  if (!rt || !path) return fail(EG_ERR_ARG, "load_safetensors: null argument");
  if (n_uploaded) *n_uploaded = 0;
  std::vector<std::string> shards;
  eg_status s = shard_paths(path, shards);
  if (s) return s;
  std::vector<float> buf;
  int n = 0;
  for (auto& sp : shards) {
    Shard sh;
    if ((s = open_shard(sp, sh))) return s;
    for (auto& r : sh.tensors) {
      if (!elem_bytes(r.dtype))
        return fail(EG_ERR_ARG, "unsupported dtype %s for %s", r.dtype.c_str(), r.name.c_str());
      if ((int64_t)buf.size() < r.numel) buf.resize((size_t)r.numel);
      if ((s = decode(sh, r, buf.data()))) return s;
      // schema check, quantisation and upload; unknown names are skipped
      if ((s = eg_upload_tensor(rt, r.name.c_str(), buf.data(), r.shape.data(), (int)r.shape.size())))
        return s;
      n++;
    }
  }
  if (n_uploaded) *n_uploaded = n;
  return EG_OK;
}
