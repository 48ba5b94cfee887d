// safetensors.cpp — MLX safetensors weights into the DiT engine.
//
// Replaces the weight path of TransformerWeights.loadQuantized
// (Sources/ImarelloDiT/TransformerWeights.swift:13-32) and the direct engine's
// per-key uploads (DirectDiTStep.loadBlocks / loadHead,
// Sources/ImarelloDirect/DirectDiTStep.swift:278-335,844-884): shard discovery
// as SafetensorsLoader.shardFileNames (Sources/ImarelloWeights/SafetensorsLoader.swift:6-29,
// index.json weight_map when present, else every *.safetensors sorted), later
// shards overriding earlier ones as in loadMergedArrays
// (SafetensorsLoader+MLX.swift:6-16).
//
// File format (safetensors): u64 little-endian header length N, N bytes of JSON
// {"<name>": {"dtype": "...", "shape": [...], "data_offsets": [begin, end]},
// "__metadata__": {...}}, then the data block (offsets relative to its start).
// Shards are mapped read-only; tensors are copied to a device staging buffer
// and handed to aex_dit_load_linear / aex_dit_load_norm.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <dirent.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "internal.h"

namespace aex {
namespace st {
namespace {

// ------------------------------------------------------------------ JSON
struct JVal {
  enum Type { kNull, kBool, kNum, kStr, kArr, kObj } type = kNull;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct Parser {
  const char* p;
  const char* end;
  std::string err;
  int depth = 0;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool fail(const char* what) {
    if (err.empty()) err = what;
    return false;
  }
  static void put_utf8(std::string& s, unsigned c) {
    if (c < 0x80) {
      s += static_cast<char>(c);
    } else if (c < 0x800) {
      s += static_cast<char>(0xC0 | (c >> 6));
      s += static_cast<char>(0x80 | (c & 0x3F));
    } else {
      s += static_cast<char>(0xE0 | (c >> 12));
      s += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
      s += static_cast<char>(0x80 | (c & 0x3F));
    }
  }
  bool string(std::string& out) {
    if (p >= end || *p != '"') return fail("expected a string");
    ++p;
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) return fail("truncated escape");
        switch (*p) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (end - p < 5) return fail("truncated \\u escape");
            unsigned c = 0;
            for (int i = 1; i <= 4; ++i) {
              const char h = p[i];
              c <<= 4;
              if (h >= '0' && h <= '9') c |= h - '0';
              else if (h >= 'a' && h <= 'f') c |= h - 'a' + 10;
              else if (h >= 'A' && h <= 'F') c |= h - 'A' + 10;
              else return fail("bad \\u escape");
            }
            put_utf8(out, c);
            p += 4;
            break;
          }
          default: return fail("bad escape");
        }
        ++p;
      } else {
        out += *p++;
      }
    }
    if (p >= end) return fail("unterminated string");
    ++p;
    return true;
  }
  bool value(JVal& v) {
    if (++depth > 64) return fail("nesting too deep");
    ws();
    if (p >= end) return fail("unexpected end of JSON");
    bool ok = true;
    if (*p == '{') {
      v.type = JVal::kObj;
      ++p;
      ws();
      if (p < end && *p == '}') {
        ++p;
      } else {
        while (ok) {
          ws();
          std::string k;
          if (!string(k)) return false;
          ws();
          if (p >= end || *p != ':') return fail("expected ':'");
          ++p;
          v.obj.emplace_back(std::move(k), JVal());
          if (!value(v.obj.back().second)) return false;
          ws();
          if (p < end && *p == ',') {
            ++p;
            continue;
          }
          if (p < end && *p == '}') {
            ++p;
            break;
          }
          return fail("expected ',' or '}'");
        }
      }
    } else if (*p == '[') {
      v.type = JVal::kArr;
      ++p;
      ws();
      if (p < end && *p == ']') {
        ++p;
      } else {
        while (true) {
          v.arr.emplace_back();
          if (!value(v.arr.back())) return false;
          ws();
          if (p < end && *p == ',') {
            ++p;
            continue;
          }
          if (p < end && *p == ']') {
            ++p;
            break;
          }
          return fail("expected ',' or ']'");
        }
      }
    } else if (*p == '"') {
      v.type = JVal::kStr;
      ok = string(v.str);
    } else if (end - p >= 4 && !strncmp(p, "true", 4)) {
      v.type = JVal::kBool;
      v.b = true;
      p += 4;
    } else if (end - p >= 5 && !strncmp(p, "false", 5)) {
      v.type = JVal::kBool;
      p += 5;
    } else if (end - p >= 4 && !strncmp(p, "null", 4)) {
      p += 4;
    } else if (*p == '-' || (*p >= '0' && *p <= '9')) {
      const char* q = p;
      while (q < end && (strchr("+-.eE", *q) || (*q >= '0' && *q <= '9'))) ++q;
      const std::string tok(p, q);
      char* e = nullptr;
      v.type = JVal::kNum;
      v.num = strtod(tok.c_str(), &e);
      if (!e || *e) return fail("bad number");
      p = q;
    } else {
      return fail("unexpected character");
    }
    --depth;
    return ok;
  }
};

bool parse_json(const char* data, size_t n, JVal& out, std::string& err) {
  Parser ps{data, data + n, {}};
  if (!ps.value(out)) {
    err = ps.err;
    return false;
  }
  ps.ws();
  if (ps.p != ps.end) {
    err = "trailing bytes after the JSON value";
    return false;
  }
  return true;
}

// ------------------------------------------------------------------ shards
struct Tensor {
  std::string dtype;
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  size_t file_offset = 0;
  std::string file;
};

int dtype_size(const std::string& d) {
  if (d == "BOOL" || d == "U8" || d == "I8" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  if (d == "U16" || d == "I16" || d == "F16" || d == "BF16") return 2;
  if (d == "U32" || d == "I32" || d == "F32") return 4;
  if (d == "U64" || d == "I64" || d == "F64") return 8;
  return 0;
}

struct Mapping {
  void* base = MAP_FAILED;
  size_t size = 0;
  ~Mapping() {
    if (base != MAP_FAILED) munmap(base, size);
  }
};

struct Store {
  std::vector<std::unique_ptr<Mapping>> maps;
  std::map<std::string, Tensor> tensors;  // later shards override earlier ones
  std::string err;

  bool fail(const std::string& e) {
    err = e;
    return false;
  }

  bool add_file(const std::string& path) {
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) return fail("cannot open " + path);
    struct stat sb {};
    if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
      close(fd);
      return fail(path + ": not a safetensors file (shorter than 8 bytes)");
    }
    auto m = std::make_unique<Mapping>();
    m->size = static_cast<size_t>(sb.st_size);
    m->base = mmap(nullptr, m->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m->base == MAP_FAILED) return fail("cannot map " + path);
    const auto* bytes = static_cast<const uint8_t*>(m->base);
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | bytes[i];
    if (hlen > m->size - 8) return fail(path + ": header length runs past the end of the file");
    JVal h;
    std::string jerr;
    if (!parse_json(reinterpret_cast<const char*>(bytes + 8), static_cast<size_t>(hlen), h, jerr))
      return fail(path + ": bad header JSON (" + jerr + ")");
    if (h.type != JVal::kObj) return fail(path + ": header is not a JSON object");
    const uint8_t* data = bytes + 8 + hlen;
    const size_t data_len = m->size - 8 - static_cast<size_t>(hlen);
    for (auto& kv : h.obj) {
      if (kv.first == "__metadata__") continue;
      const JVal& t = kv.second;
      const JVal* dt = t.get("dtype");
      const JVal* sh = t.get("shape");
      const JVal* off = t.get("data_offsets");
      if (t.type != JVal::kObj || !dt || dt->type != JVal::kStr || !sh || sh->type != JVal::kArr || !off ||
          off->type != JVal::kArr || off->arr.size() != 2)
        return fail(path + ": malformed entry for tensor " + kv.first);
      Tensor ten;
      ten.dtype = dt->str;
      const int es = dtype_size(ten.dtype);
      if (!es) return fail(path + ": tensor " + kv.first + " has unsupported dtype " + ten.dtype);
      uint64_t numel = 1;
      for (auto& d : sh->arr) {
        if (d.type != JVal::kNum || d.num < 0 || d.num != static_cast<double>(static_cast<int64_t>(d.num)))
          return fail(path + ": tensor " + kv.first + " has a bad shape");
        ten.shape.push_back(static_cast<int64_t>(d.num));
        numel *= static_cast<uint64_t>(d.num);
      }
      for (auto& o : off->arr)
        if (o.type != JVal::kNum || o.num < 0) return fail(path + ": tensor " + kv.first + " has bad data_offsets");
      const uint64_t b = static_cast<uint64_t>(off->arr[0].num), e = static_cast<uint64_t>(off->arr[1].num);
      if (b > e || e > data_len) return fail(path + ": tensor " + kv.first + " lies outside the data block");
      if (e - b != numel * static_cast<uint64_t>(es))
        return fail(path + ": tensor " + kv.first + " byte size does not match its shape and dtype");
      ten.data = data + b;
      ten.nbytes = static_cast<size_t>(e - b);
      ten.file_offset = 8 + static_cast<size_t>(hlen) + static_cast<size_t>(b);
      ten.file = path;
      tensors[kv.first] = std::move(ten);
    }
    maps.push_back(std::move(m));
    return true;
  }

  bool add_path(const std::string& path) {
    struct stat sb {};
    if (stat(path.c_str(), &sb) != 0) return fail("no such file or directory: " + path);
    if (!S_ISDIR(sb.st_mode)) return add_file(path);
    std::vector<std::string> names;
    const std::string index = path + "/model.safetensors.index.json";
    struct stat ib {};
    if (stat(index.c_str(), &ib) == 0) {
      std::string text;
      if (FILE* f = fopen(index.c_str(), "rb")) {
        text.resize(static_cast<size_t>(ib.st_size));
        const size_t got = fread(&text[0], 1, text.size(), f);
        fclose(f);
        text.resize(got);
      }
      JVal j;
      std::string jerr;
      if (!parse_json(text.data(), text.size(), j, jerr)) return fail(index + ": bad JSON (" + jerr + ")");
      const JVal* wm = j.get("weight_map");
      if (!wm || wm->type != JVal::kObj) return fail(index + ": no weight_map object");
      std::set<std::string> files;
      for (auto& kv : wm->obj)
        if (kv.second.type == JVal::kStr) files.insert(kv.second.str);
      names.assign(files.begin(), files.end());
    } else {
      if (DIR* dir = opendir(path.c_str())) {
        while (dirent* e = readdir(dir)) {
          const std::string n = e->d_name;
          if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) names.push_back(n);
        }
        closedir(dir);
      }
      std::sort(names.begin(), names.end());
    }
    if (names.empty()) return fail(path + ": no .safetensors shards");
    for (auto& n : names)
      if (!add_file(path + "/" + n)) return false;
    return true;
  }
};

// bf16 bits of a 2-byte float (BF16 as is, F16 when exactly representable),
// or false.
bool to_bf16(const Tensor& t, std::vector<uint16_t>& out, std::string& err, const std::string& name) {
  const size_t n = t.nbytes / dtype_size(t.dtype);
  out.resize(n);
  if (t.dtype == "BF16") {
    memcpy(out.data(), t.data, t.nbytes);
    return true;
  }
  for (size_t i = 0; i < n; ++i) {
    float f;
    if (t.dtype == "F32") {
      memcpy(&f, t.data + 4 * i, 4);
    } else if (t.dtype == "F16") {
      uint16_t h;
      memcpy(&h, t.data + 2 * i, 2);
      const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
      if (exp == 0x1F) {
        err = name + ": non-finite value";
        return false;
      }
      f = exp ? std::ldexp(static_cast<float>(man | 0x400u), static_cast<int>(exp) - 25)
              : std::ldexp(static_cast<float>(man), -24);
      if (sign) f = -f;
    } else {
      err = name + ": dtype " + t.dtype + " is not a float type";
      return false;
    }
    uint32_t u;
    memcpy(&u, &f, 4);
    if (u & 0xFFFFu) {
      err = name + ": value not representable in bf16 (the kernels take bf16 scales and biases)";
      return false;
    }
    out[i] = static_cast<uint16_t>(u >> 16);
  }
  return true;
}

bool to_f32(const Tensor& t, std::vector<float>& out, std::string& err, const std::string& name) {
  const size_t n = t.nbytes / dtype_size(t.dtype);
  out.resize(n);
  for (size_t i = 0; i < n; ++i) {
    if (t.dtype == "F32") {
      memcpy(&out[i], t.data + 4 * i, 4);
    } else if (t.dtype == "BF16") {
      uint16_t h;
      memcpy(&h, t.data + 2 * i, 2);
      const uint32_t u = static_cast<uint32_t>(h) << 16;
      memcpy(&out[i], &u, 4);
    } else if (t.dtype == "F16") {
      uint16_t h;
      memcpy(&h, t.data + 2 * i, 2);
      const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
      float f = exp == 0x1F ? (man ? NAN : INFINITY)
                            : (exp ? std::ldexp(static_cast<float>(man | 0x400u), static_cast<int>(exp) - 25)
                                   : std::ldexp(static_cast<float>(man), -24));
      out[i] = sign ? -f : f;
    } else {
      err = name + ": dtype " + t.dtype + " is not a float type";
      return false;
    }
  }
  return true;
}

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

}  // namespace
}  // namespace st
}  // namespace aex

extern "C" {

int aex_safetensors_scan(const char* path, char* out, size_t out_len) {
  using namespace aex::st;
  if (!path || !out || out_len == 0) return AEX_ERR_INVALID_ARG;
  Store store;
  std::string text;
  int rc = AEX_OK;
  if (!store.add_path(path)) {
    text = store.err;
    rc = AEX_ERR_INVALID_ARG;
  } else {
    for (auto& kv : store.tensors) {
      text += kv.first + " " + kv.second.dtype + " ";
      for (size_t i = 0; i < kv.second.shape.size(); ++i)
        text += (i ? "," : "") + std::to_string(kv.second.shape[i]);
      text += " " + std::to_string(kv.second.file_offset) + " " + std::to_string(kv.second.nbytes) + "\n";
    }
  }
  const size_t n = std::min(text.size(), out_len - 1);
  memcpy(out, text.data(), n);
  out[n] = '\0';
  return rc;
}

int aex_dit_load_safetensors(aex_dit* d, const char* path, int* n_linear, int* n_norm, aex_stream stream) {
  using namespace aex;
  using namespace aex::st;
  if (n_linear) *n_linear = 0;
  if (n_norm) *n_norm = 0;
  if (!d || !path) return set_error(nullptr, AEX_ERR_INVALID_ARG, "NULL argument");
  aex_ctx* ctx = dit_context(d);
  Store store;
  if (!store.add_path(path)) return set_error(ctx, AEX_ERR_INVALID_ARG, "%s", store.err.c_str());
  // Classify: quantized linears (U32 weight + scales + biases), norm weights (128 floats).
  std::vector<std::string> linears, norms;
  std::set<std::string> used;
  for (auto& kv : store.tensors) {
    const std::string& k = kv.first;
    if (!ends_with(k, ".weight")) continue;  // scales / biases are claimed by their weight below
    const std::string base = k.substr(0, k.size() - 7);
    if (kv.second.dtype == "U32") {
      linears.push_back(base);
      used.insert(k);
      used.insert(base + ".scales");
      used.insert(base + ".biases");
    } else if (kv.second.shape.size() == 1 && kv.second.shape[0] == 128 && dtype_size(kv.second.dtype) >= 2) {
      norms.push_back(base);
      used.insert(k);
    } else {
      return set_error(ctx, AEX_ERR_UNSUPPORTED, "unexpected tensor %s (%s, not a 4-bit linear or a norm weight)",
                       k.c_str(), kv.second.dtype.c_str());
    }
  }
  for (auto& kv : store.tensors)
    if (!used.count(kv.first))
      return set_error(ctx, AEX_ERR_UNSUPPORTED, "unexpected tensor %s (no matching .weight)", kv.first.c_str());
  if (int r = bind_device(ctx)) return r;
  auto s = static_cast<cudaStream_t>(stream);
  // One device staging buffer, reused in stream order (each load consumes it before the next copy).
  size_t need = 128 * sizeof(float);
  for (auto& b : linears) {
    auto it = store.tensors.find(b + ".scales");
    auto ib = store.tensors.find(b + ".biases");
    if (it == store.tensors.end() || ib == store.tensors.end())
      return set_error(ctx, AEX_ERR_INVALID_ARG, "quantized linear %s lacks .scales or .biases", b.c_str());
    const size_t groups = it->second.nbytes / dtype_size(it->second.dtype);
    need = std::max(need, ((store.tensors[b + ".weight"].nbytes + 255) & ~size_t(255)) + 4 * groups + 512);
  }
  uint8_t* stage = nullptr;
  AEX_CUDA_TRY(ctx, cudaMalloc(&stage, need));
  int rc = AEX_OK;
  std::vector<uint16_t> sc, bi;
  std::vector<float> nw;
  std::string err;
  for (auto& b : linears) {
    const Tensor& w = store.tensors[b + ".weight"];
    const Tensor& ts = store.tensors[b + ".scales"];
    const Tensor& tb = store.tensors[b + ".biases"];
    if (w.shape.size() != 2 || ts.shape.size() != 2 || tb.shape.size() != 2) {
      rc = set_error(ctx, AEX_ERR_INVALID_ARG, "%s: weight, scales and biases must be 2-D", b.c_str());
      break;
    }
    const int n = static_cast<int>(w.shape[0]), k = static_cast<int>(w.shape[1] * 8);
    if (ts.shape[0] != n || tb.shape[0] != n || ts.shape[1] * 64 != k || tb.shape[1] * 64 != k) {
      rc = set_error(ctx, AEX_ERR_INVALID_ARG, "%s: scales/biases [%lld, %lld] do not match weight [%d, k=%d] at group 64",
                     b.c_str(), static_cast<long long>(ts.shape[0]), static_cast<long long>(ts.shape[1]), n, k);
      break;
    }
    if (!to_bf16(ts, sc, err, b + ".scales") || !to_bf16(tb, bi, err, b + ".biases")) {
      rc = set_error(ctx, AEX_ERR_UNSUPPORTED, "%s", err.c_str());
      break;
    }
    const size_t wb = (w.nbytes + 255) & ~size_t(255);
    const size_t gb = sc.size() * 2;
    uint8_t* dw = stage;
    uint8_t* ds = stage + wb;
    uint8_t* db = stage + wb + ((gb + 255) & ~size_t(255));
    cudaError_t e = cudaMemcpyAsync(dw, w.data, w.nbytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ds, sc.data(), gb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(db, bi.data(), gb, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
      rc = cuda_error(ctx, e, "cudaMemcpyAsync(safetensors staging)");
      break;
    }
    rc = aex_dit_load_linear(d, b.c_str(), reinterpret_cast<const uint32_t*>(dw), reinterpret_cast<const uint16_t*>(ds),
                             reinterpret_cast<const uint16_t*>(db), n, k, stream);
    if (rc) break;
    if (n_linear) ++*n_linear;
  }
  for (size_t i = 0; !rc && i < norms.size(); ++i) {
    const std::string& b = norms[i];
    if (!to_f32(store.tensors[b + ".weight"], nw, err, b + ".weight")) {
      rc = set_error(ctx, AEX_ERR_UNSUPPORTED, "%s", err.c_str());
      break;
    }
    cudaError_t e = cudaMemcpyAsync(stage, nw.data(), 128 * sizeof(float), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
      rc = cuda_error(ctx, e, "cudaMemcpyAsync(safetensors staging)");
      break;
    }
    rc = aex_dit_load_norm(d, b.c_str(), reinterpret_cast<const float*>(stage), stream);
    if (!rc && n_norm) ++*n_norm;
  }
  // The staging buffer is read by kernels still in the stream: wait for them before freeing it.
  const cudaError_t se = cudaStreamSynchronize(s);
  cudaFree(stage);
  if (!rc && se != cudaSuccess) rc = cuda_error(ctx, se, "cudaStreamSynchronize(safetensors load)");
  return rc;
}

}  // extern "C"
