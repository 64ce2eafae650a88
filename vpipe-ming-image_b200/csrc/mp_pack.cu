// Pack I/O of the C-ABI (host code only; no device work here except the
// weight upload it hands to mp_weight_upload):
//   * a safetensors reader over one file or a directory of shards (the
//     checkpoint and pack files the reference reads through its WeightSet):
//     the files are memory-mapped, the JSON header parsed into a tensor index;
//   * mp_pack_upload: one projection from an open pack, detected as the
//     reference's load_qw_ does (src/ming-dit.cc:802-831, :1115-1135): packed
//     when `<name>.scales` sits beside `<name>.weight`, bits from the shapes
//     (codes [N, K*bits/32] U32, scales / biases [N, K/64]), scales and
//     biases narrowed to bf16; dense bf16 otherwise;
//   * mp_pack_quantize: a w8 / w4 pack writer with the reference's selection
//     (src/ming-quant-family.cc:31-59, pinned by tests/ming-quant-test.cc:
//     507-549): every 2-D float `.weight` whose leaf is not a norm or an
//     embedding and whose width is a multiple of 64, except the model-level
//     all_x_embedder / cap_embedder / t_embedder. / all_final_layer; each
//     becomes codes + bf16 scales + bf16 biases (per 64-wide K group:
//     scale = max((hi - lo) / (2^bits - 1), 1e-8), bias = lo, both rounded to
//     bf16, q = round-half-even((w - bias) / scale) clamped to [0, 2^bits - 1],
//     codes packed LSB first), everything else copied unchanged. For a
//     directory, every shard is written under the same name and config.json
//     gains a "quantization" block {bits, group_size}.
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/mingproj.h"

namespace {

constexpr int kGroup = 64;

// ---- minimal JSON (the safetensors header) ---------------------------------

struct JValue {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  double num = 0.0;
  bool b = false;
  std::string str;
  std::vector<JValue> arr;
  std::vector<std::pair<std::string, JValue>> obj;
  const JValue* get(const std::string& k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

class JParser {
 public:
  JParser(const char* s, size_t n) : p_(s), e_(s + n) {}
  bool parse(JValue* v) {
    if (!value(v, 0)) return false;
    ws();
    return p_ == e_ || *p_ == '\0';
  }

 private:
  const char* p_;
  const char* e_;
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool lit(const char* w) {
    const size_t n = std::strlen(w);
    if (static_cast<size_t>(e_ - p_) < n || std::strncmp(p_, w, n) != 0) return false;
    p_ += n;
    return true;
  }
  bool string(std::string* out) {
    if (p_ >= e_ || *p_ != '"') return false;
    ++p_;
    out->clear();
    while (p_ < e_ && *p_ != '"') {
      char c = *p_++;
      if (c == '\\') {
        if (p_ >= e_) return false;
        const char x = *p_++;
        switch (x) {
          case '"': out->push_back('"'); break;
          case '\\': out->push_back('\\'); break;
          case '/': out->push_back('/'); break;
          case 'b': out->push_back('\b'); break;
          case 'f': out->push_back('\f'); break;
          case 'n': out->push_back('\n'); break;
          case 'r': out->push_back('\r'); break;
          case 't': out->push_back('\t'); break;
          case 'u': {
            if (e_ - p_ < 4) return false;
            unsigned cp = 0;
            for (int i = 0; i < 4; ++i) {
              const char h = *p_++;
              cp <<= 4;
              if (h >= '0' && h <= '9') cp |= static_cast<unsigned>(h - '0');
              else if (h >= 'a' && h <= 'f') cp |= static_cast<unsigned>(h - 'a' + 10);
              else if (h >= 'A' && h <= 'F') cp |= static_cast<unsigned>(h - 'A' + 10);
              else return false;
            }
            // UTF-8 of the code point (names here are ASCII; kept for metadata)
            if (cp < 0x80) {
              out->push_back(static_cast<char>(cp));
            } else if (cp < 0x800) {
              out->push_back(static_cast<char>(0xC0 | (cp >> 6)));
              out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
            } else {
              out->push_back(static_cast<char>(0xE0 | (cp >> 12)));
              out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
              out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
            }
            break;
          }
          default: return false;
        }
      } else {
        out->push_back(c);
      }
    }
    if (p_ >= e_) return false;
    ++p_;
    return true;
  }
  bool value(JValue* v, int depth) {
    if (depth > 64) return false;
    ws();
    if (p_ >= e_) return false;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v->kind = JValue::kObj;
      ws();
      if (p_ < e_ && *p_ == '}') {
        ++p_;
        return true;
      }
      while (true) {
        ws();
        std::string k;
        if (!string(&k)) return false;
        ws();
        if (p_ >= e_ || *p_ != ':') return false;
        ++p_;
        JValue x;
        if (!value(&x, depth + 1)) return false;
        v->obj.emplace_back(std::move(k), std::move(x));
        ws();
        if (p_ < e_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < e_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '[') {
      ++p_;
      v->kind = JValue::kArr;
      ws();
      if (p_ < e_ && *p_ == ']') {
        ++p_;
        return true;
      }
      while (true) {
        JValue x;
        if (!value(&x, depth + 1)) return false;
        v->arr.push_back(std::move(x));
        ws();
        if (p_ < e_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < e_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '"') {
      v->kind = JValue::kStr;
      return string(&v->str);
    }
    if (lit("true")) {
      v->kind = JValue::kBool;
      v->b = true;
      return true;
    }
    if (lit("false")) {
      v->kind = JValue::kBool;
      return true;
    }
    if (lit("null")) return true;
    // number
    const char* s = p_;
    if (p_ < e_ && (*p_ == '-' || *p_ == '+')) ++p_;
    while (p_ < e_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                       *p_ == '-' || *p_ == '+'))
      ++p_;
    if (p_ == s) return false;
    v->kind = JValue::kNum;
    v->num = std::strtod(std::string(s, p_).c_str(), nullptr);
    return true;
  }
};

std::string json_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '"' || c == '\\') {
      o.push_back('\\');
      o.push_back(c);
    } else if (static_cast<unsigned char>(c) < 0x20) {
      char buf[8];
      std::snprintf(buf, sizeof(buf), "\\u%04x", static_cast<unsigned>(c));
      o += buf;
    } else {
      o.push_back(c);
    }
  }
  return o;
}

// ---- files -----------------------------------------------------------------

struct MappedFile {
  std::string path;
  const uint8_t* base = nullptr;
  size_t size = 0;
  ~MappedFile() {
    if (base != nullptr) munmap(const_cast<uint8_t*>(base), size);
  }
};

struct Tensor {
  std::string name;
  std::string dtype;
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t bytes = 0;
};

int dtype_size(const std::string& dt) {
  if (dt == "BF16" || dt == "F16" || dt == "I16" || dt == "U16") return 2;
  if (dt == "F32" || dt == "I32" || dt == "U32") return 4;
  if (dt == "F64" || dt == "I64" || dt == "U64") return 8;
  if (dt == "U8" || dt == "I8" || dt == "BOOL" || dt == "F8_E4M3" || dt == "F8_E5M2") return 1;
  return 0;
}

bool is_dir(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}

bool ends_with(const std::string& s, const std::string& t) {
  return s.size() >= t.size() && s.compare(s.size() - t.size(), t.size(), t) == 0;
}

std::vector<std::string> shard_names(const std::string& dir) {
  std::vector<std::string> out;
  DIR* d = opendir(dir.c_str());
  if (d == nullptr) return out;
  while (dirent* e = readdir(d)) {
    const std::string n = e->d_name;
    if (ends_with(n, ".safetensors")) out.push_back(n);
  }
  closedir(d);
  std::sort(out.begin(), out.end());
  return out;
}

// bf16 <-> f32 (round to nearest, ties to even; NaN kept quiet)
uint16_t f32_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
  return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}
float bf16_to_f32(uint16_t b) {
  const uint32_t u = static_cast<uint32_t>(b) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
float f16_to_f32(uint16_t h) {
  const uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  float v;
  if (e == 0) v = std::ldexp(static_cast<float>(m), -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp(static_cast<float>(m | 0x400u), static_cast<int>(e) - 25);
  return s ? -v : v;
}

// one element of a float tensor as f32
bool element_f32(const Tensor& t, size_t i, float* out) {
  if (t.dtype == "BF16") {
    uint16_t b;
    std::memcpy(&b, t.data + 2 * i, 2);
    *out = bf16_to_f32(b);
  } else if (t.dtype == "F16") {
    uint16_t h;
    std::memcpy(&h, t.data + 2 * i, 2);
    *out = f16_to_f32(h);
  } else if (t.dtype == "F32") {
    std::memcpy(out, t.data + 4 * i, 4);
  } else if (t.dtype == "F64") {
    double d;
    std::memcpy(&d, t.data + 8 * i, 8);
    *out = static_cast<float>(d);
  } else {
    return false;
  }
  return true;
}

bool is_float(const std::string& dt) {
  return dt == "BF16" || dt == "F16" || dt == "F32" || dt == "F64";
}

}  // namespace

struct mp_pack {
  std::vector<std::unique_ptr<MappedFile>> files;
  std::vector<Tensor> tensors;
  std::map<std::string, size_t> index;
  std::map<std::string, std::string> metadata;
  std::string error;
};

namespace {

int pack_fail(mp_pack* p, int status, const char* fmt, ...) {
  if (p != nullptr) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    p->error = buf;
  }
  return status;
}

int map_one(mp_pack* p, const std::string& path) {
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return pack_fail(p, MP_EINVAL, "cannot open %s", path.c_str());
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 8) {
    close(fd);
    return pack_fail(p, MP_EINVAL, "%s: not a safetensors file (too short)", path.c_str());
  }
  const size_t size = static_cast<size_t>(st.st_size);
  void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) return pack_fail(p, MP_ENOMEM, "%s: mmap failed", path.c_str());
  auto f = std::make_unique<MappedFile>();
  f->path = path;
  f->base = static_cast<const uint8_t*>(m);
  f->size = size;
  uint64_t hlen;
  std::memcpy(&hlen, f->base, 8);
  if (hlen > size - 8)
    return pack_fail(p, MP_EINVAL, "%s: header length %llu past the end", path.c_str(),
                     static_cast<unsigned long long>(hlen));
  JValue hdr;
  JParser jp(reinterpret_cast<const char*>(f->base + 8), static_cast<size_t>(hlen));
  if (!jp.parse(&hdr) || hdr.kind != JValue::kObj)
    return pack_fail(p, MP_EINVAL, "%s: the header is not a JSON object", path.c_str());
  const uint8_t* data = f->base + 8 + hlen;
  const size_t data_size = size - 8 - static_cast<size_t>(hlen);
  for (const auto& kv : hdr.obj) {
    if (kv.first == "__metadata__") {
      for (const auto& m2 : kv.second.obj)
        if (m2.second.kind == JValue::kStr) p->metadata[m2.first] = m2.second.str;
      continue;
    }
    const JValue* dt = kv.second.get("dtype");
    const JValue* sh = kv.second.get("shape");
    const JValue* off = kv.second.get("data_offsets");
    if (dt == nullptr || dt->kind != JValue::kStr || sh == nullptr || sh->kind != JValue::kArr ||
        off == nullptr || off->kind != JValue::kArr || off->arr.size() != 2)
      return pack_fail(p, MP_EINVAL, "%s: bad entry for %s", path.c_str(), kv.first.c_str());
    Tensor t;
    t.name = kv.first;
    t.dtype = dt->str;
    int64_t elems = 1;
    for (const auto& d : sh->arr) {
      if (d.kind != JValue::kNum || d.num < 0)
        return pack_fail(p, MP_EINVAL, "%s: bad shape for %s", path.c_str(), t.name.c_str());
      t.shape.push_back(static_cast<int64_t>(d.num));
      elems *= static_cast<int64_t>(d.num);
    }
    const double a = off->arr[0].num, b = off->arr[1].num;
    if (a < 0 || b < a || static_cast<size_t>(b) > data_size)
      return pack_fail(p, MP_EINVAL, "%s: data offsets of %s out of range", path.c_str(),
                       t.name.c_str());
    t.data = data + static_cast<size_t>(a);
    t.bytes = static_cast<size_t>(b - a);
    const int es = dtype_size(t.dtype);
    if (es > 0 && static_cast<size_t>(elems) * static_cast<size_t>(es) != t.bytes)
      return pack_fail(p, MP_EINVAL, "%s: %s holds %zu bytes for %lld elements of %s",
                       path.c_str(), t.name.c_str(), t.bytes, static_cast<long long>(elems),
                       t.dtype.c_str());
    if (p->index.count(t.name) != 0)
      return pack_fail(p, MP_EINVAL, "%s: tensor %s appears twice", path.c_str(), t.name.c_str());
    p->index[t.name] = p->tensors.size();
    p->tensors.push_back(std::move(t));
  }
  p->files.push_back(std::move(f));
  return MP_OK;
}

const Tensor* find(const mp_pack* p, const std::string& name) {
  auto it = p->index.find(name);
  return it == p->index.end() ? nullptr : &p->tensors[it->second];
}

void fill_info(const Tensor& t, mp_tensor_info* info) {
  std::memset(info, 0, sizeof(*info));
  info->name = t.name.c_str();
  info->dtype = t.dtype.c_str();
  info->ndim = static_cast<int32_t>(std::min<size_t>(t.shape.size(), 8));
  for (int i = 0; i < info->ndim; ++i) info->shape[i] = t.shape[i];
  info->data = t.data;
  info->bytes = t.bytes;
}

// The reference's selection (src/ming-quant-family.cc:31-59).
bool selected(const Tensor& t) {
  if (!ends_with(t.name, ".weight") || t.shape.size() != 2 || !is_float(t.dtype)) return false;
  const std::string base = t.name.substr(0, t.name.size() - 7);
  const size_t dot = base.rfind('.');
  const std::string leaf = dot == std::string::npos ? base : base.substr(dot + 1);
  if (leaf.find("norm") != std::string::npos || leaf.find("embed") != std::string::npos) return false;
  for (const char* ex : {"all_x_embedder", "cap_embedder", "t_embedder.", "all_final_layer"})
    if (t.name.find(ex) != std::string::npos) return false;
  return t.shape[1] % kGroup == 0 && t.shape[1] > 0;
}

// Affine quantization of one [n, k] float tensor (see the file comment).
void quantize(const Tensor& t, int bits, std::vector<uint32_t>* codes, std::vector<uint16_t>* sc,
              std::vector<uint16_t>* bi) {
  const int64_t n = t.shape[0], k = t.shape[1], groups = k / kGroup;
  const int qmax = (1 << bits) - 1;
  const int per = 32 / bits;
  codes->assign(static_cast<size_t>(n * (k / per)), 0u);
  sc->resize(static_cast<size_t>(n * groups));
  bi->resize(static_cast<size_t>(n * groups));
  std::vector<float> g(kGroup);
  for (int64_t r = 0; r < n; ++r) {
    for (int64_t gi = 0; gi < groups; ++gi) {
      float lo = INFINITY, hi = -INFINITY;
      for (int e = 0; e < kGroup; ++e) {
        element_f32(t, static_cast<size_t>(r * k + gi * kGroup + e), &g[e]);
        lo = std::min(lo, g[e]);
        hi = std::max(hi, g[e]);
      }
      const float scale = std::max((hi - lo) / static_cast<float>(qmax), 1e-8f);
      const uint16_t sb = f32_to_bf16(scale), bb = f32_to_bf16(lo);
      (*sc)[static_cast<size_t>(r * groups + gi)] = sb;
      (*bi)[static_cast<size_t>(r * groups + gi)] = bb;
      const float s32 = bf16_to_f32(sb), b32 = bf16_to_f32(bb);
      for (int e = 0; e < kGroup; ++e) {
        float q = std::nearbyint((g[e] - b32) / s32);  // round half to even
        q = std::min(std::max(q, 0.0f), static_cast<float>(qmax));
        const int64_t col = gi * kGroup + e;
        const uint32_t code = static_cast<uint32_t>(q);
        (*codes)[static_cast<size_t>(r * (k / per) + col / per)] |=
            code << (bits * static_cast<int>(col % per));
      }
    }
  }
}

struct OutTensor {
  std::string name, dtype;
  std::vector<int64_t> shape;
  const uint8_t* src = nullptr;   // unchanged bytes, or
  std::vector<uint8_t> own;       // new bytes
  size_t bytes() const { return src != nullptr ? src_bytes : own.size(); }
  size_t src_bytes = 0;
};

int write_file(mp_pack* p, const std::string& path, const std::vector<OutTensor>& ts,
               const std::map<std::string, std::string>& meta) {
  std::ostringstream h;
  h << "{";
  size_t off = 0;
  bool first = true;
  if (!meta.empty()) {
    h << "\"__metadata__\":{";
    bool f2 = true;
    for (const auto& kv : meta) {
      h << (f2 ? "" : ",") << "\"" << json_escape(kv.first) << "\":\"" << json_escape(kv.second)
        << "\"";
      f2 = false;
    }
    h << "}";
    first = false;
  }
  for (const auto& t : ts) {
    h << (first ? "" : ",") << "\"" << json_escape(t.name) << "\":{\"dtype\":\"" << t.dtype
      << "\",\"shape\":[";
    for (size_t i = 0; i < t.shape.size(); ++i) h << (i ? "," : "") << t.shape[i];
    h << "],\"data_offsets\":[" << off << "," << off + t.bytes() << "]}";
    off += t.bytes();
    first = false;
  }
  h << "}";
  std::string hs = h.str();
  while (hs.size() % 8 != 0) hs.push_back(' ');
  FILE* f = std::fopen(path.c_str(), "wb");
  if (f == nullptr) return pack_fail(p, MP_EINVAL, "cannot write %s", path.c_str());
  const uint64_t hlen = hs.size();
  bool ok = std::fwrite(&hlen, 8, 1, f) == 1 && std::fwrite(hs.data(), 1, hs.size(), f) == hs.size();
  for (const auto& t : ts) {
    if (!ok) break;
    const size_t nb = t.bytes();
    if (nb == 0) continue;
    ok = std::fwrite(t.src != nullptr ? t.src : t.own.data(), 1, nb, f) == nb;
  }
  ok = (std::fclose(f) == 0) && ok;
  return ok ? MP_OK : pack_fail(p, MP_EINVAL, "writing %s failed", path.c_str());
}

int quantize_one(mp_pack* log, const std::string& src, const std::string& dst, int bits,
                 int* n_quant, int* n_kept) {
  mp_pack in;
  int rc = map_one(&in, src);
  if (rc != MP_OK) return pack_fail(log, rc, "%s", in.error.c_str());
  std::vector<OutTensor> out;
  for (const Tensor& t : in.tensors) {
    if (selected(t)) {
      std::vector<uint32_t> codes;
      std::vector<uint16_t> sc, bi;
      quantize(t, bits, &codes, &sc, &bi);
      const std::string base = t.name.substr(0, t.name.size() - 7);
      const int64_t n = t.shape[0], k = t.shape[1];
      OutTensor c, s, b;
      c.name = t.name;
      c.dtype = "U32";
      c.shape = {n, k * bits / 32};
      c.own.resize(codes.size() * 4);
      std::memcpy(c.own.data(), codes.data(), c.own.size());
      s.name = base + ".scales";
      s.dtype = "BF16";
      s.shape = {n, k / kGroup};
      s.own.resize(sc.size() * 2);
      std::memcpy(s.own.data(), sc.data(), s.own.size());
      b.name = base + ".biases";
      b.dtype = "BF16";
      b.shape = {n, k / kGroup};
      b.own.resize(bi.size() * 2);
      std::memcpy(b.own.data(), bi.data(), b.own.size());
      out.push_back(std::move(c));
      out.push_back(std::move(s));
      out.push_back(std::move(b));
      ++*n_quant;
    } else {
      OutTensor o;
      o.name = t.name;
      o.dtype = t.dtype;
      o.shape = t.shape;
      o.src = t.data;
      o.src_bytes = t.bytes;
      out.push_back(std::move(o));
      ++*n_kept;
    }
  }
  return write_file(log, dst, out, in.metadata);
}

thread_local std::string g_pack_error;  // why the last mp_pack_open / mp_pack_quantize failed

}  // namespace

extern "C" {

int mp_pack_open(const char* path, mp_pack** out) {
  if (path == nullptr || out == nullptr) return MP_EINVAL;
  *out = nullptr;
  g_pack_error.clear();
  auto p = std::make_unique<mp_pack>();
  const std::string root = path;
  int rc;
  if (is_dir(root)) {
    const auto names = shard_names(root);
    if (names.empty()) {
      g_pack_error = root + ": no .safetensors files";
      return MP_EINVAL;
    }
    for (const auto& n : names) {
      rc = map_one(p.get(), root + "/" + n);
      if (rc != MP_OK) {
        g_pack_error = p->error;
        return rc;
      }
    }
  } else {
    rc = map_one(p.get(), root);
    if (rc != MP_OK) {
      g_pack_error = p->error;
      return rc;
    }
  }
  *out = p.release();
  return MP_OK;
}

const char* mp_pack_last_error(void) { return g_pack_error.c_str(); }

int mp_pack_close(mp_pack* p) {
  delete p;
  return MP_OK;
}

int mp_pack_count(const mp_pack* p) {
  return p == nullptr ? -1 : static_cast<int>(p->tensors.size());
}

int mp_pack_tensor_at(const mp_pack* p, int i, mp_tensor_info* info) {
  if (p == nullptr || info == nullptr || i < 0 || i >= static_cast<int>(p->tensors.size()))
    return MP_EINVAL;
  fill_info(p->tensors[static_cast<size_t>(i)], info);
  return MP_OK;
}

int mp_pack_find(const mp_pack* p, const char* name, mp_tensor_info* info) {
  if (p == nullptr || name == nullptr || info == nullptr) return MP_EINVAL;
  const Tensor* t = find(p, name);
  if (t == nullptr) return MP_EINVAL;
  fill_info(*t, info);
  return MP_OK;
}

const char* mp_pack_metadata(const mp_pack* p, const char* key) {
  if (p == nullptr || key == nullptr) return nullptr;
  auto it = p->metadata.find(key);
  return it == p->metadata.end() ? nullptr : it->second.c_str();
}

const char* mp_pack_error(const mp_pack* p) {
  return p == nullptr ? "" : p->error.c_str();
}

int mp_pack_upload(mp_ctx* ctx, const mp_pack* p, const char* base, mp_weight** out) {
  if (ctx == nullptr || p == nullptr || base == nullptr || out == nullptr) return MP_EINVAL;
  const std::string b = base;
  const Tensor* w = find(p, b + ".weight");
  if (w == nullptr) w = find(p, b);
  if (w == nullptr || w->shape.size() != 2) return MP_EINVAL;
  const Tensor* sc = find(p, b + ".scales");
  mp_weight_desc d;
  std::memset(&d, 0, sizeof(d));
  d.group = kGroup;
  if (sc != nullptr) {
    // a pack: K from the scales (group 64), bits from the codes' width
    if (w->dtype != "U32" || sc->shape.size() != 2 || sc->shape[0] != w->shape[0]) return MP_EINVAL;
    const int64_t n = w->shape[0], k = sc->shape[1] * kGroup;
    const int64_t bits = k > 0 ? w->shape[1] * 32 / k : 0;
    if (bits != 4 && bits != 8) return MP_EINVAL;
    const Tensor* bi = find(p, b + ".biases");
    d.n = static_cast<int32_t>(n);
    d.k = static_cast<int32_t>(k);
    d.bits = static_cast<int32_t>(bits);
    d.mode = bi != nullptr ? MP_QUANT_AFFINE : MP_QUANT_SYMMETRIC;
    if (d.mode == MP_QUANT_SYMMETRIC && bits != 8) return MP_EINVAL;
    // scales / biases narrowed to bf16 (load_qw_ narrows them, src/ming-dit.cc:816-822)
    auto narrow = [](const Tensor* t, std::vector<uint16_t>* v) -> bool {
      const size_t cnt = static_cast<size_t>(t->shape[0] * t->shape[1]);
      v->resize(cnt);
      if (t->dtype == "BF16") {
        std::memcpy(v->data(), t->data, cnt * 2);
        return true;
      }
      for (size_t i = 0; i < cnt; ++i) {
        float f;
        if (!element_f32(*t, i, &f)) return false;
        (*v)[i] = f32_to_bf16(f);
      }
      return true;
    };
    std::vector<uint16_t> s16, b16;
    if (!narrow(sc, &s16)) return MP_EINVAL;
    if (bi != nullptr && (bi->shape != sc->shape || !narrow(bi, &b16))) return MP_EINVAL;
    return mp_weight_upload(ctx, &d, w->data, s16.data(), bi != nullptr ? b16.data() : nullptr, out);
  }
  // dense: bf16 as stored, or narrowed to bf16
  if (!is_float(w->dtype)) return MP_EINVAL;
  d.n = static_cast<int32_t>(w->shape[0]);
  d.k = static_cast<int32_t>(w->shape[1]);
  d.bits = 0;
  d.mode = MP_QUANT_AFFINE;
  if (w->dtype == "BF16") return mp_weight_upload(ctx, &d, w->data, nullptr, nullptr, out);
  std::vector<uint16_t> v(static_cast<size_t>(w->shape[0] * w->shape[1]));
  for (size_t i = 0; i < v.size(); ++i) {
    float f;
    element_f32(*w, i, &f);
    v[i] = f32_to_bf16(f);
  }
  return mp_weight_upload(ctx, &d, v.data(), nullptr, nullptr, out);
}

int mp_pack_quantize(const char* src, const char* dst, int bits, int* n_quantized, int* n_kept) {
  if (src == nullptr || dst == nullptr || (bits != 4 && bits != 8)) return MP_EINVAL;
  int nq = 0, nk = 0;
  mp_pack log;
  g_pack_error.clear();
  struct Report {
    mp_pack* l;
    ~Report() { g_pack_error = l->error; }
  } report{&log};
  const std::string s = src, d = dst;
  int rc = MP_OK;
  if (is_dir(s)) {
    const auto names = shard_names(s);
    if (names.empty()) return MP_EINVAL;
    if (!is_dir(d) && mkdir(d.c_str(), 0755) != 0) return MP_EINVAL;
    for (const auto& n : names) {
      rc = quantize_one(&log, s + "/" + n, d + "/" + n, bits, &nq, &nk);
      if (rc != MP_OK) return rc;
    }
    // config.json: the source's keys plus a "quantization" block
    std::ifstream cin(s + "/config.json");
    if (cin) {
      std::string text((std::istreambuf_iterator<char>(cin)), std::istreambuf_iterator<char>());
      JValue cfg;
      JParser jp(text.data(), text.size());
      if (!jp.parse(&cfg) || cfg.kind != JValue::kObj) return MP_EINVAL;
      const size_t close = text.rfind('}');
      const bool empty = cfg.obj.empty();
      std::string q = std::string(empty ? "" : ",") + "\n  \"quantization\": {\"bits\": " +
                      std::to_string(bits) + ", \"group_size\": " + std::to_string(kGroup) + "}\n";
      if (cfg.get("quantization") == nullptr) text.insert(close, q);
      std::ofstream cout(d + "/config.json");
      cout << text;
      if (!cout) return MP_EINVAL;
    }
  } else {
    rc = quantize_one(&log, s, d, bits, &nq, &nk);
    if (rc != MP_OK) return rc;
  }
  if (n_quantized != nullptr) *n_quantized = nq;
  if (n_kept != nullptr) *n_kept = nk;
  return MP_OK;
}

}  // extern "C"
