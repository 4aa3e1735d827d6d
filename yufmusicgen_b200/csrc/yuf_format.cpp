// Reader of the .yuf checkpoint container (format of
// vulkan/scripts/export_checkpoint.py:47-146, read by vulkan/src/checkpoint.rs:90-149):
//   "YUFM" | version u32 LE (= 1) | header_len u64 LE | JSON header | f32 LE blob
// The header's "model_config" gives the architecture and "tensors" lists
// {name, shape, offset (in floats into the blob), count}.  A tied lm_head is
// absent (the engine reuses token_embedding.weight).  The low-rank width is read
// from the w1 tensor's shape, so checkpoints written with either rounding rule
// of the low-rank width load correctly.

#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/yufb200.h"

namespace yuf {
void set_error(const char* fmt, ...);
struct HostTensor {
  const float* p;
  int64_t n;
};
yuf_status_t model_create_from_map(const yuf_model_config* cfg, int precision, int device,
                                   const std::unordered_map<std::string, HostTensor>& t,
                                   yuf_model** out);

// Minimal JSON value (objects, arrays, strings, numbers, bools, null).
struct JVal {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<JVal> arr;
  std::map<std::string, JVal> obj;
  const JVal* get(const char* k) const {
    if (kind != OBJ) return nullptr;
    auto it = obj.find(k);
    return it == obj.end() ? nullptr : &it->second;
  }
};

struct JParser {
  const char* p;
  const char* end;
  bool ok = true;
  void ws() { while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
  bool lit(const char* s) {
    size_t n = std::strlen(s);
    if ((size_t)(end - p) >= n && std::strncmp(p, s, n) == 0) { p += n; return true; }
    return false;
  }
  static void utf8(std::string& o, unsigned cp) {
    if (cp < 0x80) o += (char)cp;
    else if (cp < 0x800) { o += (char)(0xC0 | (cp >> 6)); o += (char)(0x80 | (cp & 0x3F)); }
    else if (cp < 0x10000) { o += (char)(0xE0 | (cp >> 12)); o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F)); }
    else { o += (char)(0xF0 | (cp >> 18)); o += (char)(0x80 | ((cp >> 12) & 0x3F)); o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F)); }
  }
  unsigned hex4() {
    unsigned v = 0;
    for (int i = 0; i < 4; ++i) {
      if (p >= end) { ok = false; return 0; }
      char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else { ok = false; return 0; }
    }
    return v;
  }
  bool string(std::string& o) {
    if (p >= end || *p != '"') return ok = false;
    ++p;
    while (p < end && *p != '"') {
      char c = *p++;
      if (c != '\\') { o += c; continue; }
      if (p >= end) return ok = false;
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
          unsigned cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00 && p + 1 < end && p[0] == '\\' && p[1] == 'u') {
            p += 2;
            unsigned lo = hex4();
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(o, cp);
          break;
        }
        default: return ok = false;
      }
    }
    if (p >= end) return ok = false;
    ++p;
    return true;
  }
  bool value(JVal& v, int depth = 0) {
    if (depth > 64) return ok = false;
    ws();
    if (p >= end) return ok = false;
    if (*p == '{') {
      ++p; v.kind = JVal::OBJ; ws();
      if (p < end && *p == '}') { ++p; return true; }
      while (ok) {
        ws(); std::string k;
        if (!string(k)) return false;
        ws(); if (p >= end || *p != ':') return ok = false;
        ++p;
        if (!value(v.obj[k], depth + 1)) return false;
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == '}') { ++p; return true; }
        return ok = false;
      }
      return false;
    }
    if (*p == '[') {
      ++p; v.kind = JVal::ARR; ws();
      if (p < end && *p == ']') { ++p; return true; }
      while (ok) {
        v.arr.emplace_back();
        if (!value(v.arr.back(), depth + 1)) return false;
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == ']') { ++p; return true; }
        return ok = false;
      }
      return false;
    }
    if (*p == '"') { v.kind = JVal::STR; return string(v.str); }
    if (lit("true")) { v.kind = JVal::BOOL; v.b = true; return true; }
    if (lit("false")) { v.kind = JVal::BOOL; v.b = false; return true; }
    if (lit("null")) { v.kind = JVal::NUL; return true; }
    char* q = nullptr;
    std::string tmp(p, std::min<size_t>(64, end - p));
    v.num = std::strtod(tmp.c_str(), &q);
    if (q == tmp.c_str()) return ok = false;
    p += (q - tmp.c_str());
    v.kind = JVal::NUM;
    return true;
  }
};

static yuf_status_t fail(yuf_status_t st, const char* msg, const char* path) {
  set_error("yuf: %s (%s)", msg, path);
  return st;
}

}  // namespace yuf

using namespace yuf;

extern "C" yuf_status_t yuf_model_create_from_yuf(const char* path, int precision, int device,
                                                  yuf_model** out) {
  if (!path || !out) { set_error("yuf: null argument"); return YUF_ERR_INVALID_ARGUMENT; }
  std::unique_ptr<FILE, int (*)(FILE*)> f(std::fopen(path, "rb"), &std::fclose);
  if (!f) return fail(YUF_ERR_IO, "cannot open file", path);
  char magic[4];
  uint32_t version = 0;
  uint64_t hlen = 0;
  if (std::fread(magic, 1, 4, f.get()) != 4 || std::memcmp(magic, "YUFM", 4) != 0)
    return fail(YUF_ERR_IO, "bad magic (expected YUFM)", path);
  if (std::fread(&version, 4, 1, f.get()) != 1 || version != 1)
    return fail(YUF_ERR_UNSUPPORTED, "unsupported container version (expected 1)", path);
  if (std::fread(&hlen, 8, 1, f.get()) != 1 || hlen == 0 || hlen > (1ull << 31))
    return fail(YUF_ERR_IO, "bad header length", path);
  std::string header(hlen, '\0');
  if (std::fread(&header[0], 1, hlen, f.get()) != hlen) return fail(YUF_ERR_IO, "truncated header", path);
  JVal root;
  JParser jp{header.data(), header.data() + header.size()};
  if (!jp.value(root) || !jp.ok || root.kind != JVal::OBJ) return fail(YUF_ERR_IO, "header is not valid JSON", path);
  const JVal* mc = root.get("model_config");
  const JVal* tensors = root.get("tensors");
  if (!mc || mc->kind != JVal::OBJ || !tensors || tensors->kind != JVal::ARR)
    return fail(YUF_ERR_IO, "header lacks model_config or tensors", path);
  auto geti = [&](const char* k, int& o) {
    const JVal* v = mc->get(k);
    if (!v || v->kind != JVal::NUM) return false;
    o = (int)v->num;
    return true;
  };
  yuf_model_config cfg{};
  if (!geti("vocab_size", cfg.vocab_size) || !geti("d_model", cfg.d_model) ||
      !geti("n_layers", cfg.n_layers) || !geti("n_heads", cfg.n_heads) ||
      !geti("head_size", cfg.head_size) || !geti("rosa_size", cfg.rosa_size))
    return fail(YUF_ERR_IO, "model_config lacks a size field", path);
  // blob
  const long blob_start = std::ftell(f.get());
  std::fseek(f.get(), 0, SEEK_END);
  const long file_end = std::ftell(f.get());
  std::fseek(f.get(), blob_start, SEEK_SET);
  const size_t blob_floats = (size_t)(file_end - blob_start) / 4;
  std::vector<float> blob(blob_floats);
  if (blob_floats && std::fread(blob.data(), 4, blob_floats, f.get()) != blob_floats)
    return fail(YUF_ERR_IO, "truncated tensor data", path);
  std::unordered_map<std::string, HostTensor> t;
  for (const JVal& e : tensors->arr) {
    const JVal* n = e.get("name");
    const JVal* off = e.get("offset");
    const JVal* cnt = e.get("count");
    if (!n || n->kind != JVal::STR || !off || !cnt) return fail(YUF_ERR_IO, "bad tensor entry", path);
    const size_t o = (size_t)off->num, c = (size_t)cnt->num;
    if (o + c > blob_floats) return fail(YUF_ERR_IO, "tensor extends past the end of the file", path);
    t[n->str] = HostTensor{blob.data() + o, (int64_t)c};
    if (n->str == "blocks.0.time_mix.w1") {
      const JVal* sh = e.get("shape");
      if (sh && sh->kind == JVal::ARR && sh->arr.size() == 2) cfg.low_rank = (int)sh->arr[1].num;
    }
  }
  return model_create_from_map(&cfg, precision, device, t, out);
}
