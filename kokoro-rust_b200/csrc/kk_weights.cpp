// Minimal safetensors reader and weight-resolution rules (see kk_weights.h).
#include "kk_weights.h"
#include "kk_pth.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>

namespace kk {

namespace {

// A tiny JSON reader sufficient for a safetensors header: objects, arrays, strings, integers.
struct Json {
  enum Kind { NUL, NUM, STR, ARR, OBJ } kind = NUL;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* find(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct Parser {
  const char* p;
  const char* e;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
  }
  [[noreturn]] void fail(const char* what) { throw KKError(5, std::string("safetensors header: ") + what); }
  std::string string() {
    if (p >= e || *p != '"') fail("expected string");
    p++;
    std::string s;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        p++;
        if (p >= e) fail("bad escape");
        char c = *p;
        if (c == 'n') s += '\n';
        else if (c == 't') s += '\t';
        else if (c == 'u') {
          if (e - p < 5) fail("bad unicode escape");
          unsigned v = (unsigned)strtoul(std::string(p + 1, p + 5).c_str(), nullptr, 16);
          if (v < 0x80) s += (char)v;
          else if (v < 0x800) { s += (char)(0xC0 | (v >> 6)); s += (char)(0x80 | (v & 0x3F)); }
          else { s += (char)(0xE0 | (v >> 12)); s += (char)(0x80 | ((v >> 6) & 0x3F)); s += (char)(0x80 | (v & 0x3F)); }
          p += 4;
        } else s += c;
        p++;
      } else {
        s += *p++;
      }
    }
    if (p >= e) fail("unterminated string");
    p++;
    return s;
  }
  Json value() {
    ws();
    if (p >= e) fail("unexpected end");
    Json j;
    if (*p == '{') {
      j.kind = Json::OBJ;
      p++;
      ws();
      if (p < e && *p == '}') { p++; return j; }
      while (true) {
        ws();
        std::string k = string();
        ws();
        if (p >= e || *p != ':') fail("expected ':'");
        p++;
        j.obj.emplace_back(k, value());
        ws();
        if (p < e && *p == ',') { p++; continue; }
        if (p < e && *p == '}') { p++; break; }
        fail("expected ',' or '}'");
      }
    } else if (*p == '[') {
      j.kind = Json::ARR;
      p++;
      ws();
      if (p < e && *p == ']') { p++; return j; }
      while (true) {
        j.arr.push_back(value());
        ws();
        if (p < e && *p == ',') { p++; continue; }
        if (p < e && *p == ']') { p++; break; }
        fail("expected ',' or ']'");
      }
    } else if (*p == '"') {
      j.kind = Json::STR;
      j.str = string();
    } else if (*p == '-' || (*p >= '0' && *p <= '9')) {
      j.kind = Json::NUM;
      char* end = nullptr;
      std::string tmp(p, std::min<ptrdiff_t>(e - p, 64));
      j.num = strtod(tmp.c_str(), &end);
      if (end == tmp.c_str()) fail("bad number");
      p += end - tmp.c_str();
    } else if (e - p >= 4 && !strncmp(p, "null", 4)) {
      p += 4;
    } else if (e - p >= 4 && !strncmp(p, "true", 4)) {
      p += 4;
    } else if (e - p >= 5 && !strncmp(p, "false", 5)) {
      p += 5;
    } else {
      fail("unexpected character");
    }
    return j;
  }
};

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); i++) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

}  // namespace

Checkpoint::Checkpoint(const std::string& path) {
  if (path.size() >= 4 && path.compare(path.size() - 4, 4, ".pth") == 0) {  // torch.save zip (kk_pth.cpp)
    for (auto& kv : load_pth_checkpoint(path)) map_[kv.first] = std::move(kv.second);
    return;
  }
  std::ifstream f(path, std::ios::binary);
  if (!f) throw KKError(5, "cannot open weights file " + path);
  f.seekg(0, std::ios::end);
  const int64_t fsize = (int64_t)f.tellg();
  f.seekg(0);
  if (fsize < 8) throw KKError(5, "file too short for header length: " + path);
  uint64_t hlen = 0;
  f.read(reinterpret_cast<char*>(&hlen), 8);
  if ((int64_t)(8 + hlen) > fsize) throw KKError(5, "header length exceeds file size: " + path);
  std::string header(hlen, '\0');
  f.read(&header[0], (std::streamsize)hlen);
  std::vector<char> payload((size_t)(fsize - 8 - (int64_t)hlen));
  f.read(payload.data(), (std::streamsize)payload.size());
  if (!f) throw KKError(5, "short read: " + path);
  Parser ps{header.data(), header.data() + header.size()};
  Json root = ps.value();
  if (root.kind != Json::OBJ) throw KKError(5, "header is not a JSON object");
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") continue;
    const Json& info = kv.second;
    const Json* dt = info.find("dtype");
    const Json* sh = info.find("shape");
    const Json* off = info.find("data_offsets");
    if (!dt || !sh || !off || dt->kind != Json::STR || sh->kind != Json::ARR || off->kind != Json::ARR ||
        off->arr.size() != 2)
      throw KKError(5, "malformed entry for " + kv.first);
    HostTensor t;
    int64_t numel = 1;
    for (auto& d : sh->arr) {
      t.shape.push_back((int64_t)d.num);
      numel *= (int64_t)d.num;
    }
    const uint64_t s = (uint64_t)off->arr[0].num, e = (uint64_t)off->arr[1].num;
    if (s > e || e > payload.size()) throw KKError(5, "offsets out of range for " + kv.first);
    const char* raw = payload.data() + s;
    const size_t nb = (size_t)(e - s);
    t.data.resize((size_t)numel);
    if (dt->str == "F32") {
      if (nb != (size_t)numel * 4) throw KKError(5, "size mismatch for " + kv.first);
      memcpy(t.data.data(), raw, nb);
    } else if (dt->str == "F64") {
      if (nb != (size_t)numel * 8) throw KKError(5, "size mismatch for " + kv.first);
      for (int64_t i = 0; i < numel; i++) {
        double v;
        memcpy(&v, raw + 8 * i, 8);
        t.data[i] = (float)v;
      }
    } else if (dt->str == "I64") {
      if (nb != (size_t)numel * 8) throw KKError(5, "size mismatch for " + kv.first);
      for (int64_t i = 0; i < numel; i++) {
        int64_t v;
        memcpy(&v, raw + 8 * i, 8);
        t.data[i] = (float)v;
      }
    } else {
      throw KKError(5, "unsupported dtype " + dt->str + " for " + kv.first);
    }
    map_.emplace(kv.first, std::move(t));
  }
}

std::vector<float> Checkpoint::get(const std::string& name, const std::vector<int64_t>& shape) const {
  auto it = map_.find(name);
  if (it == map_.end()) throw KKError(5, "missing tensor " + name);
  if (it->second.shape != shape)
    throw KKError(5, "tensor " + name + ": shape " + shape_str(it->second.shape) + ", expected " + shape_str(shape));
  return it->second.data;
}

std::vector<float> weight_norm(const std::vector<float>& v, const std::vector<float>& g) {
  const size_t rows = g.size();
  const size_t per = v.size() / rows;
  std::vector<float> w(v.size());
  for (size_t r = 0; r < rows; r++) {
    double ss = 0.0;
    for (size_t i = 0; i < per; i++) ss += (double)v[r * per + i] * (double)v[r * per + i];
    const float norm = (float)std::sqrt(ss);
    const float scale = g[r] / norm;
    for (size_t i = 0; i < per; i++) w[r * per + i] = v[r * per + i] * scale;
  }
  return w;
}

std::vector<float> Checkpoint::conv_weight(const std::string& prefix, const std::vector<int64_t>& shape) const {
  if (has(prefix + ".weight")) return get(prefix + ".weight", shape);
  std::vector<float> v = get(prefix + ".weight_v", shape);
  std::vector<float> g = get(prefix + ".weight_g", {shape[0], 1, 1});
  return weight_norm(v, g);
}

std::vector<float> Checkpoint::norm_affine(const std::string& name, int64_t c, float init) const {
  if (has(name)) return get(name, {c});
  const bool ok = name.size() > 12 && (name.compare(name.size() - 12, 12, ".norm.weight") == 0 ||
                                       name.compare(name.size() - 10, 10, ".norm.bias") == 0);
  if (!ok) throw KKError(5, "missing tensor " + name);
  return std::vector<float>((size_t)c, init);
}

}  // namespace kk
