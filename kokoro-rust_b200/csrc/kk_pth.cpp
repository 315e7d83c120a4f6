// PyTorch zip checkpoint reader (see kk_pth.h): zip central directory -> entries, data.pkl
// interpreted by a restricted pickle machine into dicts / tuples / tensor views, tensor views
// materialised from their storages (little-endian f32).
#include "kk_pth.h"

#include <cstring>
#include <fstream>
#include <memory>
#include <unordered_map>
#include <vector>

namespace kk {
namespace {

[[noreturn]] void fail(const std::string& m) { throw KKError(5, m); }

struct Zip {
  std::vector<uint8_t> bytes;
  std::unordered_map<std::string, std::pair<size_t, size_t>> entries;  // name -> (offset, size)

  uint32_t u16(size_t o) const {
    if (o + 2 > bytes.size()) fail("zip truncated");
    return (uint32_t)bytes[o] | ((uint32_t)bytes[o + 1] << 8);
  }
  uint32_t u32(size_t o) const {
    if (o + 4 > bytes.size()) fail("zip truncated");
    return u16(o) | (u16(o + 2) << 16);
  }

  explicit Zip(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) fail("cannot open " + path);
    f.seekg(0, std::ios::end);
    bytes.resize((size_t)f.tellg());
    f.seekg(0);
    f.read(reinterpret_cast<char*>(bytes.data()), (std::streamsize)bytes.size());
    if (!f) fail("short read: " + path);
    if (bytes.size() < 22) fail("not a zip file: " + path);
    // end-of-central-directory record: last 22 bytes, or earlier when an archive comment follows
    size_t eocd = bytes.size() - 22, lo = bytes.size() > 22 + 65535 ? bytes.size() - 22 - 65535 : 0;
    for (;; eocd--) {
      if (u32(eocd) == 0x06054b50u) break;
      if (eocd == lo) fail("zip end-of-central-directory not found");
    }
    const size_t n = u16(eocd + 10);
    const uint32_t cd = u32(eocd + 16);
    if (cd == 0xFFFFFFFFu) fail("zip64 archives are not supported");
    size_t p = cd;
    for (size_t k = 0; k < n; k++) {
      if (u32(p) != 0x02014b50u) fail("bad central directory entry");
      const uint32_t method = u16(p + 10), csize = u32(p + 20), usize = u32(p + 24);
      const size_t nlen = u16(p + 28), xlen = u16(p + 30), clen = u16(p + 32);
      const size_t lho = u32(p + 42);
      if (p + 46 + nlen > bytes.size()) fail("zip truncated");
      const std::string name(reinterpret_cast<const char*>(&bytes[p + 46]), nlen);
      if (method != 0) fail("zip entry " + name + " is compressed (method " + std::to_string(method) + "); only STORED is supported");
      if (csize != usize || csize == 0xFFFFFFFFu) fail("zip entry " + name + ": unsupported sizes");
      if (u32(lho) != 0x04034b50u) fail("bad local header for " + name);
      const size_t data = lho + 30 + u16(lho + 26) + u16(lho + 28);
      if (data + csize > bytes.size()) fail("zip entry " + name + " out of range");
      entries[name] = {data, csize};
      p += 46 + nlen + xlen + clen;
    }
  }
  const uint8_t* get(const std::string& name, size_t* size) const {
    auto it = entries.find(name);
    if (it == entries.end()) fail("zip entry " + name + " missing");
    *size = it->second.second;
    return bytes.data() + it->second.first;
  }
};

// Pickle values: the subset torch.save writes for dicts of f32 tensors.
struct Val;
using VP = std::shared_ptr<Val>;
struct Val {
  enum Kind { NONE, BOOL, INT, STR, TUPLE, DICT, GLOBAL, STORAGE, TENSOR, MARK } kind = NONE;
  int64_t i = 0;
  std::string s;                       // STR, GLOBAL name, STORAGE key, TENSOR storage key
  std::vector<VP> items;               // TUPLE
  std::vector<std::pair<VP, VP>> dict; // DICT
  std::vector<int64_t> shape, stride;  // TENSOR
};
VP mk(Val::Kind k) {
  auto v = std::make_shared<Val>();
  v->kind = k;
  return v;
}

std::vector<int64_t> int_tuple(const VP& v) {
  if (v->kind != Val::TUPLE) fail("expected tuple of ints");
  std::vector<int64_t> out;
  for (auto& x : v->items) {
    if (x->kind != Val::INT || x->i < 0) fail("expected non-negative int");
    out.push_back(x->i);
  }
  return out;
}

VP unpickle(const uint8_t* d, size_t n) {
  std::vector<VP> st;
  std::unordered_map<uint32_t, VP> memo;
  size_t i = 0;
  auto rd = [&](size_t k) -> const uint8_t* {
    if (i + k > n) fail("pickle truncated");
    const uint8_t* p = d + i;
    i += k;
    return p;
  };
  auto le = [](const uint8_t* p, int k) {
    uint64_t v = 0;
    for (int b = k - 1; b >= 0; b--) v = (v << 8) | p[b];
    return v;
  };
  auto pop = [&](const char* what) {
    if (st.empty()) fail(std::string(what) + " underflow");
    VP v = st.back();
    st.pop_back();
    return v;
  };
  auto pop_mark = [&]() {
    size_t m = st.size();
    while (m > 0 && st[m - 1]->kind != Val::MARK) m--;
    if (m == 0) fail("MARK not found");
    std::vector<VP> items(st.begin() + m, st.end());
    st.resize(m - 1);
    return items;
  };
  while (true) {
    const uint8_t op = *rd(1);
    switch (op) {
      case 0x80: rd(1); break;  // PROTO
      case '}': st.push_back(mk(Val::DICT)); break;
      case ')': case ']': st.push_back(mk(Val::TUPLE)); break;  // EMPTY_TUPLE / EMPTY_LIST
      case 'N': st.push_back(mk(Val::NONE)); break;
      case 0x88: case 0x89: st.push_back(mk(Val::BOOL)); break;
      case '(': st.push_back(mk(Val::MARK)); break;
      case 'X': {
        const size_t k = (size_t)le(rd(4), 4);
        auto v = mk(Val::STR);
        v->s.assign(reinterpret_cast<const char*>(rd(k)), k);
        st.push_back(v);
        break;
      }
      case 'J': { auto v = mk(Val::INT); v->i = (int32_t)le(rd(4), 4); st.push_back(v); break; }
      case 'K': { auto v = mk(Val::INT); v->i = *rd(1); st.push_back(v); break; }
      case 'M': { auto v = mk(Val::INT); v->i = (int64_t)le(rd(2), 2); st.push_back(v); break; }
      case 'q': { const uint32_t k = *rd(1); if (st.empty()) fail("BINPUT on empty stack"); memo[k] = st.back(); break; }
      case 'r': { const uint32_t k = (uint32_t)le(rd(4), 4); if (st.empty()) fail("LONG_BINPUT on empty stack"); memo[k] = st.back(); break; }
      case 'h': case 'j': {
        const uint32_t k = op == 'h' ? *rd(1) : (uint32_t)le(rd(4), 4);
        auto it = memo.find(k);
        if (it == memo.end()) fail("BINGET miss");
        st.push_back(it->second);
        break;
      }
      case 'c': {  // GLOBAL "module\nname\n"
        size_t a = i;
        while (a < n && d[a] != '\n') a++;
        size_t b = a + 1;
        while (b < n && d[b] != '\n') b++;
        if (b >= n) fail("bad GLOBAL");
        const std::string g = std::string(reinterpret_cast<const char*>(d + i), a - i) + "." +
                              std::string(reinterpret_cast<const char*>(d + a + 1), b - a - 1);
        i = b + 1;
        if (g != "collections.OrderedDict" && g != "torch._utils._rebuild_tensor_v2" && g != "torch.FloatStorage")
          fail("refusing unsupported pickle global " + g);
        auto v = mk(Val::GLOBAL);
        v->s = g;
        st.push_back(v);
        break;
      }
      case 't': { auto v = mk(Val::TUPLE); v->items = pop_mark(); st.push_back(v); break; }
      case 0x85: case 0x86: case 0x87: {  // TUPLE1..3
        const size_t k = op - 0x84;
        if (st.size() < k) fail("TUPLE underflow");
        auto v = mk(Val::TUPLE);
        v->items.assign(st.end() - k, st.end());
        st.resize(st.size() - k);
        st.push_back(v);
        break;
      }
      case 'Q': {  // BINPERSID: ('storage', torch.FloatStorage, key, location, numel)
        VP pid = pop("BINPERSID");
        if (pid->kind != Val::TUPLE || pid->items.size() != 5 || pid->items[0]->kind != Val::STR ||
            pid->items[0]->s != "storage" || pid->items[1]->kind != Val::GLOBAL ||
            pid->items[1]->s != "torch.FloatStorage" || pid->items[2]->kind != Val::STR)
          fail("unsupported persistent id");
        auto v = mk(Val::STORAGE);
        v->s = pid->items[2]->s;
        st.push_back(v);
        break;
      }
      case 'R': {
        VP args = pop("REDUCE"), f = pop("REDUCE");
        if (f->kind == Val::GLOBAL && f->s == "collections.OrderedDict" && args->kind == Val::TUPLE) {
          st.push_back(mk(Val::DICT));
        } else if (f->kind == Val::GLOBAL && f->s == "torch._utils._rebuild_tensor_v2" && args->kind == Val::TUPLE) {
          if (args->items.size() < 4) fail("_rebuild_tensor_v2 args");
          if (args->items[0]->kind != Val::STORAGE) fail("tensor without storage");
          if (args->items[1]->kind != Val::INT || args->items[1]->i < 0) fail("bad storage offset");
          auto v = mk(Val::TENSOR);
          v->s = args->items[0]->s;
          v->i = args->items[1]->i;
          v->shape = int_tuple(args->items[2]);
          v->stride = int_tuple(args->items[3]);
          if (v->shape.size() != v->stride.size()) fail("tensor shape / stride rank mismatch");
          st.push_back(v);
        } else {
          fail("unsupported REDUCE");
        }
        break;
      }
      case 'b': pop("BUILD"); break;  // object state (OrderedDict._metadata): ignored
      case 's': {
        VP v = pop("SETITEM"), k = pop("SETITEM");
        if (st.empty() || st.back()->kind != Val::DICT) fail("SETITEM on non-dict");
        st.back()->dict.push_back({k, v});
        break;
      }
      case 'u': {
        std::vector<VP> items = pop_mark();
        if (items.size() % 2) fail("SETITEMS odd count");
        if (st.empty() || st.back()->kind != Val::DICT) fail("SETITEMS on non-dict");
        for (size_t k = 0; k < items.size(); k += 2) st.back()->dict.push_back({items[k], items[k + 1]});
        break;
      }
      case '.': return pop("STOP");
      default: fail("unsupported pickle opcode " + std::to_string(op) + " at " + std::to_string(i - 1));
    }
  }
}

struct Loader {
  Zip zip;
  std::string prefix;
  VP root;
  explicit Loader(const std::string& path) : zip(path) {
    std::string pkl;
    for (auto& e : zip.entries)
      if (e.first.size() >= 9 && e.first.compare(e.first.size() - 9, 9, "/data.pkl") == 0) pkl = e.first;
    if (pkl.empty()) fail("no data.pkl in checkpoint " + path);
    prefix = pkl.substr(0, pkl.size() - 8);
    if (zip.entries.count(prefix + "byteorder")) {
      size_t k = 0;
      const uint8_t* p = zip.get(prefix + "byteorder", &k);
      if (std::string(reinterpret_cast<const char*>(p), k) != "little") fail("unsupported byteorder");
    }
    size_t k = 0;
    const uint8_t* p = zip.get(pkl, &k);
    root = unpickle(p, k);
  }
  // A tensor view materialised as contiguous row-major f32 (strides in elements of its storage).
  HostTensor tensor(const VP& v) const {
    if (v->kind != Val::TENSOR) fail("expected tensor");
    size_t bytes = 0;
    const uint8_t* raw = zip.get(prefix + "data/" + v->s, &bytes);
    if (bytes % 4) fail("storage " + v->s + " size not a multiple of 4");
    const int64_t avail = (int64_t)(bytes / 4);
    HostTensor t;
    t.shape = v->shape;
    int64_t numel = 1, last = v->i;
    for (size_t d = 0; d < v->shape.size(); d++) {
      numel *= v->shape[d];
      if (v->shape[d] > 0) last += (v->shape[d] - 1) * v->stride[d];
    }
    if (numel > 0 && last >= avail) fail("tensor view exceeds storage " + v->s);
    t.data.resize((size_t)numel);
    const size_t nd = v->shape.size();
    std::vector<int64_t> idx(nd, 0);
    for (int64_t e = 0; e < numel; e++) {
      int64_t off = v->i;
      for (size_t d = 0; d < nd; d++) off += idx[d] * v->stride[d];
      memcpy(&t.data[(size_t)e], raw + 4 * off, 4);  // little-endian f32 (byteorder checked)
      for (size_t d = nd; d-- > 0;) {
        if (++idx[d] < v->shape[d]) break;
        idx[d] = 0;
      }
    }
    return t;
  }
};

const std::string& key_str(const VP& v) {
  if (v->kind != Val::STR) fail("non-string dict key");
  return v->s;
}

}  // namespace

std::map<std::string, HostTensor> load_pth_checkpoint(const std::string& path) {
  Loader ld(path);
  if (ld.root->kind != Val::DICT) fail("checkpoint root is not a dict");
  std::map<std::string, HostTensor> out;
  for (auto& kv : ld.root->dict) {
    const std::string& sub = key_str(kv.first);
    if (kv.second->kind != Val::DICT) fail(sub + " is not a state dict");
    for (auto& pt : kv.second->dict) {
      std::string name = key_str(pt.first);
      if (name.compare(0, 7, "module.") == 0) name = name.substr(7);
      out[sub + "." + name] = ld.tensor(pt.second);
    }
  }
  return out;
}

HostTensor load_pth_voice(const std::string& path) {
  Loader ld(path);
  HostTensor t = ld.tensor(ld.root);
  if (t.shape.size() != 3 || t.shape[1] != 1 || t.shape[2] != 256) {
    std::string s;
    for (auto d : t.shape) s += (s.empty() ? "" : ", ") + std::to_string(d);
    fail("unexpected voice pack shape [" + s + "]");
  }
  return t;
}

}  // namespace kk

// ---------------------------------------------------------------------------- C ABI
#include "../../include/kokoro_b200.h"

struct kk_pth {
  std::vector<std::string> names;
  std::vector<kk::HostTensor> tensors;
};

namespace {
thread_local std::string g_pth_error;
}

extern "C" {

KK_API kk_status kk_pth_open(const char* path, int kind, kk_pth** out) {
  if (!path || !out || (kind != KK_PTH_CHECKPOINT && kind != KK_PTH_VOICE)) {
    g_pth_error = "invalid argument";
    return KK_ERR_INVALID_ARG;
  }
  *out = nullptr;
  try {
    auto p = std::make_unique<kk_pth>();
    if (kind == KK_PTH_CHECKPOINT) {
      for (auto& kv : kk::load_pth_checkpoint(path)) {
        p->names.push_back(kv.first);
        p->tensors.push_back(std::move(kv.second));
      }
    } else {
      p->names.push_back("voice");
      p->tensors.push_back(kk::load_pth_voice(path));
    }
    *out = p.release();
    return KK_OK;
  } catch (const kk::KKError& e) {
    g_pth_error = e.what();
    return (kk_status)e.status;
  } catch (const std::exception& e) {
    g_pth_error = e.what();
    return KK_ERR_IO;
  }
}

KK_API int kk_pth_count(const kk_pth* p) { return p ? (int)p->names.size() : 0; }

KK_API const char* kk_pth_name(const kk_pth* p, int i) {
  return (p && i >= 0 && i < (int)p->names.size()) ? p->names[(size_t)i].c_str() : nullptr;
}

KK_API int kk_pth_shape(const kk_pth* p, int i, int64_t* dims, int cap) {
  if (!p || i < 0 || i >= (int)p->names.size()) return -1;
  const auto& s = p->tensors[(size_t)i].shape;
  for (int d = 0; d < (int)s.size() && d < cap; d++) dims[d] = s[(size_t)d];
  return (int)s.size();
}

KK_API const float* kk_pth_data(const kk_pth* p, int i) {
  return (p && i >= 0 && i < (int)p->names.size()) ? p->tensors[(size_t)i].data.data() : nullptr;
}

KK_API void kk_pth_close(kk_pth* p) { delete p; }

KK_API const char* kk_pth_error(void) { return g_pth_error.c_str(); }

}  // extern "C"
