#include "safetensors.hpp"

#include <cstring>

namespace hkb {
namespace {

struct Cursor {
  const char* p;
  const char* end;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < end && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool string(std::string* s) {
    ws();
    if (p >= end || *p != '"') return false;
    ++p;
    s->clear();
    while (p < end && *p != '"') {
      if (*p == '\\' && p + 1 < end) ++p;
      s->push_back(*p++);
    }
    if (p >= end) return false;
    ++p;
    return true;
  }
  bool integer(int64_t* v) {
    ws();
    bool neg = false;
    if (p < end && *p == '-') {
      neg = true;
      ++p;
    }
    if (p >= end || *p < '0' || *p > '9') return false;
    int64_t x = 0;
    while (p < end && *p >= '0' && *p <= '9') x = x * 10 + (*p++ - '0');
    *v = neg ? -x : x;
    return true;
  }
  // Skips any JSON value (used for __metadata__ and unknown keys).
  bool skip() {
    ws();
    if (p >= end) return false;
    if (*p == '"') {
      std::string s;
      return string(&s);
    }
    if (*p == '{' || *p == '[') {
      const char open = *p, close = open == '{' ? '}' : ']';
      int depth = 0;
      while (p < end) {
        if (*p == '"') {
          std::string s;
          if (!string(&s)) return false;
          continue;
        }
        if (*p == open) ++depth;
        if (*p == close && --depth == 0) {
          ++p;
          return true;
        }
        ++p;
      }
      return false;
    }
    while (p < end && *p != ',' && *p != '}' && *p != ']') ++p;
    return true;
  }
};

}  // namespace

bool parse_safetensors(const void* blob, size_t length,
                       std::map<std::string, TensorView>* out,
                       std::vector<float>* storage, const char** why) {
  const auto* bytes = static_cast<const unsigned char*>(blob);
  if (blob == nullptr || length < 8) {
    *why = "safetensors image is empty or truncated";
    return false;
  }
  uint64_t hlen = 0;
  std::memcpy(&hlen, bytes, 8);
  if (hlen > length - 8) {
    *why = "safetensors header length exceeds the image";
    return false;
  }
  const char* h = reinterpret_cast<const char*>(bytes + 8);
  const size_t data_base = 8 + hlen;
  const size_t data_len = length - data_base;
  Cursor c{h, h + hlen};
  if (!c.eat('{')) {
    *why = "safetensors header is not a JSON object";
    return false;
  }
  struct Pending {
    std::string name;
    std::vector<int64_t> shape;
    int64_t begin, end;
  };
  std::vector<Pending> items;
  bool first = true;
  while (true) {
    if (c.eat('}')) break;
    if (!first && !c.eat(',')) {
      *why = "safetensors header: expected ','";
      return false;
    }
    first = false;
    std::string name;
    if (!c.string(&name) || !c.eat(':')) {
      *why = "safetensors header: bad key";
      return false;
    }
    if (name == "__metadata__") {
      if (!c.skip()) {
        *why = "safetensors header: bad metadata";
        return false;
      }
      continue;
    }
    if (!c.eat('{')) {
      *why = "safetensors header: tensor entry is not an object";
      return false;
    }
    Pending pd{name, {}, -1, -1};
    std::string dtype;
    bool f = true;
    while (true) {
      if (c.eat('}')) break;
      if (!f && !c.eat(',')) {
        *why = "safetensors header: expected ',' in tensor entry";
        return false;
      }
      f = false;
      std::string key;
      if (!c.string(&key) || !c.eat(':')) {
        *why = "safetensors header: bad tensor field";
        return false;
      }
      if (key == "dtype") {
        if (!c.string(&dtype)) return (*why = "safetensors header: bad dtype", false);
      } else if (key == "shape" || key == "data_offsets") {
        std::vector<int64_t> v;
        if (!c.eat('[')) return (*why = "safetensors header: bad array", false);
        if (!c.eat(']')) {
          while (true) {
            int64_t x;
            if (!c.integer(&x)) return (*why = "safetensors header: bad integer", false);
            v.push_back(x);
            if (c.eat(']')) break;
            if (!c.eat(',')) return (*why = "safetensors header: bad array separator", false);
          }
        }
        if (key == "shape") {
          pd.shape = v;
        } else {
          if (v.size() != 2) return (*why = "safetensors header: bad data_offsets", false);
          pd.begin = v[0];
          pd.end = v[1];
        }
      } else if (!c.skip()) {
        *why = "safetensors header: bad field value";
        return false;
      }
    }
    if (dtype != "F32") {
      *why = "safetensors tensor dtype must be F32";
      return false;
    }
    items.push_back(pd);
  }
  size_t total = 0;
  for (const auto& it : items) {
    int64_t n = 1;
    for (int64_t d : it.shape) n *= d;
    if (it.begin < 0 || it.end < it.begin || (size_t)it.end > data_len ||
        it.end - it.begin != n * 4) {
      *why = "safetensors tensor extent disagrees with its shape";
      return false;
    }
    total += (size_t)n;
  }
  // Copy into aligned float storage (the image may sit at any alignment).
  storage->assign(total, 0.0f);
  size_t at = 0;
  out->clear();
  for (const auto& it : items) {
    const int64_t n = (it.end - it.begin) / 4;
    std::memcpy(storage->data() + at, bytes + data_base + it.begin, (size_t)n * 4);
    TensorView tv;
    tv.shape = it.shape;
    tv.count = n;
    tv.data = storage->data() + at;
    (*out)[it.name] = tv;
    at += (size_t)n;
  }
  return true;
}

}  // namespace hkb
