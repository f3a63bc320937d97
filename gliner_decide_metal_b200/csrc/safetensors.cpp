// safetensors reader: a minimal JSON parser for the header object
//   {"name": {"dtype": "F16", "shape": [..], "data_offsets": [b, e]}, "__metadata__": {..}}
// plus bounds checks of every tensor against the file size.
#include "safetensors.h"

#include <cstdio>
#include <cstring>

#include "common.h"

namespace gdc {
namespace {

struct JsonCursor {
  const char* p;
  const char* end;
  bool ok = true;

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
  bool expect(char c) {
    if (!eat(c)) ok = false;
    return ok;
  }
  bool string(std::string* s) {
    ws();
    if (p >= end || *p != '"') return ok = false;
    ++p;
    s->clear();
    while (p < end && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= end) return ok = false;
        char c = *p;
        if (c == 'u') {  // keep escaped code units verbatim (names are ASCII in practice)
          if (end - p < 5) return ok = false;
          s->append("\\u");
          s->append(p + 1, 4);
          p += 5;
          continue;
        }
        s->push_back(c == 'n' ? '\n' : c == 't' ? '\t' : c);
        ++p;
      } else {
        s->push_back(*p++);
      }
    }
    if (p >= end) return ok = false;
    ++p;
    return true;
  }
  bool integer(int64_t* v) {
    ws();
    const char* s = p;
    bool neg = false;
    if (p < end && *p == '-') {
      neg = true;
      ++p;
    }
    if (p >= end || *p < '0' || *p > '9') return ok = false;
    uint64_t acc = 0;
    while (p < end && *p >= '0' && *p <= '9') {
      if (acc > (UINT64_MAX - 9) / 10) return ok = false;
      acc = acc * 10 + uint64_t(*p - '0');
      ++p;
    }
    (void)s;
    if (acc > uint64_t(INT64_MAX)) return ok = false;
    *v = neg ? -int64_t(acc) : int64_t(acc);
    return true;
  }
  // Skips any JSON value (used for __metadata__ and unknown fields).
  bool skip_value(int depth = 0) {
    if (depth > 32) return ok = false;
    ws();
    if (p >= end) return ok = false;
    if (*p == '"') {
      std::string tmp;
      return string(&tmp);
    }
    if (*p == '{' || *p == '[') {
      char close = (*p == '{') ? '}' : ']';
      bool obj = (*p == '{');
      ++p;
      if (eat(close)) return true;
      while (ok) {
        if (obj) {
          std::string k;
          if (!string(&k) || !expect(':')) return false;
        }
        if (!skip_value(depth + 1)) return false;
        if (eat(',')) continue;
        return expect(close);
      }
      return false;
    }
    while (p < end && *p != ',' && *p != '}' && *p != ']') ++p;  // number / literal
    return true;
  }
  bool int_array(std::vector<int64_t>* v) {
    v->clear();
    if (!expect('[')) return false;
    if (eat(']')) return true;
    while (ok) {
      int64_t x;
      if (!integer(&x)) return false;
      v->push_back(x);
      if (eat(',')) continue;
      return expect(']');
    }
    return false;
  }
};

size_t dtype_size(const std::string& d) {
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  return 0;
}

}  // namespace

gdc_status parse_safetensors_header(const char* json, size_t len, uint64_t data_bytes,
                                    std::map<std::string, TensorInfo>* out) {
  JsonCursor c{json, json + len};
  out->clear();
  if (!c.expect('{')) return set_error(GDC_ERR_IO, "safetensors header is not a JSON object");
  if (c.eat('}')) return GDC_OK;
  while (c.ok) {
    std::string key;
    if (!c.string(&key) || !c.expect(':')) break;
    if (key == "__metadata__") {
      if (!c.skip_value()) break;
    } else {
      TensorInfo t;
      bool have_dtype = false, have_shape = false, have_off = false;
      if (!c.expect('{')) break;
      if (!c.eat('}')) {
        while (c.ok) {
          std::string field;
          if (!c.string(&field) || !c.expect(':')) break;
          if (field == "dtype") {
            have_dtype = c.string(&t.dtype);
          } else if (field == "shape") {
            have_shape = c.int_array(&t.shape);
          } else if (field == "data_offsets") {
            std::vector<int64_t> off;
            have_off = c.int_array(&off) && off.size() == 2 && off[0] >= 0 && off[1] >= off[0];
            if (have_off) {
              t.begin = uint64_t(off[0]);
              t.end = uint64_t(off[1]);
            } else {
              c.ok = false;
            }
          } else {
            c.skip_value();
          }
          if (!c.ok) break;
          if (c.eat(',')) continue;
          c.expect('}');
          break;
        }
      }
      if (!c.ok) break;
      if (!have_dtype || !have_shape || !have_off)
        return set_error(GDC_ERR_IO, "safetensors entry '%s' lacks dtype/shape/data_offsets",
                         key.c_str());
      size_t es = dtype_size(t.dtype);
      if (es == 0) return set_error(GDC_ERR_IO, "tensor '%s' has unknown dtype %s", key.c_str(), t.dtype.c_str());
      uint64_t n = 1;
      for (int64_t d : t.shape) {
        if (d < 0) return set_error(GDC_ERR_IO, "tensor '%s' has a negative dimension", key.c_str());
        n *= uint64_t(d);
      }
      if (t.end - t.begin != n * es)
        return set_error(GDC_ERR_IO, "tensor '%s': byte range %llu does not match shape", key.c_str(),
                         (unsigned long long)(t.end - t.begin));
      if (t.end > data_bytes)
        return set_error(GDC_ERR_IO, "tensor '%s' extends past the end of the file (truncated?)",
                         key.c_str());
      (*out)[key] = t;
    }
    if (c.eat(',')) continue;
    c.expect('}');
    break;
  }
  if (!c.ok) return set_error(GDC_ERR_IO, "malformed safetensors JSON header");
  return GDC_OK;
}

gdc_status SafetensorsFile::open(const std::string& path) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return set_error(GDC_ERR_IO, "cannot open weights file %s", path.c_str());
  std::fseek(f, 0, SEEK_END);
  long long size = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  if (size < 8) {
    std::fclose(f);
    return set_error(GDC_ERR_IO, "%s is too small to be a safetensors file", path.c_str());
  }
  bytes_.resize(size_t(size));
  size_t got = std::fread(bytes_.data(), 1, bytes_.size(), f);
  std::fclose(f);
  if (got != bytes_.size()) return set_error(GDC_ERR_IO, "short read on %s", path.c_str());
  uint64_t n = 0;
  std::memcpy(&n, bytes_.data(), 8);
  if (n > bytes_.size() - 8) return set_error(GDC_ERR_IO, "safetensors header length exceeds file size");
  data_offset_ = 8 + size_t(n);
  return parse_safetensors_header(reinterpret_cast<const char*>(bytes_.data() + 8), size_t(n),
                                  bytes_.size() - data_offset_, &tensors_);
}

const TensorInfo* SafetensorsFile::info(const std::string& key) const {
  auto it = tensors_.find(key);
  return it == tensors_.end() ? nullptr : &it->second;
}

static std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) {
    if (i) r += ", ";
    r += std::to_string(s[i]);
  }
  return r + "]";
}

gdc_status SafetensorsFile::get_f16(const std::string& key, const std::vector<int64_t>* expected_shape,
                                    std::vector<uint16_t>* out, std::vector<int64_t>* shape_out) const {
  const TensorInfo* t = info(key);
  if (!t) return set_error(GDC_ERR_MISSING_WEIGHT, "Missing model weight: %s", key.c_str());
  if (expected_shape && *expected_shape != t->shape)
    return set_error(GDC_ERR_INVALID_SHAPE, "Weight %s has shape %s, expected %s", key.c_str(),
                     shape_str(t->shape).c_str(), shape_str(*expected_shape).c_str());
  uint64_t n = 1;
  for (int64_t d : t->shape) n *= uint64_t(d);
  out->resize(n);
  const uint8_t* src = data(*t);
  if (t->dtype == "F16") {
    std::memcpy(out->data(), src, n * 2);
  } else if (t->dtype == "F32") {
    for (uint64_t i = 0; i < n; ++i) {
      float v;
      std::memcpy(&v, src + 4 * i, 4);
      (*out)[i] = f32_to_f16_bits(v);
    }
  } else if (t->dtype == "BF16") {
    for (uint64_t i = 0; i < n; ++i) {
      uint16_t b;
      std::memcpy(&b, src + 2 * i, 2);
      uint32_t u = uint32_t(b) << 16;
      float v;
      std::memcpy(&v, &u, 4);
      (*out)[i] = f32_to_f16_bits(v);
    }
  } else {
    return set_error(GDC_ERR_INVALID_SHAPE, "Weight %s has dtype %s, expected a float type", key.c_str(),
                     t->dtype.c_str());
  }
  if (shape_out) *shape_out = t->shape;
  return GDC_OK;
}

}  // namespace gdc
