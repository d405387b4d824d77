// SafeTensors weight loading for the model step (ModelWeights::load,
// rust/engine/src/weights.rs:117-190, with its helpers :206-300).
//
// The file format is the `safetensors` crate's (0.6.2 in the reference's
// Cargo.lock, not vendored here), restated from its published format: an
// 8-byte little-endian header length N, N bytes of a JSON object mapping
// tensor names to {"dtype", "shape", "data_offsets": [begin, end]} (offsets
// into the byte buffer that follows; an optional "__metadata__" entry maps
// strings to strings), then the byte buffer. The buffer must be indexed
// entirely and without holes: sorted by offset, every tensor starts where the
// previous one ends, the last ends at the buffer's end, and each spans its
// element count times its dtype's size.
//
// On top of the format, weights.rs checks: exactly the expected tensor names
// (expected_layout, :344-378; missing and unexpected names are both listed),
// every tensor F32 with the expected shape, little-endian values, and the
// total parameter count against the configuration's expected count.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "slmkv.h"
#include "slmkv_internal.h"

namespace slmkv {
void set_contextless_error(const std::string& message);
}

namespace {

// ---- a small JSON reader for the header ------------------------------------
struct Json {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  bool b = false;
  double num = 0;
  bool integral = false;  // the number was written without fraction or exponent
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;  // in file order
};

class JsonParser {
 public:
  JsonParser(const char* p, size_t n) : p_(p), end_(p + n) {}
  bool parse(Json* out, std::string* err) {
    if (!value(out, 0)) {
      *err = err_.empty() ? "malformed JSON header" : err_;
      return false;
    }
    ws();
    if (p_ != end_) {
      *err = "trailing bytes after the JSON header";
      return false;
    }
    return true;
  }

 private:
  const char* p_;
  const char* end_;
  std::string err_;
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if (static_cast<size_t>(end_ - p_) < n || memcmp(p_, s, n) != 0) return false;
    p_ += n;
    return true;
  }
  bool string(std::string* out) {
    if (p_ >= end_ || *p_ != '"') return false;
    ++p_;
    out->clear();
    while (p_ < end_ && *p_ != '"') {
      char c = *p_++;
      if (static_cast<unsigned char>(c) < 0x20) return false;
      if (c == '\\') {
        if (p_ >= end_) return false;
        const char e = *p_++;
        switch (e) {
          case '"': c = '"'; break;
          case '\\': c = '\\'; break;
          case '/': c = '/'; break;
          case 'b': c = '\b'; break;
          case 'f': c = '\f'; break;
          case 'n': c = '\n'; break;
          case 'r': c = '\r'; break;
          case 't': c = '\t'; break;
          case 'u': {  // \uXXXX as UTF-8 (surrogate pairs combined)
            auto hex4 = [&](uint32_t* v) {
              if (end_ - p_ < 4) return false;
              *v = 0;
              for (int i = 0; i < 4; ++i) {
                const char h = *p_++;
                *v <<= 4;
                if (h >= '0' && h <= '9') *v |= static_cast<uint32_t>(h - '0');
                else if (h >= 'a' && h <= 'f') *v |= static_cast<uint32_t>(h - 'a' + 10);
                else if (h >= 'A' && h <= 'F') *v |= static_cast<uint32_t>(h - 'A' + 10);
                else return false;
              }
              return true;
            };
            uint32_t cp = 0;
            if (!hex4(&cp)) return false;
            if (cp >= 0xD800 && cp < 0xDC00) {
              uint32_t lo = 0;
              if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return false;
              p_ += 2;
              if (!hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return false;
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            }
            if (cp < 0x80) {
              out->push_back(static_cast<char>(cp));
            } else if (cp < 0x800) {
              out->push_back(static_cast<char>(0xC0 | (cp >> 6)));
              out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
            } else if (cp < 0x10000) {
              out->push_back(static_cast<char>(0xE0 | (cp >> 12)));
              out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
              out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
            } else {
              out->push_back(static_cast<char>(0xF0 | (cp >> 18)));
              out->push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
              out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
              out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
            }
            continue;
          }
          default: return false;
        }
      }
      out->push_back(c);
    }
    if (p_ >= end_) return false;
    ++p_;
    return true;
  }
  bool number(Json* out) {
    const char* s = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    bool digits = false, integral = true;
    while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_, digits = true;
    if (p_ < end_ && *p_ == '.') {
      integral = false;
      ++p_;
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      integral = false;
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (!digits) return false;
    const std::string txt(s, static_cast<size_t>(p_ - s));
    out->kind = Json::kNum;
    out->num = strtod(txt.c_str(), nullptr);
    out->integral = integral;
    return true;
  }
  bool value(Json* out, int depth) {
    if (depth > 16) {
      err_ = "JSON header nested too deeply";
      return false;
    }
    ws();
    if (p_ >= end_) return false;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      out->kind = Json::kObj;
      ws();
      if (p_ < end_ && *p_ == '}') return ++p_, true;
      for (;;) {
        ws();
        std::string key;
        if (!string(&key)) return false;
        ws();
        if (p_ >= end_ || *p_ != ':') return false;
        ++p_;
        Json v;
        if (!value(&v, depth + 1)) return false;
        out->obj.emplace_back(std::move(key), std::move(v));
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') return ++p_, true;
        return false;
      }
    }
    if (c == '[') {
      ++p_;
      out->kind = Json::kArr;
      ws();
      if (p_ < end_ && *p_ == ']') return ++p_, true;
      for (;;) {
        Json v;
        if (!value(&v, depth + 1)) return false;
        out->arr.push_back(std::move(v));
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') return ++p_, true;
        return false;
      }
    }
    if (c == '"') {
      out->kind = Json::kStr;
      return string(&out->str);
    }
    if (lit("true")) return out->kind = Json::kBool, out->b = true, true;
    if (lit("false")) return out->kind = Json::kBool, out->b = false, true;
    if (lit("null")) return out->kind = Json::kNull, true;
    return number(out);
  }
};

// Element sizes of the format's dtypes (the names it defines).
int64_t dtype_size(const std::string& d) {
  static const std::map<std::string, int64_t> sizes = {
      {"BOOL", 1}, {"U8", 1}, {"I8", 1}, {"F8_E5M2", 1}, {"F8_E4M3", 1}, {"I16", 2},
      {"U16", 2},  {"F16", 2}, {"BF16", 2}, {"I32", 4},  {"U32", 4},    {"F32", 4},
      {"I64", 8},  {"U64", 8}, {"F64", 8}};
  auto it = sizes.find(d);
  return it == sizes.end() ? -1 : it->second;
}

struct TensorView {
  std::string dtype;
  std::vector<int64_t> shape;
  int64_t begin = 0, end = 0;
};

// The file's bytes and its tensors, validated against the format.
struct SafeTensorsFile {
  std::vector<uint8_t> bytes;
  size_t data_start = 0;
  std::map<std::string, TensorView> tensors;
};

bool read_safetensors(const char* path, SafeTensorsFile* f, std::string* err) {
  FILE* fp = fopen(path, "rb");
  if (!fp) {
    *err = std::string("cannot open ") + path;
    return false;
  }
  if (fseek(fp, 0, SEEK_END) != 0) {
    fclose(fp);
    *err = std::string("cannot read ") + path;
    return false;
  }
  const long len = ftell(fp);
  fseek(fp, 0, SEEK_SET);
  if (len < 8) {
    fclose(fp);
    *err = "file is shorter than the 8-byte header length";
    return false;
  }
  f->bytes.resize(static_cast<size_t>(len));
  const size_t got = fread(f->bytes.data(), 1, f->bytes.size(), fp);
  fclose(fp);
  if (got != f->bytes.size()) {
    *err = std::string("cannot read ") + path;
    return false;
  }
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | f->bytes[static_cast<size_t>(i)];  // little-endian
  if (n > f->bytes.size() - 8 || n > (100ull << 20)) {
    *err = "header length exceeds the file (or 100 MiB)";
    return false;
  }
  Json root;
  JsonParser jp(reinterpret_cast<const char*>(f->bytes.data()) + 8, static_cast<size_t>(n));
  if (!jp.parse(&root, err)) return false;
  if (root.kind != Json::kObj) {
    *err = "header is not a JSON object";
    return false;
  }
  f->data_start = 8 + static_cast<size_t>(n);
  const int64_t buffer = static_cast<int64_t>(f->bytes.size() - f->data_start);
  std::vector<std::pair<int64_t, int64_t>> spans;
  for (const auto& [name, v] : root.obj) {
    if (name == "__metadata__") {
      bool ok = v.kind == Json::kObj;
      for (const auto& kv : v.obj) ok = ok && kv.second.kind == Json::kStr;
      if (!ok) {
        *err = "__metadata__ must map strings to strings";
        return false;
      }
      continue;
    }
    if (v.kind != Json::kObj) {
      *err = "tensor " + name + ": entry is not an object";
      return false;
    }
    TensorView t;
    bool have_dtype = false, have_shape = false, have_offsets = false;
    for (const auto& [k, x] : v.obj) {
      if (k == "dtype" && x.kind == Json::kStr) {
        t.dtype = x.str;
        have_dtype = true;
      } else if (k == "shape" && x.kind == Json::kArr) {
        have_shape = true;
        for (const Json& d : x.arr) {
          if (d.kind != Json::kNum || !d.integral || d.num < 0 || d.num > 9.0e15) {
            *err = "tensor " + name + ": shape entries must be non-negative integers";
            return false;
          }
          t.shape.push_back(static_cast<int64_t>(d.num));
        }
      } else if (k == "data_offsets" && x.kind == Json::kArr && x.arr.size() == 2) {
        for (const Json& d : x.arr)
          if (d.kind != Json::kNum || !d.integral || d.num < 0 || d.num > 9.0e15) {
            *err = "tensor " + name + ": data_offsets must be non-negative integers";
            return false;
          }
        t.begin = static_cast<int64_t>(x.arr[0].num);
        t.end = static_cast<int64_t>(x.arr[1].num);
        have_offsets = true;
      } else {
        *err = "tensor " + name + ": unexpected field " + k;
        return false;
      }
    }
    if (!have_dtype || !have_shape || !have_offsets) {
      *err = "tensor " + name + ": dtype, shape and data_offsets are required";
      return false;
    }
    const int64_t es = dtype_size(t.dtype);
    if (es < 0) {
      *err = "tensor " + name + ": unknown dtype " + t.dtype;
      return false;
    }
    int64_t count = 1;
    for (int64_t d : t.shape) {
      if (d != 0 && count > (int64_t{1} << 60) / d) {
        *err = "tensor " + name + ": element count overflows";
        return false;
      }
      count *= d;
    }
    if (t.end < t.begin || t.end - t.begin != count * es) {
      *err = "tensor " + name + ": data_offsets do not span its shape and dtype";
      return false;
    }
    if (f->tensors.count(name)) {
      *err = "tensor " + name + " appears twice";
      return false;
    }
    spans.emplace_back(t.begin, t.end);
    f->tensors.emplace(name, std::move(t));
  }
  std::sort(spans.begin(), spans.end());
  int64_t at = 0;
  for (const auto& sp : spans) {
    if (sp.first != at) {
      *err = "the byte buffer has holes or overlapping tensors";
      return false;
    }
    at = sp.second;
  }
  if (at != buffer) {
    *err = "the tensors do not index the whole byte buffer";
    return false;
  }
  return true;
}

}  // namespace

namespace {

// weights.rs:344-378 (expected_layout), in the order slm_model_create takes
std::vector<std::pair<std::string, std::vector<int64_t>>> expected_layout(const slm_model_config& c,
                                                                           int32_t layers, int64_t kv) {
  const int64_t H = c.hidden_size, I = c.intermediate_size;
  std::vector<std::pair<std::string, std::vector<int64_t>>> out;
  out.push_back({"token_embedding.weight", {c.vocab_size, H}});
  for (int32_t l = 0; l < layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    out.push_back({p + "attention_norm.weight", {H}});
    out.push_back({p + "q_proj.weight", {H, H}});
    out.push_back({p + "k_proj.weight", {kv, H}});
    out.push_back({p + "v_proj.weight", {kv, H}});
    out.push_back({p + "o_proj.weight", {H, H}});
    out.push_back({p + "ffn_norm.weight", {H}});
    out.push_back({p + "gate_proj.weight", {I, H}});
    out.push_back({p + "up_proj.weight", {I, H}});
    out.push_back({p + "down_proj.weight", {H, I}});
  }
  out.push_back({"final_norm.weight", {H}});
  return out;
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); ++i) o += (i ? ", " : "") + std::to_string(s[i]);
  return o + "]";
}

// weights.rs:126-183: names (validate_names, :246-272), dtype, shape, little-
// endian F32 values, the parameter count. Fills `values` in the model's order.
bool load_layout(const slm_model_config& c, int32_t layers, int64_t kv, const char* path,
                 int64_t expected_count, std::vector<std::vector<float>>* values, int64_t* count,
                 std::string* err) {
  SafeTensorsFile f;
  if (!read_safetensors(path, &f, err)) {
    *err = "invalid weights: " + *err;
    return false;
  }
  const auto expected = expected_layout(c, layers, kv);
  std::set<std::string> want, have;
  for (const auto& e : expected) want.insert(e.first);
  for (const auto& t : f.tensors) have.insert(t.first);
  std::vector<std::string> missing, unexpected;
  std::set_difference(want.begin(), want.end(), have.begin(), have.end(), std::back_inserter(missing));
  std::set_difference(have.begin(), have.end(), want.begin(), want.end(), std::back_inserter(unexpected));
  if (!missing.empty() || !unexpected.empty()) {
    auto list = [](const std::vector<std::string>& v) {
      std::string o = "[";
      for (size_t i = 0; i < v.size() && i < 8; ++i) o += (i ? ", " : "") + v[i];
      if (v.size() > 8) o += ", ...";
      return o + "]";
    };
    *err = "invalid weights: tensor-name mismatch; missing=" + list(missing) + "; unexpected=" + list(unexpected);
    return false;
  }
  int64_t total = 0;
  values->clear();
  for (const auto& [name, shape] : expected) {
    const TensorView& t = f.tensors.at(name);
    if (t.dtype != "F32") {
      *err = "invalid weights: " + name + " must have dtype F32, found " + t.dtype;
      return false;
    }
    if (t.shape != shape) {
      *err = "invalid weights: " + name + " has shape " + shape_str(t.shape) + ", expected " + shape_str(shape);
      return false;
    }
    const int64_t n = (t.end - t.begin) / 4;
    std::vector<float> v(static_cast<size_t>(n));
    // little-endian F32 (weights.rs:216-226); the buffer need not be aligned
    const uint8_t* src = f.bytes.data() + f.data_start + t.begin;
    for (int64_t i = 0; i < n; ++i) {
      const uint32_t b = static_cast<uint32_t>(src[4 * i]) | (static_cast<uint32_t>(src[4 * i + 1]) << 8) |
                         (static_cast<uint32_t>(src[4 * i + 2]) << 16) |
                         (static_cast<uint32_t>(src[4 * i + 3]) << 24);
      std::memcpy(&v[static_cast<size_t>(i)], &b, 4);
    }
    values->push_back(std::move(v));
    total += n;
  }
  if (expected_count > 0 && total != expected_count) {
    *err = "invalid weights: loaded " + std::to_string(total) + " parameters, expected " +
           std::to_string(expected_count);
    return false;
  }
  *count = total;
  return true;
}

}  // namespace

extern "C" {

slm_status slm_safetensors_check(const slm_model_config* config, int32_t num_layers,
                                 int32_t num_key_value_heads, int32_t head_dimension, const char* path,
                                 int64_t expected_parameter_count, int64_t* parameter_count) {
  if (!config || !path || num_layers < 1 || num_key_value_heads < 1 || head_dimension < 1)
    return SLM_ERR_INVALID_INPUT;
  std::vector<std::vector<float>> values;
  int64_t count = 0;
  std::string err;
  if (!load_layout(*config, num_layers, static_cast<int64_t>(num_key_value_heads) * head_dimension, path,
                   expected_parameter_count, &values, &count, &err)) {
    slmkv::set_contextless_error(err);
    return SLM_ERR_INVALID_INPUT;
  }
  if (parameter_count) *parameter_count = count;
  return SLM_OK;
}

slm_status slm_model_load_safetensors(slm_ctx* ctx, const slm_model_config* config, const char* path,
                                      int64_t expected_parameter_count, slm_model** out) {
  if (!ctx || !config || !path || !out) return SLM_ERR_INVALID_INPUT;
  slm_config c{};
  slm_status rc = slm_ctx_config(ctx, &c);
  if (rc) return rc;
  std::vector<std::vector<float>> values;
  int64_t count = 0;
  std::string err;
  if (!load_layout(*config, c.num_layers, static_cast<int64_t>(c.num_key_value_heads) * c.head_dimension,
                   path, expected_parameter_count, &values, &count, &err))
    return slmkv::ctx_fail(ctx, SLM_ERR_INVALID_INPUT, err.c_str());
  std::vector<const float*> ptrs;
  for (const auto& v : values) ptrs.push_back(v.data());
  return slm_model_create(ctx, config, ptrs.data(), static_cast<int32_t>(ptrs.size()), out);
}

}  // extern "C"
