// Qwen3 checkpoint reading: config.json validation, safetensors indexing and
// validation (host only). Replaces load_and_validate_config /
// load_and_validate_checkpoint / expected_shape (qwen3/model.cpp:376-495),
// generalised from the reference's fixed Qwen3-8B shape to any Qwen3 shape
// with head_dim 128 (0.6B and 8B among them), tied or untied embeddings, and
// either a sharded checkpoint (model.safetensors.index.json) or a single
// model.safetensors file. The checks follow the reference: BF16 only, shapes
// exactly as the config implies, every expected tensor present and nothing
// else, payloads inside their shard and not overlapping, the index's
// total_size equal to the payload bytes. The upload into an engine is in
// engine.cu (per tensor-parallel rank, through pinned staging buffers).
#include <fcntl.h>
#include <cerrno>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "xpu_internal.h"

namespace xpu {
namespace {

// ---------------------------------------------------------------- JSON ----
// A small recursive-descent JSON reader: objects, arrays, strings (with
// escapes, \u to UTF-8), numbers, true/false/null.
struct JValue {
  enum Type { Null, Bool, Number, String, Array, Object } type = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<JValue> arr;
  std::vector<std::pair<std::string, JValue>> obj;

  const JValue *get(const std::string &key) const {
    if (type != Object) return nullptr;
    for (const auto &kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class JReader {
 public:
  JReader(const std::string &text, const std::string &what) : s_(text), what_(what) {}

  JValue document() {
    JValue v = value(0);
    space();
    if (i_ != s_.size()) error("unexpected trailing characters");
    return v;
  }

 private:
  [[noreturn]] void error(const std::string &msg) const {
    throw std::runtime_error(what_ + ": malformed JSON at byte " + std::to_string(i_) + " (" + msg + ")");
  }
  void space() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\t' || s_[i_] == '\n' || s_[i_] == '\r')) ++i_;
  }
  char next() {
    if (i_ >= s_.size()) error("input ends early");
    return s_[i_++];
  }
  void expect_word(const char *w) {
    for (const char *p = w; *p; ++p)
      if (next() != *p) error(std::string("expected '") + w + "'");
  }
  static void utf8(std::string &out, uint32_t cp) {
    if (cp < 0x80) {
      out += static_cast<char>(cp);
    } else if (cp < 0x800) {
      out += static_cast<char>(0xC0 | (cp >> 6));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      out += static_cast<char>(0xE0 | (cp >> 12));
      out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    } else {
      out += static_cast<char>(0xF0 | (cp >> 18));
      out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
      out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = next();
      v <<= 4;
      if (c >= '0' && c <= '9') v |= static_cast<uint32_t>(c - '0');
      else if (c >= 'a' && c <= 'f') v |= static_cast<uint32_t>(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= static_cast<uint32_t>(c - 'A' + 10);
      else error("bad \\u escape");
    }
    return v;
  }
  std::string string_body() {
    std::string out;
    for (;;) {
      const char c = next();
      if (c == '"') return out;
      if (static_cast<unsigned char>(c) < 0x20) error("control character in string");
      if (c != '\\') { out += c; continue; }
      const char e = next();
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            if (next() != '\\' || next() != 'u') error("unpaired surrogate");
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) error("unpaired surrogate");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(out, cp);
          break;
        }
        default: error("bad escape");
      }
    }
  }
  JValue number() {
    const size_t start = i_;
    if (s_[i_] == '-') ++i_;
    auto digits = [&] {
      const size_t d0 = i_;
      while (i_ < s_.size() && s_[i_] >= '0' && s_[i_] <= '9') ++i_;
      if (i_ == d0) error("expected digits");
    };
    digits();
    if (i_ < s_.size() && s_[i_] == '.') { ++i_; digits(); }
    if (i_ < s_.size() && (s_[i_] == 'e' || s_[i_] == 'E')) {
      ++i_;
      if (i_ < s_.size() && (s_[i_] == '+' || s_[i_] == '-')) ++i_;
      digits();
    }
    JValue v;
    v.type = JValue::Number;
    v.num = std::strtod(s_.substr(start, i_ - start).c_str(), nullptr);
    return v;
  }
  JValue value(int depth) {
    if (depth > 64) error("nesting too deep");
    space();
    if (i_ >= s_.size()) error("expected a value");
    JValue v;
    const char c = s_[i_];
    if (c == '{') {
      ++i_;
      v.type = JValue::Object;
      space();
      if (i_ < s_.size() && s_[i_] == '}') { ++i_; return v; }
      for (;;) {
        space();
        if (next() != '"') error("expected a key");
        std::string key = string_body();
        for (const auto &kv : v.obj)
          if (kv.first == key) error("duplicate key '" + key + "'");
        space();
        if (next() != ':') error("expected ':'");
        v.obj.emplace_back(std::move(key), value(depth + 1));
        space();
        const char d = next();
        if (d == '}') return v;
        if (d != ',') error("expected ',' or '}'");
      }
    }
    if (c == '[') {
      ++i_;
      v.type = JValue::Array;
      space();
      if (i_ < s_.size() && s_[i_] == ']') { ++i_; return v; }
      for (;;) {
        v.arr.push_back(value(depth + 1));
        space();
        const char d = next();
        if (d == ']') return v;
        if (d != ',') error("expected ',' or ']'");
      }
    }
    if (c == '"') {
      ++i_;
      v.type = JValue::String;
      v.str = string_body();
      return v;
    }
    if (c == 't') { expect_word("true"); v.type = JValue::Bool; v.b = true; return v; }
    if (c == 'f') { expect_word("false"); v.type = JValue::Bool; return v; }
    if (c == 'n') { expect_word("null"); return v; }
    if (c == '-' || (c >= '0' && c <= '9')) return number();
    error("unexpected character");
  }

  const std::string &s_;
  std::string what_;
  size_t i_ = 0;
};

// ------------------------------------------------------------------ files ----
using Fd = FileReader;

bool file_exists(const std::string &path) {
  struct stat st {};
  return ::stat(path.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

std::string read_text(const std::string &path, uint64_t limit) {
  Fd f(path);
  const uint64_t n = f.size();
  if (n > limit) throw std::runtime_error(path + " is larger than " + std::to_string(limit) + " bytes");
  std::string s(n, '\0');
  if (n) f.read(&s[0], n, 0);
  return s;
}

// ---------------------------------------------------------- config fields ----
const JValue &field(const JValue &root, const char *name, const std::string &file) {
  const JValue *v = root.get(name);
  if (!v) throw std::runtime_error(file + ": missing field '" + name + "'");
  return *v;
}

uint32_t u32_field(const JValue &root, const char *name, const std::string &file) {
  const JValue &v = field(root, name, file);
  if (v.type != JValue::Number || v.num < 0 || v.num > 4294967295.0 || v.num != std::floor(v.num))
    throw std::runtime_error(file + ": '" + name + "' must be an unsigned 32-bit integer");
  return static_cast<uint32_t>(v.num);
}

double num_field(const JValue &root, const char *name, const std::string &file) {
  const JValue &v = field(root, name, file);
  if (v.type != JValue::Number) throw std::runtime_error(file + ": '" + name + "' must be a number");
  return v.num;
}

std::string str_field(const JValue &root, const char *name, const std::string &file) {
  const JValue &v = field(root, name, file);
  if (v.type != JValue::String) throw std::runtime_error(file + ": '" + name + "' must be a string");
  return v.str;
}

uint64_t exact_u64(const JValue &v, const std::string &what) {
  if (v.type != JValue::Number || v.num < 0 || v.num > 9007199254740992.0 || v.num != std::floor(v.num))
    throw std::runtime_error(what + " must be a non-negative integer");
  return static_cast<uint64_t>(v.num);
}

}  // namespace

FileReader::FileReader(const std::string &path) : fd_(::open(path.c_str(), O_RDONLY | O_CLOEXEC)), path_(path) {
  if (fd_ < 0) throw std::runtime_error("cannot open " + path + ": " + std::strerror(errno));
}

FileReader::~FileReader() {
  if (fd_ >= 0) ::close(fd_);
}

uint64_t FileReader::size() const {
  struct stat st {};
  if (fstat(fd_, &st) != 0) throw std::runtime_error("cannot stat " + path_);
  return static_cast<uint64_t>(st.st_size);
}

void FileReader::read(void *dst, uint64_t bytes, uint64_t offset) const {
  auto *p = static_cast<uint8_t *>(dst);
  while (bytes) {
    const ssize_t n = ::pread(fd_, p, std::min<uint64_t>(bytes, 1ull << 30), static_cast<off_t>(offset));
    if (n <= 0) throw std::runtime_error("short read from " + path_);
    p += n;
    bytes -= static_cast<uint64_t>(n);
    offset += static_cast<uint64_t>(n);
  }
}

// ------------------------------------------------------- expected tensors ----
std::vector<std::string> qwen3_tensor_names(const xpu_qwen3_shape &s) {
  std::vector<std::string> names{"model.embed_tokens.weight", "model.norm.weight"};
  if (!s.tie_word_embeddings) names.push_back("lm_head.weight");
  static const char *suffix[] = {
      "input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
      "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
      "self_attn.q_norm.weight", "self_attn.k_norm.weight", "mlp.gate_proj.weight",
      "mlp.up_proj.weight", "mlp.down_proj.weight"};
  for (uint32_t l = 0; l < s.num_hidden_layers; ++l)
    for (const char *x : suffix) names.push_back("model.layers." + std::to_string(l) + "." + x);
  return names;
}

std::vector<uint64_t> qwen3_tensor_shape(const xpu_qwen3_shape &s, const std::string &name) {
  const uint64_t H = s.hidden_size, I = s.intermediate_size, V = s.vocab_size;
  const uint64_t Q = 128ull * s.num_attention_heads, KV = 128ull * s.num_key_value_heads;
  if (name == "model.embed_tokens.weight" || name == "lm_head.weight") return {V, H};
  if (name == "model.norm.weight") return {H};
  const std::string prefix = "model.layers.";
  const size_t dot = name.compare(0, prefix.size(), prefix) == 0 ? name.find('.', prefix.size()) : std::string::npos;
  const std::string suf = dot == std::string::npos ? "" : name.substr(dot + 1);
  if (suf == "input_layernorm.weight" || suf == "post_attention_layernorm.weight") return {H};
  if (suf == "self_attn.q_norm.weight" || suf == "self_attn.k_norm.weight") return {128};
  if (suf == "self_attn.q_proj.weight") return {Q, H};
  if (suf == "self_attn.k_proj.weight" || suf == "self_attn.v_proj.weight") return {KV, H};
  if (suf == "self_attn.o_proj.weight") return {H, Q};
  if (suf == "mlp.gate_proj.weight" || suf == "mlp.up_proj.weight") return {I, H};
  if (suf == "mlp.down_proj.weight") return {H, I};
  throw std::runtime_error("unknown Qwen3 tensor name: " + name);
}

// ------------------------------------------------------------------ config ----
void read_qwen3_config(const std::string &dir, xpu_qwen3_shape *out, uint32_t *eos_token_id) {
  const std::string file = dir + "/config.json";
  const std::string text = read_text(file, 1u << 24);
  const JValue root = JReader(text, file).document();
  if (root.type != JValue::Object) throw std::runtime_error(file + ": not a JSON object");
  xpu_qwen3_shape s{};
  s.hidden_size = u32_field(root, "hidden_size", file);
  s.intermediate_size = u32_field(root, "intermediate_size", file);
  s.num_hidden_layers = u32_field(root, "num_hidden_layers", file);
  s.num_attention_heads = u32_field(root, "num_attention_heads", file);
  s.num_key_value_heads = u32_field(root, "num_key_value_heads", file);
  s.vocab_size = u32_field(root, "vocab_size", file);
  s.rms_norm_eps = static_cast<float>(num_field(root, "rms_norm_eps", file));
  s.rope_theta = num_field(root, "rope_theta", file);
  const JValue &tie = field(root, "tie_word_embeddings", file);
  if (tie.type != JValue::Bool) throw std::runtime_error(file + ": 'tie_word_embeddings' must be true or false");
  s.tie_word_embeddings = tie.b ? 1 : 0;
  const uint32_t head_dim = root.get("head_dim") ? u32_field(root, "head_dim", file)
                                                 : (s.num_attention_heads ? s.hidden_size / s.num_attention_heads : 0);
  if (str_field(root, "model_type", file) != "qwen3")
    throw std::runtime_error(file + ": model_type must be \"qwen3\"");
  if (str_field(root, "hidden_act", file) != "silu") throw std::runtime_error(file + ": hidden_act must be \"silu\"");
  // transformers writes the weight dtype as torch_dtype (4.x) or dtype (5.x).
  const char *dtype_key = root.get("torch_dtype") ? "torch_dtype" : "dtype";
  if (str_field(root, dtype_key, file) != "bfloat16") throw std::runtime_error(file + ": weights must be bfloat16");
  if (head_dim != 128) throw std::runtime_error(file + ": head_dim must be 128, got " + std::to_string(head_dim));
  if (const JValue *rs = root.get("rope_scaling"); rs && rs->type != JValue::Null)
    throw std::runtime_error(file + ": rope_scaling is not supported");
  if (s.num_key_value_heads == 0 || s.num_attention_heads % s.num_key_value_heads != 0)
    throw std::runtime_error(file + ": num_attention_heads must be a multiple of num_key_value_heads");
  if (!(s.rms_norm_eps > 0.f) || !(s.rope_theta > 0.0))
    throw std::runtime_error(file + ": rms_norm_eps and rope_theta must be positive");
  if (eos_token_id) *eos_token_id = root.get("eos_token_id") ? u32_field(root, "eos_token_id", file) : 0;
  *out = s;
}

// ---------------------------------------------------------------- tensors ----
std::vector<CkptTensor> index_qwen3_checkpoint(const std::string &dir, const xpu_qwen3_shape &shape) {
  // weight_map: tensor name -> shard file name
  std::map<std::string, std::string> weight_map;
  bool have_total = false;
  uint64_t total_size = 0;
  const std::string index_file = dir + "/model.safetensors.index.json";
  if (file_exists(index_file)) {
    const std::string text = read_text(index_file, 1u << 28);
    const JValue root = JReader(text, index_file).document();
    const JValue *wm = root.get("weight_map");
    if (!wm || wm->type != JValue::Object) throw std::runtime_error(index_file + ": missing weight_map object");
    for (const auto &kv : wm->obj) {
      if (kv.second.type != JValue::String || kv.second.str.empty() || kv.second.str.find('/') != std::string::npos ||
          kv.second.str == "." || kv.second.str == "..")
        throw std::runtime_error(index_file + ": invalid shard name for tensor " + kv.first);
      weight_map[kv.first] = kv.second.str;
    }
    if (const JValue *md = root.get("metadata"); md && md->get("total_size")) {
      total_size = exact_u64(*md->get("total_size"), index_file + ": metadata.total_size");
      have_total = true;
    }
  } else if (!file_exists(dir + "/model.safetensors")) {
    throw std::runtime_error(dir + ": neither model.safetensors.index.json nor model.safetensors found");
  }
  const bool single = weight_map.empty();

  // Expected tensors and their global shapes.
  const std::vector<std::string> expected = qwen3_tensor_names(shape);
  const std::set<std::string> expected_set(expected.begin(), expected.end());
  if (!single) {
    for (const auto &kv : weight_map)
      if (!expected_set.count(kv.first)) throw std::runtime_error("unexpected tensor in checkpoint: " + kv.first);
    for (const std::string &n : expected)
      if (!weight_map.count(n)) throw std::runtime_error("checkpoint is missing tensor: " + n);
  }

  std::map<std::string, std::vector<std::string>> by_shard;
  if (single) by_shard["model.safetensors"] = {};
  else for (const auto &kv : weight_map) by_shard[kv.second].push_back(kv.first);

  std::map<std::string, CkptTensor> found;
  for (const auto &sh : by_shard) {
    const std::string path = dir + "/" + sh.first;
    Fd f(path);
    const uint64_t fsize = f.size();
    if (fsize < 8) throw std::runtime_error(path + ": too small for a safetensors header");
    uint8_t lenbuf[8];
    f.read(lenbuf, 8, 0);
    uint64_t hlen = 0;
    for (int k = 7; k >= 0; --k) hlen = (hlen << 8) | lenbuf[k];  // little-endian
    if (hlen == 0 || hlen > (1ull << 30) || hlen > fsize - 8)
      throw std::runtime_error(path + ": invalid safetensors header length " + std::to_string(hlen));
    std::string header(hlen, '\0');
    f.read(&header[0], hlen, 8);
    const JValue root = JReader(header, path).document();
    if (root.type != JValue::Object) throw std::runtime_error(path + ": safetensors header is not an object");
    const std::set<std::string> indexed(sh.second.begin(), sh.second.end());
    std::vector<std::pair<std::pair<uint64_t, uint64_t>, std::string>> spans;
    for (const auto &kv : root.obj) {
      const std::string &name = kv.first;
      if (name == "__metadata__") continue;
      if (single) {
        if (!expected_set.count(name)) throw std::runtime_error("unexpected tensor in checkpoint: " + name);
      } else if (!indexed.count(name)) {
        throw std::runtime_error(path + ": tensor " + name + " is not listed for this shard in the index");
      }
      const JValue &e = kv.second;
      const JValue *dt = e.get("dtype"), *shp = e.get("shape"), *off = e.get("data_offsets");
      if (!dt || dt->type != JValue::String || !shp || shp->type != JValue::Array || !off ||
          off->type != JValue::Array || off->arr.size() != 2)
        throw std::runtime_error(path + ": invalid metadata for tensor " + name);
      if (dt->str != "BF16")
        throw std::runtime_error("tensor " + name + " has dtype " + dt->str + "; BF16 is required");
      CkptTensor t;
      t.name = name;
      t.path = path;
      uint64_t elems = 1;
      for (const JValue &d : shp->arr) {
        const uint64_t n = exact_u64(d, "shape of " + name);
        if (n == 0 || elems > (~0ull) / n) throw std::runtime_error("invalid shape for tensor " + name);
        elems *= n;
        t.shape.push_back(n);
      }
      const uint64_t b0 = exact_u64(off->arr[0], "data_offsets of " + name);
      const uint64_t b1 = exact_u64(off->arr[1], "data_offsets of " + name);
      if (b1 < b0) throw std::runtime_error("invalid data_offsets for tensor " + name);
      t.offset = 8 + hlen + b0;
      t.bytes = b1 - b0;
      if (t.offset > fsize || t.bytes > fsize - t.offset)
        throw std::runtime_error("tensor " + name + " extends beyond " + path);
      if (t.bytes != elems * 2) throw std::runtime_error("byte size does not match the BF16 shape of " + name);
      spans.push_back({{t.offset, t.offset + t.bytes}, name});
      found[name] = std::move(t);
    }
    for (const std::string &n : sh.second)
      if (!found.count(n)) throw std::runtime_error("index lists tensor " + n + " that " + path + " does not hold");
    std::sort(spans.begin(), spans.end());
    for (size_t k = 1; k < spans.size(); ++k)
      if (spans[k].first.first < spans[k - 1].first.second)
        throw std::runtime_error("overlapping tensor payloads: " + spans[k - 1].second + " and " + spans[k].second);
  }

  std::vector<CkptTensor> out;
  uint64_t payload = 0;
  for (const std::string &n : expected) {
    auto it = found.find(n);
    if (it == found.end()) throw std::runtime_error("checkpoint is missing tensor: " + n);
    if (it->second.shape != qwen3_tensor_shape(shape, n)) {
      std::string got;
      for (uint64_t d : it->second.shape) got += (got.empty() ? "" : "x") + std::to_string(d);
      throw std::runtime_error("wrong shape for tensor " + n + ": " + got);
    }
    payload += it->second.bytes;
    out.push_back(std::move(it->second));
  }
  if (have_total && total_size != payload)
    throw std::runtime_error(index_file + ": total_size " + std::to_string(total_size) +
                             " does not match the tensor payloads (" + std::to_string(payload) + " bytes)");
  return out;
}

}  // namespace xpu

// ------------------------------------------------------------------ C ABI ----
extern "C" int xpu_qwen3_read_config(const char *model_dir, xpu_qwen3_shape *shape) {
  try {
    if (!model_dir || !shape) return xpu::fail(XPU_ERR_INVALID, "xpu_qwen3_read_config: null pointer");
    xpu::read_qwen3_config(model_dir, shape, nullptr);
    return XPU_OK;
  } catch (const std::exception &e) {
    return xpu::fail(XPU_ERR_INVALID, e.what());
  }
}

extern "C" int xpu_qwen3_validate_checkpoint(const char *model_dir, xpu_qwen3_shape *shape, uint64_t *payload_bytes) {
  try {
    if (!model_dir || !shape) return xpu::fail(XPU_ERR_INVALID, "xpu_qwen3_validate_checkpoint: null pointer");
    xpu::read_qwen3_config(model_dir, shape, nullptr);
    const std::vector<xpu::CkptTensor> t = xpu::index_qwen3_checkpoint(model_dir, *shape);
    if (payload_bytes) {
      *payload_bytes = 0;
      for (const auto &x : t) *payload_bytes += x.bytes;
    }
    return XPU_OK;
  } catch (const std::exception &e) {
    return xpu::fail(XPU_ERR_INVALID, e.what());
  }
}
