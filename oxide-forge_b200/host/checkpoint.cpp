// checkpoint.cpp — the reference's two-file checkpoint format, version 1.
//
//   <name>.toml  format_version = 1, model_type, scalar_type = "f32_le",
//                data_file, data_bytes, then the model's metadata tables
//                (LinearMetadata linear.rs:79-86, MlpMetadata mlp.rs:22-34,
//                TransformerMetadata inference.rs:13-24, MatrixMetadata /
//                VectorMetadata metadata.rs:5-19) with [byte_start, byte_end)
//                ranges laid out contiguously in cursor order
//   <name>.bin   the parameters as little-endian f32, nothing else
//
// The metadata is TOML written the way the reference's serializer lays out
// nested structs: plain keys first, then one [table] per nested struct and
// one [[array-of-tables]] entry per MLP layer. The reader accepts any TOML
// of the same shape (tables, dotted keys, inline tables that may span lines
// as TOML 1.1 allows, arrays of inline tables); only integers, strings and
// booleans occur in the schema.
#include "checkpoint.hpp"

#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <sstream>

#include "runtime.hpp"

namespace oxf::ckpt {
namespace {

constexpr long long kFormatVersion = 1;          // model.rs:17
constexpr const char* kScalarType = "f32_le";    // model.rs:18

[[noreturn]] void fail(const std::string& msg) { throw Error(OXF_ERR_INVALID_ARG, msg); }
[[noreturn]] void fail_io(const std::string& msg) { throw Error(OXF_ERR_STATE, msg); }

const char* model_type_name(ModelType t) {  // model.rs:19-21
  switch (t) {
    case ModelType::Linear: return "linear";
    case ModelType::Mlp: return "mlp";
    default: return "transformer";
  }
}

// Activation / NormType / Loss serialise as snake_case unit variants
// (linear.rs:12-19, transformer.rs:7-13, mlp.rs:8-12).
const char* activation_name(int act) {
  switch (act) {
    case OXF_ACT_GELU: return "gelu";
    case OXF_ACT_RELU: return "relu";
    case OXF_ACT_SILU: return "silu";
    default: return "identity";
  }
}
int activation_from(const std::string& s) {
  if (s == "identity") return OXF_ACT_IDENTITY;
  if (s == "gelu") return OXF_ACT_GELU;
  if (s == "relu") return OXF_ACT_RELU;
  if (s == "silu") return OXF_ACT_SILU;
  fail("unknown variant `" + s + "`, expected one of `identity`, `gelu`, `relu`, `silu`");
}
int norm_from(const std::string& s) {
  if (s == "rms") return OXF_NORM_RMS;
  if (s == "layer") return OXF_NORM_LAYER;
  fail("unknown variant `" + s + "`, expected `rms` or `layer`");
}

// ------------------------------------------------------------------ TOML values
struct Value;
using Table = std::map<std::string, Value>;

struct Value {
  enum Kind { Int, Str, Bool, Tab, Arr } kind = Int;
  long long i = 0;
  std::string s;
  bool b = false;
  std::shared_ptr<Table> t;
  std::vector<Value> a;
  bool array_of_tables = false;  // created by [[...]] headers
};

Value make_table() {
  Value v;
  v.kind = Value::Tab;
  v.t = std::make_shared<Table>();
  return v;
}

class Parser {
 public:
  explicit Parser(const std::string& text) : s_(text) {}

  Value document() {
    Value root = make_table();
    Table* cur = root.t.get();
    for (;;) {
      skip_blank_lines();
      if (eof()) break;
      if (peek() == '[') {
        ++p_;
        const bool arr = peek() == '[';
        if (arr) ++p_;
        skip_ws();
        std::vector<std::string> path = key_path();
        skip_ws();
        expect(']');
        if (arr) expect(']');
        cur = arr ? append_array_table(root, path) : open_table(root, path);
      } else {
        std::vector<std::string> path = key_path();
        skip_ws();
        expect('=');
        skip_ws();
        Value v = value();
        Table* t = cur;
        for (size_t k = 0; k + 1 < path.size(); ++k) t = descend(t, path[k]);
        if (t->count(path.back())) fail(err("duplicate key `" + path.back() + "`"));
        (*t)[path.back()] = std::move(v);
      }
      end_of_line();
    }
    return root;
  }

 private:
  const std::string& s_;
  size_t p_ = 0;

  bool eof() const { return p_ >= s_.size(); }
  char peek() const { return eof() ? '\0' : s_[p_]; }
  std::string err(const std::string& m) const {
    size_t line = 1;
    for (size_t i = 0; i < p_ && i < s_.size(); ++i) line += s_[i] == '\n';
    return "TOML parse error at line " + std::to_string(line) + ": " + m;
  }
  void expect(char c) {
    if (peek() != c) fail(err(std::string("expected `") + c + "`"));
    ++p_;
  }
  void skip_ws() {
    while (!eof() && (peek() == ' ' || peek() == '\t')) ++p_;
  }
  void skip_comment() {
    if (peek() == '#')
      while (!eof() && peek() != '\n') ++p_;
  }
  void skip_blank_lines() {
    for (;;) {
      skip_ws();
      skip_comment();
      if (peek() == '\r') ++p_;
      if (peek() == '\n') {
        ++p_;
        continue;
      }
      return;
    }
  }
  // whitespace, newlines and comments inside arrays
  void skip_array_space() {
    for (;;) {
      skip_ws();
      skip_comment();
      if (peek() == '\r' || peek() == '\n') {
        ++p_;
        continue;
      }
      return;
    }
  }
  void end_of_line() {
    skip_ws();
    skip_comment();
    if (peek() == '\r') ++p_;
    if (eof()) return;
    if (peek() != '\n') fail(err("expected the end of the line"));
    ++p_;
  }

  static bool bare(char c) {
    return (c >= 'A' && c <= 'Z') || (c >= 'a' && c <= 'z') || (c >= '0' && c <= '9') ||
           c == '_' || c == '-';
  }
  std::string key() {
    if (peek() == '"') return basic_string();
    if (peek() == '\'') return literal_string();
    const size_t b = p_;
    while (!eof() && bare(peek())) ++p_;
    if (p_ == b) fail(err("expected a key"));
    return s_.substr(b, p_ - b);
  }
  std::vector<std::string> key_path() {
    std::vector<std::string> path{key()};
    for (;;) {
      skip_ws();
      if (peek() != '.') return path;
      ++p_;
      skip_ws();
      path.push_back(key());
    }
  }

  static void put_utf8(std::string& out, uint32_t cp) {
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
  std::string basic_string() {
    expect('"');
    std::string out;
    for (;;) {
      if (eof() || peek() == '\n') fail(err("unterminated string"));
      const char c = s_[p_++];
      if (c == '"') return out;
      if (c != '\\') {
        out += c;
        continue;
      }
      const char e = eof() ? '\0' : s_[p_++];
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case 'b': out += '\b'; break;
        case 't': out += '\t'; break;
        case 'n': out += '\n'; break;
        case 'f': out += '\f'; break;
        case 'r': out += '\r'; break;
        case 'u':
        case 'U': {
          const int n = e == 'u' ? 4 : 8;
          if (p_ + n > s_.size()) fail(err("truncated unicode escape"));
          uint32_t cp = 0;
          for (int k = 0; k < n; ++k) {
            const char h = s_[p_++];
            cp <<= 4;
            if (h >= '0' && h <= '9') cp |= h - '0';
            else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
            else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
            else fail(err("bad unicode escape"));
          }
          put_utf8(out, cp);
          break;
        }
        default: fail(err("bad escape sequence"));
      }
    }
  }
  std::string literal_string() {
    expect('\'');
    const size_t b = p_;
    while (!eof() && peek() != '\'' && peek() != '\n') ++p_;
    if (peek() != '\'') fail(err("unterminated string"));
    return s_.substr(b, p_++ - b);
  }

  Value value() {
    Value v;
    const char c = peek();
    if (c == '"' || c == '\'') {
      v.kind = Value::Str;
      v.s = c == '"' ? basic_string() : literal_string();
    } else if (s_.compare(p_, 4, "true") == 0 && !bare(p_ + 4 < s_.size() ? s_[p_ + 4] : ' ')) {
      v.kind = Value::Bool;
      v.b = true;
      p_ += 4;
    } else if (s_.compare(p_, 5, "false") == 0 &&
               !bare(p_ + 5 < s_.size() ? s_[p_ + 5] : ' ')) {
      v.kind = Value::Bool;
      p_ += 5;
    } else if (c == '{') {
      // Inline table; as in TOML 1.1 it may span lines and end with a comma.
      ++p_;
      v = make_table();
      for (;;) {
        skip_array_space();
        if (peek() == '}') {
          ++p_;
          return v;
        }
        std::vector<std::string> path = key_path();
        skip_ws();
        expect('=');
        skip_ws();
        Value item = value();
        Table* t = v.t.get();
        for (size_t k = 0; k + 1 < path.size(); ++k) t = descend(t, path[k]);
        if (t->count(path.back())) fail(err("duplicate key `" + path.back() + "`"));
        (*t)[path.back()] = std::move(item);
        skip_array_space();
        if (peek() == ',') {
          ++p_;
          continue;
        }
        expect('}');
        return v;
      }
    } else if (c == '[') {
      ++p_;
      v.kind = Value::Arr;
      for (;;) {
        skip_array_space();
        if (peek() == ']') {
          ++p_;
          return v;
        }
        v.a.push_back(value());
        skip_array_space();
        if (peek() == ',') {
          ++p_;
          continue;
        }
        expect(']');
        return v;
      }
    } else if (c == '+' || c == '-' || (c >= '0' && c <= '9')) {
      v.kind = Value::Int;
      bool neg = false;
      if (c == '+' || c == '-') {
        neg = c == '-';
        ++p_;
      }
      unsigned long long mag = 0;
      int digits = 0;
      while (!eof() && ((peek() >= '0' && peek() <= '9') || peek() == '_')) {
        if (peek() != '_') {
          const unsigned d = static_cast<unsigned>(peek() - '0');
          if (mag > (~0ull - d) / 10) fail(err("integer out of range"));
          mag = mag * 10 + d;
          ++digits;
        }
        ++p_;
      }
      if (digits == 0) fail(err("expected a value"));
      if (peek() == '.' || peek() == 'e' || peek() == 'E')
        fail(err("floating-point values do not occur in a checkpoint"));
      if (mag > static_cast<unsigned long long>(INT64_MAX)) fail(err("integer out of range"));
      v.i = neg ? -static_cast<long long>(mag) : static_cast<long long>(mag);
    } else {
      fail(err("expected a value"));
    }
    return v;
  }

  Table* descend(Table* t, const std::string& k) {
    auto it = t->find(k);
    if (it == t->end()) it = t->emplace(k, make_table()).first;
    Value& v = it->second;
    if (v.kind == Value::Tab) return v.t.get();
    if (v.kind == Value::Arr && v.array_of_tables && !v.a.empty()) return v.a.back().t.get();
    fail(err("key `" + k + "` is not a table"));
  }
  Table* open_table(Value& root, const std::vector<std::string>& path) {
    Table* t = root.t.get();
    for (const std::string& k : path) t = descend(t, k);
    return t;
  }
  Table* append_array_table(Value& root, const std::vector<std::string>& path) {
    Table* t = root.t.get();
    for (size_t k = 0; k + 1 < path.size(); ++k) t = descend(t, path[k]);
    auto it = t->find(path.back());
    if (it == t->end()) {
      Value arr;
      arr.kind = Value::Arr;
      arr.array_of_tables = true;
      it = t->emplace(path.back(), std::move(arr)).first;
    }
    Value& arr = it->second;
    if (arr.kind != Value::Arr || !arr.array_of_tables)
      fail(err("key `" + path.back() + "` is not an array of tables"));
    arr.a.push_back(make_table());
    return arr.a.back().t.get();
  }
};

// ------------------------------------------------------------------ typed access
const Value& field(const Table& t, const char* name) {
  auto it = t.find(name);
  if (it == t.end()) fail(std::string("missing field `") + name + "`");
  return it->second;
}
const Value* optional_field(const Table& t, const char* name) {
  auto it = t.find(name);
  return it == t.end() ? nullptr : &it->second;
}
long long get_uint(const Table& t, const char* name) {
  const Value& v = field(t, name);
  if (v.kind != Value::Int) fail(std::string("field `") + name + "` must be an integer");
  if (v.i < 0) fail(std::string("field `") + name + "` must not be negative");
  return v.i;
}
std::string get_str(const Table& t, const char* name) {
  const Value& v = field(t, name);
  if (v.kind != Value::Str) fail(std::string("field `") + name + "` must be a string");
  return v.s;
}
bool get_bool(const Table& t, const char* name) {
  const Value& v = field(t, name);
  if (v.kind != Value::Bool) fail(std::string("field `") + name + "` must be a boolean");
  return v.b;
}
const Table& get_table(const Table& t, const char* name) {
  const Value& v = field(t, name);
  if (v.kind != Value::Tab) fail(std::string("field `") + name + "` must be a table");
  return *v.t;
}

// ------------------------------------------------------------------ metadata
struct MatrixMeta {
  long long rows = 0, cols = 0, start = 0, end = 0;
};
struct VectorMeta {
  long long len = 0, start = 0, end = 0;
};
struct LinearMeta {
  long long in = 0, out = 0;
  int act = OXF_ACT_IDENTITY;
  MatrixMeta w;
  bool has_bias = false;
  VectorMeta b;
};
struct MlpMeta {
  long long layer_count = 0;
  bool has_res = false;
  long long res_start = 0, res_end = 0;
  std::vector<LinearMeta> layers;
};
struct TransformerMeta {
  long long block_count = 1;
  bool attention_residual = true, feed_forward_residual = true;
  int norm = OXF_NORM_LAYER;
  MatrixMeta pos;
  LinearMeta q, k, v;
  MlpMeta ffn;
  LinearMeta o;
};

MatrixMeta matrix_from(const Table& t) {
  return {get_uint(t, "rows"), get_uint(t, "cols"), get_uint(t, "byte_start"),
          get_uint(t, "byte_end")};
}
VectorMeta vector_from(const Table& t) {
  return {get_uint(t, "len"), get_uint(t, "byte_start"), get_uint(t, "byte_end")};
}
LinearMeta linear_from(const Table& t) {
  LinearMeta m;
  m.in = get_uint(t, "input_neurons");
  m.out = get_uint(t, "output_neurons");
  m.act = activation_from(get_str(t, "activation"));
  m.w = matrix_from(get_table(t, "weights"));
  if (const Value* b = optional_field(t, "bias")) {
    if (b->kind != Value::Tab) fail("field `bias` must be a table");
    m.has_bias = true;
    m.b = vector_from(*b->t);
  }
  return m;
}
MlpMeta mlp_from(const Table& t) {
  MlpMeta m;
  m.layer_count = get_uint(t, "layer_count");
  const std::string loss = get_str(t, "loss");
  if (loss != "mean_squared_error")
    fail("unknown variant `" + loss + "`, expected `mean_squared_error`");
  if (const Value* r = optional_field(t, "residual")) {
    if (r->kind != Value::Tab) fail("field `residual` must be a table");
    m.has_res = true;
    m.res_start = get_uint(*r->t, "start");
    m.res_end = get_uint(*r->t, "end");
  }
  const Value& layers = field(t, "layers");
  if (layers.kind != Value::Arr) fail("field `layers` must be an array");
  for (const Value& l : layers.a) {
    if (l.kind != Value::Tab) fail("MLP layers must be tables");
    m.layers.push_back(linear_from(*l.t));
  }
  return m;
}
TransformerMeta transformer_from(const Table& t) {
  TransformerMeta m;
  m.block_count = get_uint(t, "block_count");
  m.attention_residual = get_bool(t, "attention_residual");
  m.feed_forward_residual = get_bool(t, "feed_forward_residual");
  m.norm = norm_from(get_str(t, "normalization"));
  m.pos = matrix_from(get_table(t, "position"));
  m.q = linear_from(get_table(t, "query"));
  m.k = linear_from(get_table(t, "key"));
  m.v = linear_from(get_table(t, "value"));
  m.ffn = mlp_from(get_table(t, "feed_forward"));
  m.o = linear_from(get_table(t, "output"));
  return m;
}

// RangeValidator (model.rs:486-537): every parameter occupies the next
// contiguous byte range.
struct Ranges {
  unsigned long long position = 0;
  void range(long long start, long long end, unsigned long long elements) {
    if (elements > (~0ull) / 4) fail("parameter byte length overflow");
    const unsigned long long bytes = elements * 4;
    if (position > ~0ull - bytes) fail("checkpoint offset overflow");
    const unsigned long long expected_end = position + bytes;
    if (static_cast<unsigned long long>(start) != position ||
        static_cast<unsigned long long>(end) != expected_end)
      fail("parameter range [" + std::to_string(start) + ", " + std::to_string(end) +
           ") is not the expected contiguous range [" + std::to_string(position) + ", " +
           std::to_string(expected_end) + ")");
    position = expected_end;
  }
  void matrix(const MatrixMeta& m) {
    const unsigned long long r = static_cast<unsigned long long>(m.rows);
    const unsigned long long c = static_cast<unsigned long long>(m.cols);
    if (c != 0 && r > (~0ull) / c) fail("matrix element count overflow");
    range(m.start, m.end, r * c);
  }
  void vector(const VectorMeta& v) { range(v.start, v.end, static_cast<unsigned long long>(v.len)); }
};

// validate_linear (model.rs:425-442)
void validate(const LinearMeta& m, Ranges& r) {
  if (m.in == 0 || m.out == 0) fail("Linear dimensions must be non-zero");
  if (m.w.rows != m.in || m.w.cols != m.out)
    fail("Linear weight shape does not match its neuron counts");
  r.matrix(m.w);
  if (m.has_bias) {
    if (m.b.len != m.out) fail("Linear bias length does not match output neurons");
    r.vector(m.b);
  }
}

// validate_mlp (model.rs:389-423)
void validate(const MlpMeta& m, Ranges& r) {
  if (m.layer_count == 0 || m.layer_count != static_cast<long long>(m.layers.size()))
    fail("MLP layer_count is " + std::to_string(m.layer_count) + ", but " +
         std::to_string(m.layers.size()) + " layers are described");
  for (size_t i = 0; i < m.layers.size(); ++i) {
    validate(m.layers[i], r);
    if (i > 0 && m.layers[i - 1].out != m.layers[i].in)
      fail("MLP layer " + std::to_string(i) + " expects " + std::to_string(m.layers[i].in) +
           " neurons, previous layer produces " + std::to_string(m.layers[i - 1].out));
  }
  if (m.has_res) {
    if (m.res_start >= m.res_end || m.res_end > static_cast<long long>(m.layers.size()))
      fail("invalid MLP residual range");
    const long long in = m.layers[m.res_start].in, out = m.layers[m.res_end - 1].out;
    if (in != out)
      fail("residual connects " + std::to_string(in) + " input neurons to " +
           std::to_string(out) + " output neurons");
  }
}

// validate_transformer (model.rs:444-484)
void validate(const TransformerMeta& m, Ranges& r) {
  if (m.block_count != 1) fail("this Transformer executor requires exactly one block");
  if (!m.attention_residual || !m.feed_forward_residual)
    fail("this Transformer executor requires both residual paths");
  validate(m.q, r);
  validate(m.k, r);
  validate(m.v, r);
  r.matrix(m.pos);
  validate(m.ffn, r);
  validate(m.o, r);
  const long long emb = m.pos.cols;
  if (m.pos.rows == 0 || emb == 0) fail("position matrix dimensions must be non-zero");
  if (m.q.in != emb || m.k.in != emb || m.v.in != emb)
    fail("Q/K/V input dimensions must match the embedding size");
  if (m.q.out != m.k.out) fail("query and key dimensions must match");
  if (m.v.out != emb) fail("value output dimension must match the residual embedding");
  if (m.ffn.layers.front().in != emb || m.ffn.layers.back().out != emb)
    fail("feed-forward input/output must match the embedding size");
  if (m.o.in != emb) fail("output projection input must match the embedding size");
}

// ------------------------------------------------------------------ spec <-> metadata
int narrow(long long v, const char* what) {
  if (v > 0x7fffffffll) fail(std::string(what) + " exceeds this build's 32-bit dimensions");
  return static_cast<int>(v);
}
oxf_layer_spec to_spec(const LinearMeta& m) {
  oxf_layer_spec s{};
  s.in = narrow(m.in, "Linear input_neurons");
  s.out = narrow(m.out, "Linear output_neurons");
  s.act = m.act;
  s.bias = m.has_bias ? 1 : 0;
  return s;
}
oxf_mlp_spec to_spec(const MlpMeta& m) {
  if (m.layers.size() > OXF_MAX_LAYERS)
    throw Error(OXF_ERR_UNSUPPORTED_SHAPE,
                "checkpoint MLP has " + std::to_string(m.layers.size()) +
                    " layers; this build's executors hold at most " +
                    std::to_string(OXF_MAX_LAYERS));
  oxf_mlp_spec s{};
  s.n_layers = static_cast<int>(m.layers.size());
  for (size_t i = 0; i < m.layers.size(); ++i) s.layers[i] = to_spec(m.layers[i]);
  s.res_start = m.has_res ? static_cast<int>(m.res_start) : -1;
  s.res_end = m.has_res ? static_cast<int>(m.res_end) : -1;
  return s;
}

// MetadataCursor (metadata.rs:21-68): ranges handed out in call order.
struct Cursor {
  long long pos = 0;
  MatrixMeta matrix(long long rows, long long cols) {
    MatrixMeta m{rows, cols, pos, pos + rows * cols * 4};
    pos = m.end;
    return m;
  }
  VectorMeta vector(long long len) {
    VectorMeta v{len, pos, pos + len * 4};
    pos = v.end;
    return v;
  }
};
void check_spec(const oxf_layer_spec& s) {
  if (s.in <= 0 || s.out <= 0) fail("Linear dimensions must be positive");
  if (s.act < OXF_ACT_IDENTITY || s.act > OXF_ACT_SILU) fail("unknown activation");
}
LinearMeta linear_meta(const oxf_layer_spec& s, Cursor& c) {  // Linear::get_meta_data
  check_spec(s);
  LinearMeta m;
  m.in = s.in;
  m.out = s.out;
  m.act = s.act;
  m.w = c.matrix(s.in, s.out);
  m.has_bias = s.bias != 0;
  if (m.has_bias) m.b = c.vector(s.out);
  return m;
}
MlpMeta mlp_meta(const oxf_mlp_spec& s, Cursor& c) {
  if (s.n_layers < 1 || s.n_layers > OXF_MAX_LAYERS) fail("MLP layer count");
  MlpMeta m;
  m.layer_count = s.n_layers;
  for (int i = 0; i < s.n_layers; ++i) m.layers.push_back(linear_meta(s.layers[i], c));
  m.has_res = s.res_start >= 0;
  m.res_start = s.res_start;
  m.res_end = s.res_end;
  return m;
}
TransformerMeta transformer_meta(const oxf_transformer_spec& s, Cursor& c) {
  TransformerMeta m;
  m.norm = s.norm;
  if (s.norm != OXF_NORM_RMS && s.norm != OXF_NORM_LAYER) fail("unknown NormType");
  if (s.seq <= 0 || s.hidden <= 0) fail("position matrix dimensions must be positive");
  m.q = linear_meta(s.q, c);
  m.k = linear_meta(s.k, c);
  m.v = linear_meta(s.v, c);
  m.pos = c.matrix(s.seq, s.hidden);
  m.ffn = mlp_meta(s.ffn, c);
  m.o = linear_meta(s.out, c);
  return m;
}

// ------------------------------------------------------------------ TOML writer
void put_matrix(std::ostringstream& o, const std::string& name, const MatrixMeta& m) {
  o << "\n[" << name << "]\nrows = " << m.rows << "\ncols = " << m.cols
    << "\nbyte_start = " << m.start << "\nbyte_end = " << m.end << "\n";
}
void put_linear(std::ostringstream& o, const std::string& name, const LinearMeta& m,
                bool array_entry) {
  o << "\n" << (array_entry ? "[[" : "[") << name << (array_entry ? "]]" : "]")
    << "\ninput_neurons = " << m.in << "\noutput_neurons = " << m.out << "\nactivation = \""
    << activation_name(m.act) << "\"\n";
  put_matrix(o, name + ".weights", m.w);
  if (m.has_bias)
    o << "\n[" << name << ".bias]\nlen = " << m.b.len << "\nbyte_start = " << m.b.start
      << "\nbyte_end = " << m.b.end << "\n";
}
void put_mlp(std::ostringstream& o, const std::string& name, const MlpMeta& m) {
  o << "\n[" << name << "]\nlayer_count = " << m.layer_count
    << "\nloss = \"mean_squared_error\"\n";
  if (m.has_res)
    o << "\n[" << name << ".residual]\nstart = " << m.res_start << "\nend = " << m.res_end
      << "\n";
  for (const LinearMeta& l : m.layers) put_linear(o, name + ".layers", l, true);
}

std::string quoted(const std::string& s) {
  std::string out = "\"";
  for (char c : s) {
    if (c == '"' || c == '\\') out += '\\';
    out += c;
  }
  return out + "\"";
}

// ------------------------------------------------------------------ paths (io.rs:14-50)
struct Paths {
  std::string metadata, data, data_name;
};
size_t name_start(const std::string& p) {
  const size_t slash = p.find_last_of('/');
  return slash == std::string::npos ? 0 : slash + 1;
}
// extension of the file name, or npos when it has none (a leading dot
// alone does not start one)
size_t extension_dot(const std::string& p) {
  const size_t b = name_start(p);
  const size_t dot = p.find_last_of('.');
  if (dot == std::string::npos || dot <= b) return std::string::npos;
  return dot;
}
std::string normalize_metadata_path(const std::string& path) {
  if (path.empty() || name_start(path) == path.size())
    fail("checkpoint path has no file name");
  const size_t dot = extension_dot(path);
  if (dot == std::string::npos) return path + ".toml";
  const std::string ext = path.substr(dot + 1);
  if (ext == "toml") return path;
  fail("checkpoint metadata must use .toml, not ." + ext);
}
Paths checkpoint_paths(const std::string& path) {
  Paths p;
  p.metadata = normalize_metadata_path(path);
  p.data = p.metadata.substr(0, extension_dot(p.metadata)) + ".bin";
  p.data_name = p.data.substr(name_start(p.data));
  return p;
}
std::string resolve_data_path(const std::string& metadata_path, const std::string& data_file) {
  if (data_file.empty() || data_file == "." || data_file == ".." ||
      data_file.find('/') != std::string::npos)
    fail("checkpoint data_file must be a plain file name");
  return metadata_path.substr(0, name_start(metadata_path)) + data_file;
}

std::string read_text(const std::string& path) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) fail_io("cannot open " + path + ": " + std::strerror(errno));
  std::string text;
  char buf[1 << 14];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, n);
  const bool bad = std::ferror(f) != 0;
  std::fclose(f);
  if (bad) fail_io("cannot read " + path);
  return text;
}

void write_file(const std::string& path, const void* data, size_t bytes) {
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) fail_io("cannot create " + path + ": " + std::strerror(errno));
  const bool ok = std::fwrite(data, 1, bytes, f) == bytes;
  const bool closed = std::fclose(f) == 0;
  if (!ok || !closed) fail_io("cannot write " + path);
}

bool little_endian() {
  const uint32_t one = 1;
  unsigned char b;
  std::memcpy(&b, &one, 1);
  return b == 1;
}

void write_le_f32(const std::string& path, const std::vector<float>& values) {
  if (little_endian()) {
    write_file(path, values.data(), values.size() * sizeof(float));
    return;
  }
  std::vector<unsigned char> bytes(values.size() * 4);
  for (size_t i = 0; i < values.size(); ++i) {
    uint32_t u;
    std::memcpy(&u, &values[i], 4);
    for (int k = 0; k < 4; ++k) bytes[4 * i + k] = static_cast<unsigned char>(u >> (8 * k));
  }
  write_file(path, bytes.data(), bytes.size());
}

}  // namespace

size_t param_count(const oxf_layer_spec& s) {
  return static_cast<size_t>(s.in) * s.out + (s.bias ? static_cast<size_t>(s.out) : 0);
}
size_t param_count(const oxf_mlp_spec& s) {
  size_t n = 0;
  for (int i = 0; i < s.n_layers && i < OXF_MAX_LAYERS; ++i) n += param_count(s.layers[i]);
  return n;
}
size_t param_count(const oxf_transformer_spec& s) {
  return param_count(s.q) + param_count(s.k) + param_count(s.v) +
         static_cast<size_t>(s.seq) * s.hidden + param_count(s.ffn) + param_count(s.out);
}

void write(const std::string& path, const Model& model) {
  const Paths p = checkpoint_paths(path);
  Cursor cursor;
  std::ostringstream body;
  size_t count = 0;
  switch (model.type) {
    case ModelType::Linear: {
      const LinearMeta m = linear_meta(model.linear, cursor);
      Ranges r;
      validate(m, r);
      put_linear(body, "linear", m, false);
      count = param_count(model.linear);
      break;
    }
    case ModelType::Mlp: {
      const MlpMeta m = mlp_meta(model.mlp, cursor);
      Ranges r;
      validate(m, r);
      put_mlp(body, "mlp", m);
      count = param_count(model.mlp);
      break;
    }
    case ModelType::Transformer: {
      const TransformerMeta m = transformer_meta(model.transformer, cursor);
      Ranges r;
      validate(m, r);
      body << "\n[transformer]\nblock_count = 1\nattention_residual = true\n"
              "feed_forward_residual = true\nnormalization = \""
           << (m.norm == OXF_NORM_RMS ? "rms" : "layer") << "\"\n";
      put_matrix(body, "transformer.position", m.pos);
      put_linear(body, "transformer.query", m.q, false);
      put_linear(body, "transformer.key", m.k, false);
      put_linear(body, "transformer.value", m.v, false);
      put_mlp(body, "transformer.feed_forward", m.ffn);
      put_linear(body, "transformer.output", m.o, false);
      count = param_count(model.transformer);
      break;
    }
  }
  // write_parameters (io.rs:66-89): the exported bytes must match the metadata.
  if (model.params.size() != count || static_cast<long long>(count) * 4 != cursor.pos)
    fail("model exported " + std::to_string(model.params.size() * 4) +
         " parameter bytes, metadata declares " + std::to_string(cursor.pos));
  std::ostringstream head;
  head << "format_version = " << kFormatVersion << "\nmodel_type = \""
       << model_type_name(model.type) << "\"\nscalar_type = \"" << kScalarType
       << "\"\ndata_file = " << quoted(p.data_name) << "\ndata_bytes = " << cursor.pos << "\n"
       << body.str();
  const std::string text = head.str();
  write_file(p.metadata, text.data(), text.size());
  write_le_f32(p.data, model.params);
}

Model read(const std::string& path, ModelType expected) {
  const std::string meta_path = normalize_metadata_path(path);
  const Value doc = Parser(read_text(meta_path)).document();
  const Table& root = *doc.t;
  // validate_header (model.rs:350-375)
  const long long version = get_uint(root, "format_version");
  const std::string model_type = get_str(root, "model_type");
  const std::string scalar_type = get_str(root, "scalar_type");
  const std::string data_file = get_str(root, "data_file");
  const long long data_bytes = get_uint(root, "data_bytes");
  if (version != kFormatVersion)
    fail("unsupported checkpoint format version " + std::to_string(version) + "; expected " +
         std::to_string(kFormatVersion));
  if (model_type != model_type_name(expected))
    fail("checkpoint contains model type \"" + model_type + "\", expected \"" +
         model_type_name(expected) + "\"");
  if (scalar_type != kScalarType)
    fail("unsupported scalar encoding \"" + scalar_type + "\"; expected \"f32_le\"");

  Model model;
  model.type = expected;
  Ranges r;
  switch (expected) {
    case ModelType::Linear: {
      const LinearMeta m = linear_from(get_table(root, "linear"));
      validate(m, r);
      model.linear = to_spec(m);
      break;
    }
    case ModelType::Mlp: {
      const MlpMeta m = mlp_from(get_table(root, "mlp"));
      validate(m, r);
      model.mlp = to_spec(m);
      break;
    }
    case ModelType::Transformer: {
      const TransformerMeta m = transformer_from(get_table(root, "transformer"));
      validate(m, r);
      model.transformer.seq = narrow(m.pos.rows, "position rows");
      model.transformer.hidden = narrow(m.pos.cols, "position cols");
      model.transformer.norm = m.norm;
      model.transformer.q = to_spec(m.q);
      model.transformer.k = to_spec(m.k);
      model.transformer.v = to_spec(m.v);
      model.transformer.ffn = to_spec(m.ffn);
      model.transformer.out = to_spec(m.o);
      break;
    }
  }
  if (r.position != static_cast<unsigned long long>(data_bytes))
    fail("parameter ranges end at " + std::to_string(r.position) + ", metadata declares " +
         std::to_string(data_bytes) + " bytes");

  // ParameterReader (io.rs:126-177): the data file holds exactly data_bytes.
  const std::string data_path = resolve_data_path(meta_path, data_file);
  FILE* f = std::fopen(data_path.c_str(), "rb");
  if (!f) fail_io("cannot open " + data_path + ": " + std::strerror(errno));
  std::fseek(f, 0, SEEK_END);
  const long long file_len = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  if (file_len != data_bytes) {
    std::fclose(f);
    fail("data file has " + std::to_string(file_len) + " bytes, metadata declares " +
         std::to_string(data_bytes));
  }
  const size_t n = static_cast<size_t>(data_bytes / 4);
  std::vector<unsigned char> bytes(static_cast<size_t>(data_bytes));
  const bool ok = std::fread(bytes.data(), 1, bytes.size(), f) == bytes.size();
  std::fclose(f);
  if (!ok) fail_io("cannot read " + data_path);
  model.params.resize(n);
  for (size_t i = 0; i < n; ++i) {
    const uint32_t u = static_cast<uint32_t>(bytes[4 * i]) |
                       (static_cast<uint32_t>(bytes[4 * i + 1]) << 8) |
                       (static_cast<uint32_t>(bytes[4 * i + 2]) << 16) |
                       (static_cast<uint32_t>(bytes[4 * i + 3]) << 24);
    std::memcpy(&model.params[i], &u, 4);
  }
  return model;
}

}  // namespace oxf::ckpt
