// StableHLO text -> IR.  A recursive-descent parser over the whole text (not a
// line-by-line regex matcher like reference src/mlx_mlir_parser.h:36-2410).
// Accepts the pretty printing that jax.jit(...).lower().as_text() and
// mlirOperationPrint produce, and the generic "stablehlo.op"(...) form.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <sstream>
#include <unordered_map>

#include "ir.h"

namespace b200 {

// ----------------------------------------------------------------- dtypes --
int dtype_size(DType t) {
  switch (t) {
    case DType::PRED: case DType::S8: case DType::U8: return 1;
    case DType::S16: case DType::U16: case DType::F16: case DType::BF16: return 2;
    case DType::S32: case DType::U32: case DType::F32: return 4;
    case DType::S64: case DType::U64: case DType::F64: return 8;
    default: return 0;
  }
}
const char* dtype_name(DType t) {
  switch (t) {
    case DType::PRED: return "i1"; case DType::S8: return "i8"; case DType::S16: return "i16";
    case DType::S32: return "i32"; case DType::S64: return "i64"; case DType::U8: return "ui8";
    case DType::U16: return "ui16"; case DType::U32: return "ui32"; case DType::U64: return "ui64";
    case DType::F16: return "f16"; case DType::F32: return "f32"; case DType::F64: return "f64";
    case DType::BF16: return "bf16"; case DType::TOKEN: return "token";
    default: return "invalid";
  }
}
DType dtype_from_mlir(const std::string& s) {
  static const std::unordered_map<std::string, DType> m = {
      {"i1", DType::PRED}, {"i8", DType::S8}, {"i16", DType::S16}, {"i32", DType::S32},
      {"i64", DType::S64}, {"ui8", DType::U8}, {"ui16", DType::U16}, {"ui32", DType::U32},
      {"ui64", DType::U64}, {"f16", DType::F16}, {"f32", DType::F32}, {"f64", DType::F64},
      {"bf16", DType::BF16}};
  auto it = m.find(s);
  return it == m.end() ? DType::INVALID : it->second;
}
bool dtype_is_float(DType t) {
  return t == DType::F16 || t == DType::F32 || t == DType::F64 || t == DType::BF16;
}
bool dtype_is_unsigned(DType t) {
  return t == DType::U8 || t == DType::U16 || t == DType::U32 || t == DType::U64;
}
bool dtype_is_int(DType t) {
  return t == DType::S8 || t == DType::S16 || t == DType::S32 || t == DType::S64 ||
         dtype_is_unsigned(t);
}
std::string TensorType::str() const {
  std::string s = "tensor<";
  for (auto d : dims) s += std::to_string(d) + "x";
  return s + dtype_name(dtype) + ">";
}
std::string join_ints(const std::vector<int64_t>& v) {
  std::string s = "[";
  for (size_t i = 0; i < v.size(); ++i) s += (i ? "," : "") + std::to_string(v[i]);
  return s + "]";
}

static const std::pair<const char*, Op> kOpNames[] = {
    {"parameter", Op::Parameter}, {"constant", Op::Constant}, {"iota", Op::Iota},
    {"negate", Op::Neg}, {"abs", Op::Abs}, {"exponential", Op::Exp},
    {"exponential_minus_one", Op::Expm1}, {"log", Op::Log}, {"log_plus_one", Op::Log1p},
    {"sqrt", Op::Sqrt}, {"rsqrt", Op::Rsqrt}, {"cbrt", Op::Cbrt}, {"tanh", Op::Tanh},
    {"logistic", Op::Logistic}, {"sine", Op::Sin}, {"cosine", Op::Cos}, {"tan", Op::Tan},
    {"erf", Op::Erf}, {"floor", Op::Floor}, {"ceil", Op::Ceil},
    {"round_nearest_afz", Op::RoundAfz}, {"round_nearest_even", Op::RoundEven},
    {"sign", Op::Sign}, {"not", Op::Not}, {"is_finite", Op::IsFinite},
    {"popcnt", Op::PopCnt}, {"imag", Op::Imag}, {"real", Op::Real},
    {"add", Op::Add}, {"subtract", Op::Sub}, {"multiply", Op::Mul}, {"divide", Op::Div},
    {"remainder", Op::Rem}, {"maximum", Op::Max}, {"minimum", Op::Min}, {"power", Op::Pow},
    {"atan2", Op::Atan2}, {"and", Op::And}, {"or", Op::Or}, {"xor", Op::Xor},
    {"shift_left", Op::ShiftLeft}, {"shift_right_arithmetic", Op::ShiftRightArith},
    {"shift_right_logical", Op::ShiftRightLogical}, {"compare", Op::Compare},
    {"select", Op::Select}, {"clamp", Op::Clamp}, {"convert", Op::Convert},
    {"bitcast_convert", Op::BitcastConvert}, {"broadcast_in_dim", Op::BroadcastInDim},
    {"reshape", Op::Reshape}, {"transpose", Op::Transpose}, {"slice", Op::Slice},
    {"dynamic_slice", Op::DynamicSlice}, {"dynamic_update_slice", Op::DynamicUpdateSlice},
    {"pad", Op::Pad}, {"concatenate", Op::Concatenate}, {"reverse", Op::Reverse},
    {"reduce", Op::Reduce}, {"dot_general", Op::DotGeneral}, {"convolution", Op::Convolution},
    {"reduce_window", Op::ReduceWindow}, {"select_and_scatter", Op::SelectAndScatter},
    {"gather", Op::Gather}, {"scatter", Op::Scatter}, {"custom_call", Op::CustomCall},
    {"all_reduce", Op::AllReduce}, {"sort", Op::Sort}, {"call", Op::Call},
    {"return", Op::Return}, {"optimization_barrier", Op::OptimizationBarrier},
    {"tuple", Op::Tuple}, {"get_tuple_element", Op::GetTupleElement},
    {"fused_sdpa", Op::FusedSdpa}, {"fused_layer_norm", Op::FusedLayerNorm},
    {"fused_sdpa_bwd", Op::FusedSdpaBwd},
};

const char* op_name(Op op) {
  for (auto& p : kOpNames)
    if (p.second == op) return p.first;
  return "?";
}

namespace {

struct ParseError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

bool is_ident_char(char c) {
  return std::isalnum((unsigned char)c) || c == '_' || c == '.' || c == '$' || c == '-';
}

uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

class Parser {
 public:
  explicit Parser(const std::string& s) : s_(s) {}

  Module run() {
    Module m;
    ws();
    if (accept_word("module")) {
      ws();
      if (peek() == '@') m.name = symbol();
      ws();
      if (accept_word("attributes")) {
        auto attrs = attr_dict();
        if (attrs.count("mhlo.num_replicas")) m.num_replicas = leading_int(attrs["mhlo.num_replicas"]);
        if (attrs.count("mhlo.num_partitions"))
          m.num_partitions = leading_int(attrs["mhlo.num_partitions"]);
      }
      ws();
      expect("{");
      module_body(m, true);
    } else {
      module_body(m, false);
    }
    if (m.funcs.empty()) throw ParseError("no func.func found");
    if (!m.funcs.count("main")) m.entry = m.funcs.begin()->first;
    return m;
  }

 private:
  const std::string& s_;
  size_t p_ = 0;
  std::vector<std::unordered_map<std::string, ValueRef>> scopes_;
  Graph* g_ = nullptr;

  // ------------------------------------------------------------ lexing ---
  [[noreturn]] void fail(const std::string& msg) {
    size_t line = 1, col = 1;
    for (size_t i = 0; i < p_ && i < s_.size(); ++i) {
      if (s_[i] == '\n') { ++line; col = 1; } else { ++col; }
    }
    size_t e = s_.find('\n', p_);
    std::string ctx = s_.substr(p_, std::min<size_t>(60, (e == std::string::npos ? s_.size() : e) - p_));
    throw ParseError("StableHLO parse error at " + std::to_string(line) + ":" +
                     std::to_string(col) + ": " + msg + " near '" + ctx + "'");
  }
  char peek(size_t k = 0) const { return p_ + k < s_.size() ? s_[p_ + k] : '\0'; }
  bool eof() const { return p_ >= s_.size(); }
  void ws() {
    while (!eof()) {
      char c = peek();
      if (std::isspace((unsigned char)c)) { ++p_; continue; }
      if (c == '/' && peek(1) == '/') {
        while (!eof() && peek() != '\n') ++p_;
        continue;
      }
      break;
    }
  }
  bool starts(const char* t) const { return s_.compare(p_, std::strlen(t), t) == 0; }
  bool accept(const char* t) {
    ws();
    if (starts(t)) { p_ += std::strlen(t); return true; }
    return false;
  }
  bool accept_word(const char* t) {
    ws();
    size_t n = std::strlen(t);
    if (starts(t) && !is_ident_char(peek(n))) { p_ += n; return true; }
    return false;
  }
  void expect(const char* t) {
    if (!accept(t)) fail(std::string("expected '") + t + "'");
  }
  std::string ident() {
    ws();
    size_t b = p_;
    while (!eof() && (is_ident_char(peek()))) ++p_;
    if (b == p_) fail("expected identifier");
    return s_.substr(b, p_ - b);
  }
  std::string symbol() {  // @name
    ws();
    if (peek() != '@') fail("expected @symbol");
    ++p_;
    if (peek() == '"') return quoted();
    size_t b = p_;
    while (!eof() && is_ident_char(peek())) ++p_;
    return s_.substr(b, p_ - b);
  }
  std::string quoted() {
    ws();
    if (peek() != '"') fail("expected string");
    ++p_;
    std::string out;
    while (!eof() && peek() != '"') {
      char c = s_[p_++];
      if (c == '\\' && !eof()) {
        char n = s_[p_++];
        if (n == 'n') out += '\n';
        else if (n == 't') out += '\t';
        else if (std::isxdigit((unsigned char)n) && std::isxdigit((unsigned char)peek())) {
          char h[3] = {n, s_[p_++], 0};
          out += (char)std::strtol(h, nullptr, 16);
        } else out += n;
      } else {
        out += c;
      }
    }
    expect("\"");
    return out;
  }
  std::string value_name() {  // %name or %name#k
    ws();
    if (peek() != '%') fail("expected %value");
    size_t b = p_++;
    while (!eof() && (std::isalnum((unsigned char)peek()) || peek() == '_' || peek() == '#' ||
                      peek() == '.' || peek() == '$' || peek() == '-'))
      ++p_;
    return s_.substr(b, p_ - b);
  }
  int64_t integer() {
    ws();
    size_t b = p_;
    if (peek() == '-' || peek() == '+') ++p_;
    while (std::isdigit((unsigned char)peek())) ++p_;
    if (b == p_) fail("expected integer");
    return std::stoll(s_.substr(b, p_ - b));
  }
  static int64_t leading_int(const std::string& v) {
    size_t i = 0;
    while (i < v.size() && !(std::isdigit((unsigned char)v[i]) || v[i] == '-')) ++i;
    return std::stoll(v.substr(i));
  }
  // Raw text of one attribute value, balanced over ()[]{}<> and strings.
  std::string raw_value(const char* stops = ",}") {
    ws();
    size_t b = p_;
    int depth = 0;
    while (!eof()) {
      char c = peek();
      if (c == '"') { quoted(); continue; }
      if (depth == 0 && std::strchr(stops, c)) break;
      if (c == '(' || c == '[' || c == '{' || c == '<') ++depth;
      if (c == ')' || c == ']' || c == '}' || c == '>') {
        if (c == '>' && p_ > 0 && s_[p_ - 1] == '-') { ++p_; continue; }  // "->"
        if (depth == 0) break;
        --depth;
      }
      ++p_;
    }
    std::string r = s_.substr(b, p_ - b);
    while (!r.empty() && std::isspace((unsigned char)r.back())) r.pop_back();
    return r;
  }
  std::map<std::string, std::string> attr_dict() {
    std::map<std::string, std::string> out;
    expect("{");
    while (true) {
      ws();
      if (accept("}")) break;
      std::string key = peek() == '"' ? quoted() : ident();
      std::string val;
      if (accept("=")) val = raw_value(",}");
      out[key] = val;
      ws();
      if (accept(",")) continue;
      expect("}");
      break;
    }
    return out;
  }
  // [1, 2, 3] | array<i64: 1, 2> | array<i64>
  std::vector<int64_t> int_list() {
    std::vector<int64_t> v;
    ws();
    if (accept("array<")) {
      ident();  // i64 / i1
      if (accept(":")) {
        do {
          ws();
          if (accept_word("true")) v.push_back(1);
          else if (accept_word("false")) v.push_back(0);
          else v.push_back(integer());
        } while (accept(","));
      }
      expect(">");
      return v;
    }
    expect("[");
    if (accept("]")) return v;
    do {
      ws();
      if (accept_word("true")) v.push_back(1);
      else if (accept_word("false")) v.push_back(0);
      else v.push_back(integer());
    } while (accept(","));
    expect("]");
    return v;
  }
  static std::vector<int64_t> ints_from_raw(const std::string& raw) {
    std::vector<int64_t> v;
    size_t i = 0;
    // skip an "array<i64:" or "dense<" prefix
    auto c = raw.find(':');
    if (raw.rfind("array<", 0) == 0) i = (c == std::string::npos) ? raw.size() : c + 1;
    while (i < raw.size()) {
      if (raw.compare(i, 4, "true") == 0) { v.push_back(1); i += 4; continue; }
      if (raw.compare(i, 5, "false") == 0) { v.push_back(0); i += 5; continue; }
      if (std::isdigit((unsigned char)raw[i]) ||
          (raw[i] == '-' && i + 1 < raw.size() && std::isdigit((unsigned char)raw[i + 1]))) {
        size_t e = i + 1;
        while (e < raw.size() && std::isdigit((unsigned char)raw[e])) ++e;
        v.push_back(std::stoll(raw.substr(i, e - i)));
        i = e;
        continue;
      }
      if (raw[i] == ':') break;  // ": tensor<...>" suffix of a dense attr
      ++i;
    }
    return v;
  }

  // ------------------------------------------------------------- types ---
  TensorType type() {
    ws();
    TensorType t;
    if (accept("!stablehlo.token")) { t.dtype = DType::TOKEN; return t; }
    if (!accept("tensor<")) fail("expected tensor type");
    while (true) {
      ws();
      if (std::isdigit((unsigned char)peek())) {
        size_t b = p_;
        while (std::isdigit((unsigned char)peek())) ++p_;
        int64_t d = std::stoll(s_.substr(b, p_ - b));
        if (peek() != 'x') fail("malformed tensor type");
        ++p_;
        t.dims.push_back(d);
        continue;
      }
      if (peek() == '?') fail("dynamic shapes are not supported");
      break;
    }
    size_t b = p_;
    while (std::isalnum((unsigned char)peek())) ++p_;
    std::string et = s_.substr(b, p_ - b);
    t.dtype = dtype_from_mlir(et);
    if (t.dtype == DType::INVALID) fail("unsupported element type '" + et + "'");
    ws();
    if (accept(",")) raw_value(">");  // encoding (e.g. #stablehlo.bounds) – ignored
    expect(">");
    return t;
  }
  // "(T, T) -> T" | "(T) -> (T, T)" | "T" | "T, T" (select/optimization_barrier)
  void func_type(std::vector<TensorType>& ins, std::vector<TensorType>& outs) {
    ws();
    if (peek() == '(') {
      ++p_;
      ws();
      if (!accept(")")) {
        do { ins.push_back(type()); } while (accept(","));
        expect(")");
      }
      expect("->");
      ws();
      if (peek() == '(') {
        ++p_;
        ws();
        if (!accept(")")) {
          do {
            outs.push_back(type());
            ws();
            if (peek() == '{') attr_dict();
          } while (accept(","));
          expect(")");
        }
      } else {
        outs.push_back(type());
      }
    } else {
      do { outs.push_back(type()); } while (accept(","));
      ins = outs;
    }
  }

  // ----------------------------------------------------------- values ---
  ValueRef lookup(const std::string& name) {
    std::string base = name;
    int idx = 0;
    auto h = name.find('#');
    if (h != std::string::npos) {
      base = name.substr(0, h);
      idx = std::stoi(name.substr(h + 1));
    }
    for (auto it = scopes_.rbegin(); it != scopes_.rend(); ++it) {
      auto f = it->find(base);
      if (f != it->end()) return ValueRef{f->second.node, f->second.idx + idx};
    }
    fail("undefined value " + name);
  }
  std::vector<ValueRef> operand_list() {  // %a, %b, ...
    std::vector<ValueRef> v;
    ws();
    if (peek() != '%') return v;
    do { v.push_back(lookup(value_name())); ws(); } while (peek() == ',' && peek_value_after_comma() && accept(","));
    return v;
  }
  bool peek_value_after_comma() {
    size_t q = p_ + 1;
    while (q < s_.size() && std::isspace((unsigned char)s_[q])) ++q;
    return q < s_.size() && s_[q] == '%';
  }
  void skip_loc() {
    ws();
    if (starts("loc(")) { p_ += 3; raw_paren(); }
  }
  void raw_paren() {  // at '(' : skip balanced
    int d = 0;
    while (!eof()) {
      char c = peek();
      if (c == '"') { quoted(); continue; }
      if (c == '(') ++d;
      if (c == ')') { --d; if (d == 0) { ++p_; return; } }
      ++p_;
    }
  }

  // ---------------------------------------------------------- structure --
  void module_body(Module& m, bool braced) {
    while (true) {
      ws();
      if (eof()) {
        if (braced) fail("unterminated module");
        return;
      }
      if (braced && accept("}")) {
        ws();
        skip_trailing();
        return;
      }
      if (peek() == '#') {  // #loc = loc(...) aliases
        while (!eof() && peek() != '\n') ++p_;
        continue;
      }
      if (accept_word("func.func") || accept_word("func")) {
        auto g = std::make_shared<Graph>();
        std::string fname = function(*g);
        g->name = fname;
        m.funcs[fname] = g;
        continue;
      }
      if (accept_word("sdy.mesh")) {
        while (!eof() && peek() != '\n') ++p_;
        continue;
      }
      fail("unexpected top-level item");
    }
  }
  void skip_trailing() {
    while (!eof()) {
      ws();
      if (eof()) return;
      if (peek() == '#') { while (!eof() && peek() != '\n') ++p_; continue; }
      if (starts("loc(")) { p_ += 3; raw_paren(); continue; }
      fail("trailing text after module");
    }
  }

  std::string function(Graph& g) {
    ws();
    if (accept_word("public") || accept_word("private") || accept_word("nested")) {}
    std::string name = symbol();
    g_ = &g;
    scopes_.clear();
    scopes_.emplace_back();
    expect("(");
    ws();
    if (!accept(")")) {
      do {
        std::string an = value_name();
        expect(":");
        TensorType t = type();
        ws();
        if (peek() == '{') attr_dict();
        skip_loc();
        Node n;
        n.op = Op::Parameter;
        n.param_index = (int64_t)g.param_types.size();
        n.results.push_back(t);
        n.name = an;
        g.param_types.push_back(t);
        scopes_.back()[an] = ValueRef{g.add(std::move(n)), 0};
      } while (accept(","));
      expect(")");
    }
    if (accept("->")) {
      std::vector<TensorType> outs, dummy;
      ws();
      if (peek() == '(') {
        ++p_;
        ws();
        if (!accept(")")) {
          do {
            outs.push_back(type());
            ws();
            if (peek() == '{') attr_dict();
          } while (accept(","));
          expect(")");
        }
      } else {
        outs.push_back(type());
      }
    }
    ws();
    if (accept_word("attributes")) attr_dict();
    expect("{");
    block_body(g, /*is_region=*/false);
    skip_loc();
    return name;
  }

  // Statements until the closing '}' (consumed).
  void block_body(Graph& g, bool is_region) {
    while (true) {
      ws();
      if (accept("}")) return;
      if (peek() == '^') {  // ^bb0(%a: T, ...):
        ++p_;
        ident();
        expect("(");
        ws();
        if (!accept(")")) {
          do {
            std::string an = value_name();
            expect(":");
            TensorType t = type();
            skip_loc();
            Node n;
            n.op = Op::Parameter;
            n.param_index = (int64_t)g.param_types.size();
            n.results.push_back(t);
            n.name = an;
            g.param_types.push_back(t);
            scopes_.back()[an] = ValueRef{g.add(std::move(n)), 0};
          } while (accept(","));
          expect(")");
        }
        expect(":");
        continue;
      }
      if (accept_word("return") || accept_word("func.return") || accept_word("stablehlo.return") ||
          accept_word("mhlo.return") || accept_word("\"stablehlo.return\"")) {
        ws();
        std::vector<ValueRef> outs;
        if (peek() == '(') {  // generic "stablehlo.return"(%a) : (T) -> ()
          ++p_;
          outs = operand_list();
          expect(")");
        } else {
          outs = operand_list();
        }
        ws();
        if (accept(":")) {
          std::vector<TensorType> a, b;
          ws();
          if (peek() == '(') func_type(a, b);
          else { do { type(); } while (accept(",")); }
        }
        skip_loc();
        g.outputs = outs;
        (void)is_region;
        continue;
      }
      statement(g);
    }
  }

  void statement(Graph& g) {
    // results
    std::vector<std::pair<std::string, int>> names;
    ws();
    if (peek() == '%') {
      do {
        std::string n = value_name();
        int cnt = 1;
        if (accept(":")) cnt = (int)integer();
        names.push_back({n, cnt});
      } while (accept(","));
      expect("=");
    }
    Node n;
    op(n);
    skip_loc();
    int id = g.add(std::move(n));
    int k = 0;
    for (auto& nm : names) {
      scopes_.back()[nm.first] = ValueRef{id, k};
      k += nm.second;
    }
    if (!names.empty()) g.nodes[id].name = names[0].first;
    if ((int)g.nodes[id].results.size() < k) fail("result count mismatch");
  }

  std::shared_ptr<Graph> region() {
    // '{' [^bb0(...):] stmts '}'
    auto r = std::make_shared<Graph>();
    Graph* saved = g_;
    g_ = r.get();
    scopes_.emplace_back();
    expect("{");
    block_body(*r, true);
    scopes_.pop_back();
    g_ = saved;
    return r;
  }

  static Op lookup_op(const std::string& full, bool* ok) {
    std::string n = full;
    for (const char* pre : {"stablehlo.", "mhlo.", "chlo.", "func."}) {
      if (n.rfind(pre, 0) == 0) { n = n.substr(std::strlen(pre)); break; }
    }
    for (auto& p : kOpNames)
      if (n == p.first) { *ok = true; return p.second; }
    *ok = false;
    return Op::Parameter;
  }

  void set_body_kind(Node& n) { (void)n; }

  // ------------------------------------------------------------- ops ---
  void op(Node& n) {
    ws();
    if (peek() == '"') return generic_op(n);
    std::string name = ident();
    bool ok = false;
    // sdy.* ops carry sharding annotations only: identity on their operand.
    if (name.rfind("sdy.", 0) == 0) {
      auto ops = operand_list();
      raw_value(":");
      expect(":");
      std::vector<TensorType> ins, outs;
      func_type(ins, outs);
      n.op = Op::OptimizationBarrier;
      n.operands = ops;
      n.results = outs;
      return;
    }
    Op op = lookup_op(name, &ok);
    if (!ok) fail("unsupported op '" + name + "'");
    n.op = op;
    std::vector<TensorType> ins, outs;
    switch (op) {
      case Op::Constant: {
        ws();
        std::map<std::string, std::string> attrs;
        if (peek() == '{') attrs = attr_dict();
        std::string raw = raw_value(":");
        expect(":");
        TensorType t = type();
        n.results.push_back(t);
        parse_dense(raw, t, n.cdata);
        return;
      }
      case Op::Iota: {
        expect("dim");
        expect("=");
        n.iota_dim = integer();
        expect(":");
        n.results.push_back(type());
        return;
      }
      case Op::Compare: {
        ws();
        std::string dir = ident();
        n.cmp_dir = parse_dir(dir);
        expect(",");
        n.operands.push_back(lookup(value_name()));
        expect(",");
        n.operands.push_back(lookup(value_name()));
        if (accept(",")) n.cmp_type = parse_cmp_type(ident());
        expect(":");
        func_type(ins, outs);
        n.results = {outs.at(0)};
        if (outs[0].dtype != DType::PRED) n.results[0].dtype = DType::PRED;
        return;
      }
      case Op::BroadcastInDim: case Op::Transpose: case Op::Reverse: {
        n.operands = operand_list();
        expect(",");
        expect("dims");
        expect("=");
        n.dims = int_list();
        expect(":");
        func_type(ins, outs);
        n.results = {outs.at(0)};
        return;
      }
      case Op::Slice: {
        n.operands = operand_list();
        ws();
        if (accept("[")) {  // [a:b(:c), ...]
          if (!accept("]")) {
            do {
              n.start.push_back(integer());
              expect(":");
              n.limit.push_back(integer());
              n.strides.push_back(accept(":") ? integer() : 1);
            } while (accept(","));
            expect("]");
          }
        } else {
          expect(",");
          while (true) {
            std::string k = ident();
            expect("=");
            auto v = int_list();
            if (k == "start_indices") n.start = v;
            else if (k == "limit_indices") n.limit = v;
            else if (k == "strides") n.strides = v;
            if (!accept(",")) break;
          }
          if (n.strides.empty()) n.strides.assign(n.start.size(), 1);
        }
        expect(":");
        func_type(ins, outs);
        n.results = {outs.at(0)};
        return;
      }
      case Op::DynamicSlice: {
        n.operands = operand_list();
        expect(",");
        expect("sizes");
        expect("=");
        n.limit = int_list();
        expect(":");
        func_type(ins, outs);
        n.results = {outs.at(0)};
        return;
      }
      case Op::Pad: {
        n.operands = operand_list();
        while (accept(",")) {
          std::string k = ident();
          expect("=");
          auto v = int_list();
          if (k == "low") n.pad_lo = v;
          else if (k == "high") n.pad_hi = v;
          else if (k == "interior") n.pad_interior = v;
        }
        expect(":");
        func_type(ins, outs);
        n.results = {outs.at(0)};
        return;
      }
      case Op::Concatenate: {
        n.operands = operand_list();
        expect(",");
        expect("dim");
        expect("=");
        n.axis = integer();
        expect(":");
        func_type(ins, outs);
        n.results = {outs.at(0)};
        return;
      }
      case Op::DotGeneral: {
        n.operands = operand_list();
        while (accept(",")) {
          std::string k = ident();
          expect("=");
          if (k == "batching_dims" || k == "contracting_dims") {
            auto l = int_list();
            expect("x");
            auto r = int_list();
            if (k == "batching_dims") { n.lhs_batch = l; n.rhs_batch = r; }
            else { n.lhs_contract = l; n.rhs_contract = r; }
          } else {
            raw_value(",:");
          }
        }
        expect(":");
        func_type(ins, outs);
        n.results = {outs.at(0)};
        return;
      }
      case Op::Convolution: {
        expect("(");
        n.operands = operand_list();
        expect(")");
        while (true) {
          ws();
          if (accept_word("dim_numbers")) {
            expect("=");
            parse_conv_dims(n.conv);
          } else if (accept_word("window")) {
            expect("=");
            parse_window(n);
          } else if (peek() == '{') {
            auto a = attr_dict();
            if (a.count("feature_group_count")) n.feature_groups = leading_int(a["feature_group_count"]);
            if (a.count("batch_group_count")) n.batch_groups = leading_int(a["batch_group_count"]);
          } else if (accept(",")) {
          } else {
            break;
          }
        }
        expect(":");
        func_type(ins, outs);
        n.results = {outs.at(0)};
        fill_conv_defaults(n);
        return;
      }
      case Op::Reduce: {
        // reduce(%a init: %b)[, (%c init: %d)] applies OP across dimensions = [..] : T
        // or ... across dimensions = [..] : T reducer(%x: T, %y: T) (...) { body }
        std::vector<ValueRef> inputs, inits;
        do {
          expect("(");
          inputs.push_back(lookup(value_name()));
          expect("init");
          expect(":");
          inits.push_back(lookup(value_name()));
          expect(")");
        } while (accept(","));
        n.operands = inputs;
        n.operands.insert(n.operands.end(), inits.begin(), inits.end());
        std::string applies;
        if (accept_word("applies")) applies = ident();
        expect("across");
        expect("dimensions");
        expect("=");
        n.dims = int_list();
        expect(":");
        func_type(ins, outs);
        n.results = outs;
        if (!applies.empty()) {
          n.regions.push_back(scalar_body(applies, ins.back().dtype, (int)inputs.size()));
        } else {
          expect("reducer");
          // reducer(%a: T, %b: T) (%c: T, %d: T) { ... }
          auto r = std::make_shared<Graph>();
          Graph* saved = g_;
          g_ = r.get();
          scopes_.emplace_back();
          std::vector<std::pair<std::string, TensorType>> lhs, rhs;
          while (accept("(")) {
            std::string a = value_name();
            expect(":");
            TensorType ta = type();
            expect(",");
            std::string b = value_name();
            expect(":");
            TensorType tb = type();
            expect(")");
            lhs.push_back({a, ta});
            rhs.push_back({b, tb});
          }
          for (auto* grp : {&lhs, &rhs})
            for (auto& pr : *grp) {
              Node pn;
              pn.op = Op::Parameter;
              pn.param_index = (int64_t)r->param_types.size();
              pn.results.push_back(pr.second);
              r->param_types.push_back(pr.second);
              scopes_.back()[pr.first] = ValueRef{r->add(std::move(pn)), 0};
            }
          expect("{");
          block_body(*r, true);
          scopes_.pop_back();
          g_ = saved;
          n.regions.push_back(r);
        }
        return;
      }
      case Op::CustomCall: {
        n.target = symbol();
        expect("(");
        n.operands = operand_list();
        expect(")");
        ws();
        if (peek() == '{') {
          auto a = attr_dict();
          if (a.count("backend_config")) n.backend_config = unquote(a["backend_config"]);
        }
        expect(":");
        func_type(ins, outs);
        n.results = outs;
        return;
      }
      case Op::Call: {
        n.target = symbol();
        expect("(");
        n.operands = operand_list();
        expect(")");
        ws();
        if (peek() == '{') attr_dict();
        expect(":");
        func_type(ins, outs);
        n.results = outs;
        return;
      }
      case Op::Select: case Op::Clamp: case Op::OptimizationBarrier: case Op::Convert:
      case Op::BitcastConvert: case Op::Reshape: case Op::DynamicUpdateSlice:
      default: {
        // Elementwise and other ops with "operands : type(s)" printing.
        n.operands = operand_list();
        ws();
        if (peek() == '{') attr_dict();
        expect(":");
        func_type(ins, outs);
        if (op == Op::Select || op == Op::Clamp) {
          n.results = {outs.back()};
          if (ins.size() == outs.size() && outs.size() == 2) n.results = {outs[1]};
        } else if (op == Op::OptimizationBarrier) {
          n.results = outs;
        } else {
          n.results = {outs.back()};
        }
        if (op == Op::Select && !outs.empty() && ins.size() == 3) n.results = {outs[0]};
        return;
      }
    }
  }

  // "stablehlo.op"(%a, ...) <{props}> ({regions}) {attrs} : (T..) -> T..
  void generic_op(Node& n) {
    std::string name = quoted();
    bool ok = false;
    Op op = lookup_op(name, &ok);
    if (!ok) {
      if (name.rfind("sdy.", 0) == 0) { op = Op::OptimizationBarrier; ok = true; }
      else fail("unsupported op '" + name + "'");
    }
    n.op = op;
    expect("(");
    n.operands = operand_list();
    expect(")");
    std::map<std::string, std::string> attrs;
    ws();
    if (starts("<{")) {
      ++p_;
      auto a = attr_dict();
      expect(">");
      attrs.insert(a.begin(), a.end());
    }
    ws();
    if (starts("({")) {
      ++p_;
      do {
        ws();
        n.regions.push_back(region());
      } while (accept(","));
      expect(")");
    }
    ws();
    if (peek() == '{') {
      auto a = attr_dict();
      attrs.insert(a.begin(), a.end());
    }
    expect(":");
    std::vector<TensorType> ins, outs;
    func_type(ins, outs);
    n.results = outs;
    apply_generic_attrs(n, attrs);
  }

  void apply_generic_attrs(Node& n, std::map<std::string, std::string>& a) {
    auto ints = [&](const char* k) { return a.count(k) ? ints_from_raw(a[k]) : std::vector<int64_t>{}; };
    switch (n.op) {
      case Op::Constant: parse_dense(a["value"], n.results.at(0), n.cdata); break;
      case Op::Iota: n.iota_dim = leading_int(a["iota_dimension"]); break;
      case Op::BroadcastInDim: n.dims = ints("broadcast_dimensions"); break;
      case Op::Transpose: n.dims = ints("permutation"); break;
      case Op::Reverse: n.dims = ints("dimensions"); break;
      case Op::Reduce: n.dims = ints("dimensions"); break;
      case Op::Concatenate: n.axis = leading_int(a["dimension"]); break;
      case Op::Slice:
        n.start = ints("start_indices"); n.limit = ints("limit_indices"); n.strides = ints("strides");
        if (n.strides.empty()) n.strides.assign(n.start.size(), 1);
        break;
      case Op::DynamicSlice: n.limit = ints("slice_sizes"); break;
      case Op::Pad:
        n.pad_lo = ints("edge_padding_low"); n.pad_hi = ints("edge_padding_high");
        n.pad_interior = ints("interior_padding");
        break;
      case Op::Compare:
        n.cmp_dir = parse_dir(after_last_space_or_lt(a["comparison_direction"]));
        if (a.count("compare_type")) n.cmp_type = parse_cmp_type(after_last_space_or_lt(a["compare_type"]));
        for (auto& r : n.results) r.dtype = DType::PRED;
        break;
      case Op::ReduceWindow: case Op::SelectAndScatter: {
        n.window = ints("window_dimensions");
        n.window_strides = ints("window_strides");
        n.base_dilation = ints("base_dilations");
        n.window_dilation = ints("window_dilations");
        auto pad = ints("padding");
        size_t r = n.window.size();
        if (n.window_strides.empty()) n.window_strides.assign(r, 1);
        if (n.base_dilation.empty()) n.base_dilation.assign(r, 1);
        if (n.window_dilation.empty()) n.window_dilation.assign(r, 1);
        n.pad_lo.assign(r, 0);
        n.pad_hi.assign(r, 0);
        if (pad.size() == 1) pad.assign(2 * r, pad[0]);  // splat: dense<v> pads every edge by v
        if (pad.size() == 2 * r)
          for (size_t i = 0; i < r; ++i) { n.pad_lo[i] = pad[2 * i]; n.pad_hi[i] = pad[2 * i + 1]; }
        else if (!pad.empty())
          n.pad_lo.clear();  // a list of the wrong length: rejected by the verifier
        break;
      }
      case Op::DotGeneral: {
        auto& dn = a["dot_dimension_numbers"];
        n.lhs_batch = field_ints(dn, "lhs_batching_dimensions");
        n.rhs_batch = field_ints(dn, "rhs_batching_dimensions");
        n.lhs_contract = field_ints(dn, "lhs_contracting_dimensions");
        n.rhs_contract = field_ints(dn, "rhs_contracting_dimensions");
        break;
      }
      case Op::Gather: {
        auto& dn = a["dimension_numbers"];
        n.gather.offset_dims = field_ints(dn, "offset_dims");
        n.gather.collapsed_slice_dims = field_ints(dn, "collapsed_slice_dims");
        n.gather.operand_batching_dims = field_ints(dn, "operand_batching_dims");
        n.gather.start_indices_batching_dims = field_ints(dn, "start_indices_batching_dims");
        n.gather.start_index_map = field_ints(dn, "start_index_map");
        auto iv = field_ints(dn, "index_vector_dim");
        n.gather.index_vector_dim = iv.empty() ? 0 : iv[0];
        n.gather.slice_sizes = ints("slice_sizes");
        break;
      }
      case Op::Scatter: {
        auto& dn = a["scatter_dimension_numbers"];
        n.scatter.update_window_dims = field_ints(dn, "update_window_dims");
        n.scatter.inserted_window_dims = field_ints(dn, "inserted_window_dims");
        n.scatter.input_batching_dims = field_ints(dn, "input_batching_dims");
        n.scatter.scatter_indices_batching_dims = field_ints(dn, "scatter_indices_batching_dims");
        n.scatter.scatter_dims_to_operand_dims = field_ints(dn, "scatter_dims_to_operand_dims");
        auto iv = field_ints(dn, "index_vector_dim");
        n.scatter.index_vector_dim = iv.empty() ? 0 : iv[0];
        break;
      }
      case Op::AllReduce: {
        auto rg = a["replica_groups"];
        // dense<[[0, 1], [2, 3]]> : tensor<2x2xi64>
        auto colon = rg.rfind("tensor<");
        std::vector<int64_t> shape;
        if (colon != std::string::npos) {
          std::string t = rg.substr(colon + 7);
          size_t i = 0;
          while (i < t.size() && std::isdigit((unsigned char)t[i])) {
            size_t e = i;
            while (e < t.size() && std::isdigit((unsigned char)t[e])) ++e;
            shape.push_back(std::stoll(t.substr(i, e - i)));
            i = e + 1;
          }
        }
        auto vals = ints_from_raw(rg.substr(0, colon == std::string::npos ? rg.size() : colon));
        if (shape.size() == 2 && shape[0] * shape[1] == (int64_t)vals.size()) {
          for (int64_t gi = 0; gi < shape[0]; ++gi)
            n.replica_groups.emplace_back(vals.begin() + gi * shape[1],
                                          vals.begin() + (gi + 1) * shape[1]);
        } else if (!vals.empty()) {
          n.replica_groups.push_back(vals);
        }
        if (a.count("channel_handle")) {
          auto v = field_ints(a["channel_handle"], "handle");
          n.channel_id = v.empty() ? 0 : v[0];
        }
        break;
      }
      case Op::CustomCall:
        n.target = unquote(a["call_target_name"]);
        if (a.count("backend_config")) n.backend_config = unquote(a["backend_config"]);
        break;
      case Op::Convolution: {
        n.window_strides = ints("window_strides");
        n.lhs_dilation = ints("lhs_dilation");
        n.rhs_dilation = ints("rhs_dilation");
        auto pad = ints("padding");
        auto rev = ints("window_reversal");
        for (auto r : rev) n.window_reversal.push_back(r != 0);
        if (a.count("feature_group_count")) n.feature_groups = leading_int(a["feature_group_count"]);
        if (a.count("batch_group_count")) n.batch_groups = leading_int(a["batch_group_count"]);
        auto& dn = a["dimension_numbers"];
        // #stablehlo.conv<[b, 0, 1, f]x[0, 1, i, o]->[b, 0, 1, f]> or raw field form
        auto lb = dn.find('[');
        if (lb != std::string::npos) {
          size_t save = p_;
          std::string sub = dn.substr(lb);
          Parser sp(sub);
          sp.parse_conv_dims(n.conv);
          p_ = save;
        }
        size_t ns = n.conv.in_spatial.size();
        if (pad.size() == 1) pad.assign(2 * ns, pad[0]);  // splat: dense<v> pads every edge by v
        for (size_t i = 0; i < ns && pad.size() == 2 * ns; ++i) {
          n.pad_lo.push_back(pad[2 * i]);
          n.pad_hi.push_back(pad[2 * i + 1]);
        }
        if (!pad.empty() && pad.size() != 2 * ns)
          n.pad_lo.assign(ns + 1, 0);  // a list of the wrong length: rejected by the verifier
        fill_conv_defaults(n);
        break;
      }
      case Op::Call: n.target = a.count("callee") ? strip_at(a["callee"]) : ""; break;
      default: break;
    }
  }
  static std::string strip_at(const std::string& s) {
    std::string t = s;
    if (!t.empty() && t[0] == '@') t = t.substr(1);
    return t;
  }
  static std::string after_last_space_or_lt(const std::string& v) {
    // "#stablehlo<comparison_direction GT>" -> "GT"
    std::string t = v;
    while (!t.empty() && (t.back() == '>' || std::isspace((unsigned char)t.back()))) t.pop_back();
    auto p = t.find_last_of(" <");
    return p == std::string::npos ? t : t.substr(p + 1);
  }
  static std::vector<int64_t> field_ints(const std::string& s, const std::string& key) {
    auto p = s.find(key);
    if (p == std::string::npos) return {};
    p += key.size();
    while (p < s.size() && (s[p] == ' ' || s[p] == '=')) ++p;
    if (p < s.size() && s[p] == '[') {
      auto e = s.find(']', p);
      return ints_from_raw(s.substr(p, e - p + 1));
    }
    size_t e = p;
    while (e < s.size() && (std::isdigit((unsigned char)s[e]) || s[e] == '-')) ++e;
    if (e == p) return {};
    return {std::stoll(s.substr(p, e - p))};
  }
  static std::string unquote(const std::string& s) {
    std::string t = s;
    while (!t.empty() && std::isspace((unsigned char)t.back())) t.pop_back();
    if (t.size() >= 2 && t.front() == '"' && t.back() == '"') {
      std::string out;
      for (size_t i = 1; i + 1 < t.size(); ++i) {
        if (t[i] == '\\' && i + 2 < t.size()) {
          char n = t[++i];
          if (std::isxdigit((unsigned char)n) && std::isxdigit((unsigned char)t[i + 1])) {
            char h[3] = {n, t[i + 1], 0};
            out += (char)std::strtol(h, nullptr, 16);
            ++i;
          } else out += n;
        } else {
          out += t[i];
        }
      }
      return out;
    }
    return t;
  }

  static CmpDir parse_dir(const std::string& d) {
    if (d == "EQ") return CmpDir::EQ;
    if (d == "NE") return CmpDir::NE;
    if (d == "LT") return CmpDir::LT;
    if (d == "LE") return CmpDir::LE;
    if (d == "GT") return CmpDir::GT;
    if (d == "GE") return CmpDir::GE;
    throw ParseError("bad comparison direction " + d);
  }
  static CmpType parse_cmp_type(const std::string& d) {
    if (d == "FLOAT") return CmpType::FLOAT;
    if (d == "SIGNED") return CmpType::SIGNED;
    if (d == "UNSIGNED") return CmpType::UNSIGNED;
    if (d == "TOTALORDER") return CmpType::TOTALORDER;
    return CmpType::NOTYPE;
  }

  // [b, 0, 1, f]x[0, 1, i, o]->[b, 0, 1, f]
  void parse_conv_dims(ConvDims& c) {
    auto spec = [&](char kind, std::vector<int64_t>& spatial, int64_t& a, int64_t& b) {
      expect("[");
      std::vector<std::pair<int64_t, int64_t>> sp;  // (spatial index, position)
      int64_t pos = 0;
      do {
        ws();
        if (std::isdigit((unsigned char)peek())) {
          sp.push_back({integer(), pos});
        } else {
          char ch = s_[p_++];
          if (kind == 'k') {
            if (ch == 'i') a = pos;
            else if (ch == 'o') b = pos;
            else fail("bad kernel dim spec");
          } else {
            if (ch == 'b') a = pos;
            else if (ch == 'f') b = pos;
            else fail("bad conv dim spec");
          }
        }
        ++pos;
      } while (accept(","));
      expect("]");
      spatial.assign(sp.size(), -1);
      for (auto& q : sp) {
        if (q.first < 0 || q.first >= (int64_t)sp.size() || spatial[q.first] >= 0)
          fail("spatial dimensions must be listed once each, numbered from 0");
        spatial[q.first] = q.second;
      }
    };
    spec('l', c.in_spatial, c.in_batch, c.in_feature);
    expect("x");
    spec('k', c.k_spatial, c.k_in, c.k_out);
    expect("->");
    spec('l', c.out_spatial, c.out_batch, c.out_feature);
  }
  // {stride = [1, 1], pad = [[1, 1], [1, 1]], lhs_dilate = [..], rhs_dilate = [..], reverse = [..]}
  void parse_window(Node& n) {
    expect("{");
    while (!accept("}")) {
      std::string k = ident();
      expect("=");
      if (k == "pad") {
        expect("[");
        do {
          expect("[");
          n.pad_lo.push_back(integer());
          expect(",");
          n.pad_hi.push_back(integer());
          expect("]");
        } while (accept(","));
        expect("]");
      } else {
        auto v = int_list();
        if (k == "stride") n.window_strides = v;
        else if (k == "lhs_dilate") n.lhs_dilation = v;
        else if (k == "rhs_dilate") n.rhs_dilation = v;
        else if (k == "reverse") for (auto r : v) n.window_reversal.push_back(r != 0);
      }
      accept(",");
    }
  }
  static void fill_conv_defaults(Node& n) {
    size_t r = n.conv.in_spatial.size();
    if (n.window_strides.empty()) n.window_strides.assign(r, 1);
    if (n.lhs_dilation.empty()) n.lhs_dilation.assign(r, 1);
    if (n.rhs_dilation.empty()) n.rhs_dilation.assign(r, 1);
    if (n.pad_lo.empty()) { n.pad_lo.assign(r, 0); n.pad_hi.assign(r, 0); }
    if (n.window_reversal.empty()) n.window_reversal.assign(r, false);
  }

  // Region for "applies stablehlo.add" shorthand: (a0..an, b0..bn) -> op(a, b).
  std::shared_ptr<Graph> scalar_body(const std::string& opname, DType dt, int nin) {
    auto r = std::make_shared<Graph>();
    bool ok = false;
    Op op = lookup_op(opname, &ok);
    if (!ok) fail("unsupported reducer " + opname);
    TensorType st{dt, {}};
    for (int i = 0; i < 2 * nin; ++i) {
      Node pn;
      pn.op = Op::Parameter;
      pn.param_index = i;
      pn.results.push_back(st);
      r->param_types.push_back(st);
      r->add(std::move(pn));
    }
    for (int i = 0; i < nin; ++i) {
      Node b;
      b.op = op;
      b.operands = {ValueRef{i, 0}, ValueRef{nin + i, 0}};
      b.results.push_back(st);
      r->outputs.push_back(ValueRef{r->add(std::move(b)), 0});
    }
    return r;
  }

  // ---------------------------------------------------------- constants --
  void parse_dense(const std::string& raw0, const TensorType& t, ConstData& cd) {
    std::string raw = raw0;
    // strip a trailing ": tensor<...>" (generic attr form)
    auto c = raw.rfind(": tensor<");
    if (c != std::string::npos) raw = raw.substr(0, c);
    while (!raw.empty() && std::isspace((unsigned char)raw.back())) raw.pop_back();
    if (raw.rfind("dense<", 0) != 0) throw ParseError("unsupported constant literal: " + raw.substr(0, 40));
    std::string body = raw.substr(6, raw.size() - 7);
    const int es = dtype_size(t.dtype);
    const int64_t n = t.numel();
    if (!body.empty() && body[0] == '"') {
      // hex blob "0x...." (little-endian bytes of the whole tensor)
      std::string hex = body.substr(1, body.size() - 2);
      if (hex.rfind("0x", 0) == 0 || hex.rfind("0X", 0) == 0) hex = hex.substr(2);
      std::vector<uint8_t> bytes(hex.size() / 2);
      for (size_t i = 0; i < bytes.size(); ++i)
        bytes[i] = (uint8_t)std::strtol(hex.substr(2 * i, 2).c_str(), nullptr, 16);
      if ((int64_t)bytes.size() == (int64_t)es && n != 1) {
        cd.splat = true;
      } else if ((int64_t)bytes.size() != n * es) {
        throw ParseError("hex constant size mismatch");
      }
      cd.bytes = bytes;
      return;
    }
    std::vector<std::string> elems;
    size_t i = 0;
    while (i < body.size()) {
      char ch = body[i];
      if (ch == '[' || ch == ']' || ch == ',' || std::isspace((unsigned char)ch)) { ++i; continue; }
      if (ch == '(') throw ParseError("complex constants are not supported");
      size_t e = i;
      while (e < body.size() && body[e] != ',' && body[e] != ']' && !std::isspace((unsigned char)body[e])) ++e;
      elems.push_back(body.substr(i, e - i));
      i = e;
    }
    if (elems.size() == 1 && n != 1) cd.splat = true;
    else if ((int64_t)elems.size() != n) throw ParseError("constant element count mismatch");
    cd.bytes.resize(elems.size() * es);
    for (size_t k = 0; k < elems.size(); ++k) encode_elem(elems[k], t.dtype, cd.bytes.data() + k * es);
  }
  static void encode_elem(const std::string& e, DType dt, uint8_t* out) {
    const int es = dtype_size(dt);
    if (e.rfind("0x", 0) == 0 || e.rfind("0X", 0) == 0) {
      uint64_t bits = std::stoull(e.substr(2), nullptr, 16);
      std::memcpy(out, &bits, es);
      return;
    }
    if (e == "true" || e == "false") {
      uint64_t v = e == "true";
      if (dtype_is_float(dt)) { double d = (double)v; write_float(d, dt, out); }
      else std::memcpy(out, &v, es);
      return;
    }
    if (dtype_is_float(dt)) {
      double d;
      if (e == "inf" || e == "+inf") d = INFINITY;
      else if (e == "-inf") d = -INFINITY;
      else if (e == "nan" || e == "-nan") d = NAN;
      else d = std::strtod(e.c_str(), nullptr);
      write_float(d, dt, out);
      return;
    }
    if (dtype_is_unsigned(dt) || dt == DType::PRED) {
      uint64_t v = std::stoull(e);
      std::memcpy(out, &v, es);
    } else {
      int64_t v = std::stoll(e);
      std::memcpy(out, &v, es);  // little endian truncation
    }
  }
  static void write_float(double d, DType dt, uint8_t* out) {
    if (dt == DType::F32) { float f = (float)d; std::memcpy(out, &f, 4); }
    else if (dt == DType::F64) { std::memcpy(out, &d, 8); }
    else if (dt == DType::BF16) { uint16_t b = f32_to_bf16_bits((float)d); std::memcpy(out, &b, 2); }
    else throw ParseError("f16 constants are not supported");
  }
};

}  // namespace

// Structural checks after parsing: the attribute lists and dimension numbers
// that the planner and the code generator index by rank must have the
// operand's rank and name dimensions that exist.  The parser fills defaults
// for absent optional attributes, so every valid program passes; a program
// whose attribute text was malformed is rejected here instead of being
// indexed out of range later.
namespace {
void verify_graph(const Graph& g) {
  auto fail = [&](const Node& n, const std::string& what) {
    throw PjrtErr(3, std::string("invalid ") + op_name(n.op) + (n.name.empty() ? "" : " " + n.name) +
                         ": " + what);
  };
  auto in_range = [](const std::vector<int64_t>& v, int64_t r) {
    for (int64_t d : v)
      if (d < 0 || d >= r) return false;
    return true;
  };
  auto distinct = [](std::vector<int64_t> v) {
    std::sort(v.begin(), v.end());
    return std::adjacent_find(v.begin(), v.end()) == v.end();
  };
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    const Node& n = g.nodes[i];
    for (const ValueRef& o : n.operands)
      if (o.node < 0 || (size_t)o.node >= i || o.idx < 0 ||
          (size_t)o.idx >= g.nodes[o.node].results.size())
        fail(n, "operand refers to no earlier value");
    for (const TensorType& t : n.results)
      for (int64_t d : t.dims)
        if (d < 0) fail(n, "negative dimension");
    for (const auto& r : n.regions) verify_graph(*r);
    if (n.results.empty() || n.op == Op::Return || n.op == Op::Tuple || n.op == Op::Call ||
        n.op == Op::CustomCall || n.op == Op::OptimizationBarrier || n.op == Op::GetTupleElement)
      continue;
    const TensorType& rt = n.results[0];
    const int R = rt.rank();
    const int I = n.operands.empty() ? 0 : g.type(n.operands[0]).rank();
    const std::vector<int64_t>* idims = n.operands.empty() ? nullptr : &g.type(n.operands[0]).dims;
    // a body computes one value per reduced input from twice as many arguments
    auto body = [&](size_t r, size_t outs, size_t params) {
      if (n.regions.size() <= r) fail(n, "needs a body");
      const Graph& b = *n.regions[r];
      if (b.outputs.size() != outs) fail(n, "body returns " + std::to_string(b.outputs.size()) +
                                                " values, needs " + std::to_string(outs));
      for (const Node& x : b.nodes)
        if (x.op == Op::Parameter && (x.param_index < 0 || (size_t)x.param_index >= params))
          fail(n, "body parameter out of range");
    };
    switch (n.op) {
      case Op::Reduce:
      case Op::ReduceWindow:
        if (n.operands.empty() || n.operands.size() % 2 != 0) fail(n, "needs inputs and as many init values");
        body(0, n.operands.size() / 2, n.operands.size());
        break;
      case Op::Scatter:
        if (n.operands.size() < 3 || n.operands.size() % 2 != 1) fail(n, "needs inputs, indices and updates");
        body(0, (n.operands.size() - 1) / 2, n.operands.size() - 1);
        break;
      case Op::SelectAndScatter:
        if (n.operands.size() != 3) fail(n, "needs operand, source and init value");
        body(0, 1, 2);
        body(1, 1, 2);
        break;
      case Op::AllReduce:  // one binary computation, applied to every operand
        body(0, 1, 2);
        break;
      default:
        break;
    }
    if (n.op >= Op::Neg && n.op <= Op::Convert) {
      const size_t arity = n.op <= Op::Real ? 1
                           : n.op <= Op::ShiftRightLogical || n.op == Op::Compare ? 2
                           : n.op == Op::Select || n.op == Op::Clamp ? 3 : 1;
      if (n.operands.size() != arity) fail(n, "needs " + std::to_string(arity) + " operands");
      for (size_t k = 0; k < n.operands.size(); ++k) {
        const TensorType& t = g.type(n.operands[k]);
        const bool scalar_ok = (n.op == Op::Select && k == 0) || (n.op == Op::Clamp && k != 1);
        if (t.dims != rt.dims && !(scalar_ok && t.rank() == 0))
          fail(n, "operand shape differs from the result shape");
      }
      continue;
    }
    switch (n.op) {
      case Op::BroadcastInDim:
        if ((int)n.dims.size() != I || !in_range(n.dims, R) || !distinct(n.dims)) fail(n, "bad broadcast_dimensions");
        for (int k = 0; k < I; ++k)
          if ((*idims)[k] != 1 && (*idims)[k] != rt.dims[n.dims[k]]) fail(n, "operand dimension mismatch");
        break;
      case Op::Transpose:
        if ((int)n.dims.size() != I || I != R || !in_range(n.dims, I) || !distinct(n.dims))
          fail(n, "permutation is not one of the operand's dimensions");
        for (int k = 0; k < R; ++k)
          if (rt.dims[k] != (*idims)[n.dims[k]]) fail(n, "result shape is not the permuted operand shape");
        break;
      case Op::Reshape:
        if (g.type(n.operands.at(0)).numel() != rt.numel()) fail(n, "element count changes");
        break;
      case Op::Slice:
        if ((int)n.start.size() != I || (int)n.limit.size() != I || (int)n.strides.size() != I)
          fail(n, "start / limit / strides do not match the operand rank");
        for (int k = 0; k < I; ++k)
          if (n.start[k] < 0 || n.start[k] > n.limit[k] || n.limit[k] > (*idims)[k] || n.strides[k] < 1)
            fail(n, "slice bounds out of range");
        if (R != I) fail(n, "result rank differs from the operand rank");
        for (int k = 0; k < I; ++k)
          if (rt.dims[k] != (n.limit[k] - n.start[k] + n.strides[k] - 1) / n.strides[k])
            fail(n, "result shape does not match the slice");
        break;
      case Op::DynamicSlice:
        if ((int)n.limit.size() != I || (int)n.operands.size() != 1 + I) fail(n, "slice sizes / start indices do not match the operand rank");
        for (int k = 0; k < I; ++k)
          if (n.limit[k] < 0 || n.limit[k] > (*idims)[k]) fail(n, "slice size out of range");
        if (rt.dims != n.limit) fail(n, "result shape differs from the slice sizes");
        break;
      case Op::DynamicUpdateSlice:
        if ((int)n.operands.size() != 2 + I || g.type(n.operands.at(1)).rank() != I)
          fail(n, "update / start indices do not match the operand rank");
        if (rt.dims != *idims) fail(n, "result shape differs from the operand shape");
        for (int k = 0; k < I; ++k)
          if (g.type(n.operands[1]).dims[k] > (*idims)[k]) fail(n, "update larger than the operand");
        break;
      case Op::Pad:
        if ((int)n.pad_lo.size() != I || (int)n.pad_hi.size() != I ||
            !(n.pad_interior.empty() || (int)n.pad_interior.size() == I))
          fail(n, "padding does not match the operand rank");
        for (int64_t v : n.pad_interior)
          if (v < 0) fail(n, "negative interior padding");
        if (R != I) fail(n, "result rank differs from the operand rank");
        for (int k = 0; k < I; ++k) {
          const int64_t d = (*idims)[k], in = n.pad_interior.empty() ? 0 : n.pad_interior[k];
          if (rt.dims[k] != n.pad_lo[k] + n.pad_hi[k] + d + (d > 0 ? (d - 1) * in : 0))
            fail(n, "result shape does not match the padding");
        }
        break;
      case Op::Concatenate:
        if (n.axis < 0 || n.axis >= R) fail(n, "dimension out of range");
        {
          int64_t along = 0;
          for (const ValueRef& o : n.operands) {
            const TensorType& t = g.type(o);
            if (t.rank() != R) fail(n, "operand rank differs from the result rank");
            for (int k = 0; k < R; ++k)
              if (k != n.axis && t.dims[k] != rt.dims[k]) fail(n, "operand shapes differ off the axis");
            along += t.dims[n.axis];
          }
          if (along != rt.dims[n.axis]) fail(n, "result size along the axis is not the operands' sum");
        }
        break;
      case Op::Reverse:
        if (!in_range(n.dims, I)) fail(n, "dimension out of range");
        if (rt.dims != *idims) fail(n, "result shape differs from the operand shape");
        break;
      case Op::Iota:
        if (n.iota_dim < 0 || n.iota_dim >= R) fail(n, "iota_dimension out of range");
        break;
      case Op::Reduce:
        if (n.operands.size() % 2 != 0 || n.regions.empty()) fail(n, "needs inputs, init values and a body");
        if (!in_range(n.dims, I) || !distinct(n.dims)) fail(n, "dimensions out of range");
        {
          std::vector<int64_t> kept;
          for (int k = 0; k < I; ++k)
            if (std::find(n.dims.begin(), n.dims.end(), k) == n.dims.end()) kept.push_back((*idims)[k]);
          const size_t nin = n.operands.size() / 2;
          if (n.results.size() != nin) fail(n, "needs one result per input");
          for (size_t k = 0; k < nin; ++k)
            if (g.type(n.operands[k]).dims != *idims || n.results[k].dims != kept)
              fail(n, "result shape is not the operand shape without the reduced dimensions");
        }
        break;
      case Op::ReduceWindow:
        if ((int)n.window.size() != I || (int)n.window_strides.size() != I ||
            (int)n.base_dilation.size() != I || (int)n.window_dilation.size() != I ||
            (int)n.pad_lo.size() != I || (int)n.pad_hi.size() != I)
          fail(n, "window attributes do not match the operand rank");
        for (int k = 0; k < I; ++k)
          if (n.window[k] < 1 || n.window_strides[k] < 1 || n.base_dilation[k] < 1 || n.window_dilation[k] < 1)
            fail(n, "window sizes, strides and dilations must be positive");
        if (n.regions.empty()) fail(n, "needs a body");
        {
          const size_t nin = n.operands.size() / 2;
          if (n.results.size() != nin) fail(n, "needs one result per input");
          for (size_t j = 0; j < nin; ++j) {
            if (g.type(n.operands[j]).dims != *idims || n.results[j].rank() != I)
              fail(n, "result rank differs from the operand rank");
            for (int k = 0; k < I; ++k) {
              const int64_t d = (*idims)[k];
              const int64_t padded = n.pad_lo[k] + (d == 0 ? 0 : (d - 1) * n.base_dilation[k] + 1) + n.pad_hi[k];
              const int64_t win = (n.window[k] - 1) * n.window_dilation[k] + 1;
              const int64_t cnt = (padded == 0 || win > padded) ? 0 : (padded - win) / n.window_strides[k] + 1;
              if (n.results[j].dims[k] != cnt) fail(n, "result shape does not match the windows");
            }
          }
        }
        break;
      case Op::SelectAndScatter:
        if ((int)n.window.size() != I || (int)n.window_strides.size() != I || (int)n.pad_lo.size() != I)
          fail(n, "window attributes do not match the operand rank");
        for (int k = 0; k < I; ++k)
          if (n.window[k] < 1 || n.window_strides[k] < 1) fail(n, "window sizes and strides must be positive");
        if (rt.dims != *idims || g.type(n.operands[1]).rank() != I)
          fail(n, "result / source shapes do not match the operand");
        if ((int)n.pad_hi.size() != I) fail(n, "padding does not match the operand rank");
        for (int k = 0; k < I; ++k) {  // one source element per window
          const int64_t padded = n.pad_lo[k] + (*idims)[k] + n.pad_hi[k];
          const int64_t cnt = (padded <= 0 || n.window[k] > padded) ? 0 : (padded - n.window[k]) / n.window_strides[k] + 1;
          if (g.type(n.operands[1]).dims[k] != cnt) fail(n, "source shape does not match the windows");
        }
        break;
      case Op::DotGeneral: {
        if (n.operands.size() != 2) fail(n, "needs two operands");
        const int rr = g.type(n.operands[1]).rank();
        if (n.lhs_batch.size() != n.rhs_batch.size() || n.lhs_contract.size() != n.rhs_contract.size() ||
            !in_range(n.lhs_batch, I) || !in_range(n.lhs_contract, I) || !in_range(n.rhs_batch, rr) ||
            !in_range(n.rhs_contract, rr))
          fail(n, "dimension numbers out of range");
        {
          const TensorType& lt = g.type(n.operands[0]);
          const TensorType& qt = g.type(n.operands[1]);
          std::vector<int64_t> want;
          for (size_t k = 0; k < n.lhs_batch.size(); ++k) {
            if (lt.dims[n.lhs_batch[k]] != qt.dims[n.rhs_batch[k]]) fail(n, "batch sizes differ");
            want.push_back(lt.dims[n.lhs_batch[k]]);
          }
          for (size_t k = 0; k < n.lhs_contract.size(); ++k)
            if (lt.dims[n.lhs_contract[k]] != qt.dims[n.rhs_contract[k]]) fail(n, "contracting sizes differ");
          auto free_of = [&](const TensorType& t, const std::vector<int64_t>& b, const std::vector<int64_t>& c) {
            for (int k = 0; k < t.rank(); ++k)
              if (std::find(b.begin(), b.end(), k) == b.end() && std::find(c.begin(), c.end(), k) == c.end())
                want.push_back(t.dims[k]);
          };
          free_of(lt, n.lhs_batch, n.lhs_contract);
          free_of(qt, n.rhs_batch, n.rhs_contract);
          if (!distinct(n.lhs_batch) || !distinct(n.lhs_contract) || !distinct(n.rhs_batch) ||
              !distinct(n.rhs_contract) || rt.dims != want)
            fail(n, "result shape is not batch + lhs free + rhs free");
        }
        break;
      }
      case Op::Scatter: {
        if (rt.dims != *idims) fail(n, "result shape differs from the operand shape");
        const ScatterDims& S = n.scatter;
        const int ir = g.type(n.operands.at(1)).rank();
        const int ur = g.type(n.operands.at(n.operands.size() - 1)).rank();
        if (S.index_vector_dim < 0 || S.index_vector_dim > ir || !in_range(S.scatter_dims_to_operand_dims, I) ||
            !in_range(S.inserted_window_dims, I) || !in_range(S.input_batching_dims, I) ||
            !in_range(S.scatter_indices_batching_dims, ir) ||
            S.input_batching_dims.size() != S.scatter_indices_batching_dims.size() ||
            !in_range(S.update_window_dims, ur))
          fail(n, "scatter dimension numbers out of range");
        {
          // the updates' scatter dimensions are the indices' batch dimensions
          const TensorType& it = g.type(n.operands[1]);
          const TensorType& ut = g.type(n.operands.back());
          std::vector<int64_t> ibatch, ubatch;
          for (int k = 0; k < ir; ++k)
            if (k != S.index_vector_dim) ibatch.push_back(it.dims[k]);
          for (int k = 0; k < ur; ++k)
            if (std::find(S.update_window_dims.begin(), S.update_window_dims.end(), k) == S.update_window_dims.end())
              ubatch.push_back(ut.dims[k]);
          if (ibatch != ubatch) fail(n, "update scatter dimensions differ from the indices' batch dimensions");
          const int64_t nvec = S.index_vector_dim < ir ? it.dims[S.index_vector_dim] : 1;
          if ((int64_t)S.scatter_dims_to_operand_dims.size() != nvec)
            fail(n, "scatter_dims_to_operand_dims does not match the index vector");
        }
        break;
      }
      case Op::Gather: {
        const GatherDims& G = n.gather;
        const TensorType& it = g.type(n.operands.at(1));
        const int ir = it.rank();
        if ((int)G.slice_sizes.size() != I || G.index_vector_dim < 0 || G.index_vector_dim > ir ||
            !in_range(G.start_index_map, I) || !in_range(G.collapsed_slice_dims, I) ||
            !in_range(G.operand_batching_dims, I) || !in_range(G.start_indices_batching_dims, ir) ||
            G.operand_batching_dims.size() != G.start_indices_batching_dims.size() ||
            !in_range(G.offset_dims, R) || !distinct(G.offset_dims) || !distinct(G.start_index_map))
          fail(n, "gather dimension numbers out of range");
        for (int k = 0; k < I; ++k)
          if (G.slice_sizes[k] < 0 || G.slice_sizes[k] > (*idims)[k]) fail(n, "slice size out of range");
        const int64_t nvec = G.index_vector_dim < ir ? it.dims[G.index_vector_dim] : 1;
        if ((int64_t)G.start_index_map.size() != nvec) fail(n, "start_index_map does not match the index vector");
        // result: offset_dims take the kept slice sizes in order, the rest the
        // indices' batch dimensions in order
        std::vector<int64_t> offs, batch;
        for (int k = 0; k < I; ++k)
          if (std::find(G.collapsed_slice_dims.begin(), G.collapsed_slice_dims.end(), k) ==
                  G.collapsed_slice_dims.end() &&
              std::find(G.operand_batching_dims.begin(), G.operand_batching_dims.end(), k) ==
                  G.operand_batching_dims.end())
            offs.push_back(G.slice_sizes[k]);
        for (int k = 0; k < ir; ++k)
          if (k != G.index_vector_dim) batch.push_back(it.dims[k]);
        if (offs.size() != G.offset_dims.size() || (size_t)R != offs.size() + batch.size())
          fail(n, "result rank does not match the gather");
        size_t oj = 0, bj = 0;
        for (int k = 0; k < R; ++k) {
          const bool off = std::find(G.offset_dims.begin(), G.offset_dims.end(), k) != G.offset_dims.end();
          if (rt.dims[k] != (off ? offs[oj++] : batch[bj++])) fail(n, "result shape does not match the gather");
        }
        break;
      }
      case Op::Convolution: {
        const size_t sp = I >= 2 ? (size_t)(I - 2) : 0;
        if (n.operands.size() != 2 || n.window_strides.size() != sp || n.lhs_dilation.size() != sp ||
            n.rhs_dilation.size() != sp || n.pad_lo.size() != sp || n.pad_hi.size() != sp ||
            n.conv.in_spatial.size() != sp || n.conv.k_spatial.size() != sp || n.conv.out_spatial.size() != sp)
          fail(n, "window attributes do not match the number of spatial dimensions");
        const int kr = g.type(n.operands[1]).rank();
        if (kr != I || R != I) fail(n, "kernel / result rank differs from the input rank");
        {
          auto perm = [&](int64_t a, int64_t b, const std::vector<int64_t>& sp2, int r) {
            std::vector<int64_t> v = sp2;
            v.push_back(a);
            v.push_back(b);
            return (int)v.size() == r && in_range(v, r) && distinct(v);
          };
          if (!perm(n.conv.in_batch, n.conv.in_feature, n.conv.in_spatial, I) ||
              !perm(n.conv.k_in, n.conv.k_out, n.conv.k_spatial, kr) ||
              !perm(n.conv.out_batch, n.conv.out_feature, n.conv.out_spatial, R))
            fail(n, "dimension numbers are not a permutation of each operand's dimensions");
          const std::vector<int64_t>& kdims = g.type(n.operands[1]).dims;
          if (n.feature_groups == 1 && n.batch_groups == 1 &&
              ((*idims)[n.conv.in_feature] != kdims[n.conv.k_in] ||
               rt.dims[n.conv.out_feature] != kdims[n.conv.k_out] ||
               rt.dims[n.conv.out_batch] != (*idims)[n.conv.in_batch]))
            fail(n, "feature / batch sizes do not match");
        }
        if (!in_range(n.conv.in_spatial, I) || !in_range(n.conv.k_spatial, kr) || !in_range(n.conv.out_spatial, R) ||
            !in_range({n.conv.in_batch, n.conv.in_feature}, I) || !in_range({n.conv.k_in, n.conv.k_out}, kr) ||
            !in_range({n.conv.out_batch, n.conv.out_feature}, R))
          fail(n, "dimension numbers out of range");
        {
          const std::vector<int64_t>& kd = g.type(n.operands[1]).dims;
          for (size_t s2 = 0; s2 < sp; ++s2) {
            const int64_t in = (*idims)[n.conv.in_spatial[s2]], k = kd[n.conv.k_spatial[s2]];
            const int64_t padded = n.pad_lo[s2] + (in == 0 ? 0 : (in - 1) * n.lhs_dilation[s2] + 1) + n.pad_hi[s2];
            const int64_t win = k == 0 ? 0 : (k - 1) * n.rhs_dilation[s2] + 1;
            if (n.window_strides[s2] < 1 || n.lhs_dilation[s2] < 1 || n.rhs_dilation[s2] < 1)
              fail(n, "strides and dilations must be positive");
            const int64_t cnt = (padded <= 0 || win > padded) ? 0 : (padded - win) / n.window_strides[s2] + 1;
            if (rt.dims[n.conv.out_spatial[s2]] != cnt) fail(n, "result spatial size does not match the window");
          }
        }
        break;
      }
      default:
        break;
    }
  }
}
}  // namespace

Module parse_module(const std::string& text) {
  try {
    Parser p(text);
    Module m = p.run();
    for (const auto& f : m.funcs) verify_graph(*f.second);
    return m;
  } catch (const PjrtErr&) {
    throw;
  } catch (const ParseError& e) {
    throw PjrtErr(3, e.what());
  } catch (const std::exception& e) {
    throw PjrtErr(3, std::string("StableHLO parse error: ") + e.what());
  }
}

}  // namespace b200
