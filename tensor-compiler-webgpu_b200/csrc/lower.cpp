// lower.cpp -- the lowering half of the drop-in boundary, in the library itself.
//
// The reference's host turns a graph into launches with lower() (src/gpu/lower.js:68-114),
// lowerFused() (src/fusion/lower-fused.js:32-45) and fusedKernel() (src/fusion/codegen-fused.js:357-362),
// all emitting WGSL.  Here those entry points take the reference's Graph.toJSON form
// (src/ir/graph.js:48-50) -- fused nodes carrying {kind, pattern, body, output}, as its fusion pass
// (src/fusion/fuse.js:278-279) leaves them -- and emit CUDA C++ instantiating the library's sm_100a
// templates, with each kernel's grid, block, parameters, tensor maps and scratch.  The text produced is
// the same, character for character, as the repository's Python host produces, so a JavaScript host
// holding only this library gets the kernels (and the cubin cache entries) the tests judge.
//
// Emission rules (shared with the Python host):
//  * every body value is computed once per index context (a base index or a gathered one);
//  * scalar constants are inlined as their exact float32 bits;
//  * shapes and strides are compile-time constants; each load is classified as direct, row broadcast
//    (i % P), column broadcast (i / Q), scalar, or a general strided gather;
//  * environment overrides of the Python host's GEMM tile choices are not read: defaults only.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <optional>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "lower.h"

namespace tcb_detail {
int fail_msg(int status, const std::string& msg);
}

namespace tcl {

constexpr int SM_COUNT = 148;
constexpr int WG = 256;
constexpr int TC_MIN_K = 32;
constexpr i64 GEMM_BM = 128;
constexpr i64 SMEM_LIMIT = 227 * 1024;
constexpr i64 KPAD = 32;
constexpr i64 TMA_ATOM32 = (i64)1 << 32;
constexpr i64 GEMM_STAGING = 4 * 2 * 32 * 32 * 4;
constexpr int FS_MAX_REREAD = 8;
constexpr i64 TAIL_MIN_KB = 32;

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

static i64 cdiv(i64 a, i64 b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------- IR
static i64 size_of(const std::vector<i64>& s) {
  i64 n = 1;
  for (i64 d : s) n *= d;
  return n;
}

static std::vector<i64> strides_of(const std::vector<i64>& shape) {
  std::vector<i64> s(shape.size());
  i64 acc = 1;
  for (int i = (int)shape.size() - 1; i >= 0; --i) {
    s[i] = acc;
    acc *= shape[i];
  }
  return s;
}

static std::vector<i64> int_list(const Value& v) {
  std::vector<i64> out;
  for (auto& x : v.arr) out.push_back(x.as_int());
  return out;
}

static std::shared_ptr<Graph> graph_from_json(const Value& js);

static Node node_from_json(const Value& n, int id) {
  Node nd;
  nd.id = id;
  nd.op = n.at("op").as_string();
  for (auto& i : n.at("inputs").arr) nd.inputs.push_back((int)i.as_int());
  nd.shape = int_list(n.at("shape"));
  const Value* a = n.find("attrs");
  if (a && a->is_object()) {
    nd.attrs_json = *a;
    if (auto* v = a->find("name")) nd.name = v->as_string();
    if (auto* v = a->find("axis")) nd.axis = (int)v->as_int();
    if (auto* v = a->find("keepDims")) nd.keepDims = v->truthy();
    if (auto* v = a->find("perm"))
      for (auto& p : v->arr) nd.perm.push_back((int)p.as_int());
    if (auto* v = a->find("shape")) nd.attr_shape = int_list(*v);
    if (auto* v = a->find("value")) {
      nd.has_value = true;
      if (v->is_array()) {
        nd.scalar_value = false;
        for (auto& x : v->arr) nd.values.push_back(x.as_double());
      } else {
        nd.value = v->as_double();
      }
    }
    if (auto* v = a->find("kind")) nd.kind = v->as_string();
    if (auto* v = a->find("pattern")) nd.pattern = v->is_string() ? v->as_string() : "";
    if (auto* v = a->find("output")) nd.output = (int)v->as_int();
    if (auto* v = a->find("body")) nd.body = graph_from_json(*v);
  }
  for (int i : nd.inputs)
    if (i < 0 || i >= id) throw Error("node " + std::to_string(id) + ": input " + std::to_string(i) + " is not an earlier node");
  return nd;
}

static std::shared_ptr<Graph> graph_from_json(const Value& js) {
  auto g = std::make_shared<Graph>();
  const Value& nodes = js.at("nodes");
  for (size_t k = 0; k < nodes.arr.size(); ++k) g->nodes.push_back(node_from_json(nodes.arr[k], (int)k));
  return g;
}

static bool is_bin(const std::string& op) { return op == "add" || op == "sub" || op == "mul" || op == "div"; }
static bool is_un(const std::string& op) {
  return op == "neg" || op == "exp" || op == "log" || op == "relu" || op == "tanh" || op == "sqrt" || op == "step" ||
         op == "stopGradient";
}
static std::string bin_fn(const std::string& op) { return "tcb::op_" + op; }
static std::string un_fn(const std::string& op) { return op == "stopGradient" ? "tcb::op_copy" : "tcb::op_" + op; }

// A one-op body: inputs a0.. with the given shapes, the op, its result.
static std::shared_ptr<Graph> one_op_body(const Node& like, const std::vector<std::vector<i64>>& shapes, int* out) {
  auto g = std::make_shared<Graph>();
  for (size_t k = 0; k < shapes.size(); ++k) {
    Node in;
    in.id = (int)k;
    in.op = "input";
    in.name = "a" + std::to_string(k);
    in.shape = shapes[k];
    in.attr_shape = shapes[k];
    g->nodes.push_back(in);
  }
  Node n = like;
  n.id = (int)shapes.size();
  n.inputs.clear();
  for (size_t k = 0; k < shapes.size(); ++k) n.inputs.push_back((int)k);
  n.body.reset();
  g->nodes.push_back(n);
  *out = n.id;
  return g;
}

// ---------------------------------------------------------------- index gathers
static std::string f32_literal(double v) {
  float f = (float)v;
  uint32_t b;
  std::memcpy(&b, &f, 4);
  char buf[40];
  snprintf(buf, sizeof buf, "tcb::bits(0x%08xu)", b);
  return buf;
}

static std::vector<i64> gather_strides(const std::string& op, const std::vector<i64>& out_shape,
                                       const std::vector<i64>& in_shape, const std::vector<int>& perm) {
  std::vector<i64> nat = strides_of(in_shape);
  std::vector<i64> g;
  if (op == "broadcast") {
    int lead = (int)out_shape.size() - (int)in_shape.size();
    for (int i = 0; i < (int)out_shape.size(); ++i)
      g.push_back((i < lead || in_shape[i - lead] == 1) ? 0 : nat[i - lead]);
    return g;
  }
  if (op == "transpose") {
    for (int p : perm) g.push_back(nat[p]);
    return g;
  }
  if (op == "reshape") return strides_of(out_shape);
  throw Error("not a strided move: " + op);
}

struct Gather {
  std::string kind;
  std::vector<std::pair<i64, i64>> dims;
  i64 P = 0, Q = 0;

  Gather() = default;
  Gather(const std::vector<i64>& out_shape, const std::vector<i64>& gs) {
    std::vector<std::pair<i64, i64>> raw;
    for (size_t i = 0; i < out_shape.size(); ++i)
      if (out_shape[i] != 1) raw.emplace_back(out_shape[i], gs[i]);
    for (auto [d, g] : raw) {
      if (!dims.empty() && dims.back().second == g * d) {
        dims.back() = {dims.back().first * d, g};
      } else if (!dims.empty() && dims.back().second == 0 && g == 0) {
        dims.back() = {dims.back().first * d, 0};
      } else {
        dims.emplace_back(d, g);
      }
    }
    int n = (int)dims.size();
    std::vector<int> nz;
    for (int i = 0; i < n; ++i)
      if (dims[i].second != 0) nz.push_back(i);
    if (nz.empty()) {
      kind = "scalar";
    } else if (n == 1 && dims[0].second == 1) {
      kind = "identity";
    } else if (nz.size() == 1 && nz[0] == n - 1 && dims[nz[0]].second == 1) {
      kind = "rowb";
      P = dims.back().first;
    } else if (n == 2 && dims[0].second == 1 && dims[1].second == 0) {
      kind = "colb";
      Q = dims[1].first;
    } else {
      kind = "general";
    }
  }

  std::string expr(const std::string& i, const std::string& T) const {
    if (kind == "scalar") return "((" + T + ")0)";
    if (kind == "identity") return "(" + i + ")";
    if (kind == "rowb") return "((" + i + ") % (" + T + ")" + std::to_string(P) + "ull)";
    if (kind == "colb") return "((" + i + ") / (" + T + ")" + std::to_string(Q) + "ull)";
    struct Ax { i64 d, g, s; };
    std::vector<Ax> out;
    i64 ost = 1;
    for (int k = (int)dims.size() - 1; k >= 0; --k) {
      out.push_back({dims[k].first, dims[k].second, ost});
      ost *= dims[k].first;
    }
    std::reverse(out.begin(), out.end());
    std::vector<std::string> terms;
    for (size_t k = 0; k < out.size(); ++k) {
      if (out[k].g == 0) continue;
      std::string q = out[k].s == 1 ? "(" + i + ")" : "((" + i + ") / (" + T + ")" + std::to_string(out[k].s) + "ull)";
      if (k > 0) q = "(" + q + " % (" + T + ")" + std::to_string(out[k].d) + "ull)";
      terms.push_back(out[k].g == 1 ? q : q + " * (" + T + ")" + std::to_string(out[k].g) + "ull");
    }
    std::string s = "(";
    for (size_t k = 0; k < terms.size(); ++k) s += (k ? " + " : "") + terms[k];
    return s + ")";
  }

  // A general gather whose innermost run is contiguous (stride 1, a multiple of 4 long) and whose
  // other strides are multiples of 4: 4 consecutive outputs from a multiple of 4 read 4 aligned floats.
  bool vec4() const {
    if (kind != "general" || dims.empty()) return false;
    if (dims.back().second != 1 || dims.back().first % 4 != 0) return false;
    for (size_t k = 0; k + 1 < dims.size(); ++k)
      if (dims[k].second % 4 != 0) return false;
    return true;
  }

  std::string key() const {
    std::string s = kind + "[";
    for (auto& d : dims) s += std::to_string(d.first) + ":" + std::to_string(d.second) + ",";
    return s + "]";
  }
};

struct Ctx {
  std::string key;
  Ctx* parent = nullptr;
  Gather gather;
};

static std::string idx_type(i64 n) { return n < ((i64)1 << 32) - 1 ? "u32" : "u64"; }

static std::string chain_index(const Ctx* ctx, const std::string& base, const std::string& T) {
  if (!ctx->parent) return base;
  return ctx->gather.expr(chain_index(ctx->parent, base, T), T);
}

// ---------------------------------------------------------------- the body emitter
struct Emitter {
  const Graph& b;
  std::function<std::string(int, Ctx*)> leaf;
  std::function<std::optional<std::string>(int, Ctx*)> special;
  std::map<std::pair<std::string, int>, std::string> memo;
  std::vector<std::string> lines, row_lines;
  int counter = 0;
  std::map<std::string, std::unique_ptr<Ctx>> ctxs;

  explicit Emitter(const Graph& body) : b(body) {}

  Ctx* child(Ctx* ctx, const Gather& g) {
    if (g.kind == "identity") return ctx;
    std::string key = "(" + ctx->key + "|" + g.key() + ")";
    auto it = ctxs.find(key);
    if (it != ctxs.end()) return it->second.get();
    auto c = std::make_unique<Ctx>();
    c->key = key;
    c->parent = ctx;
    c->gather = g;
    Ctx* p = c.get();
    ctxs[key] = std::move(c);
    return p;
  }

  void forget_unless_row() {
    for (auto it = memo.begin(); it != memo.end();) {
      if (it->first.first != "r") it = memo.erase(it);
      else ++it;
    }
  }

  std::string value(int nid, Ctx* ctx) {
    auto key = std::make_pair(ctx->key, nid);
    auto hit = memo.find(key);
    if (hit != memo.end()) return hit->second;
    if (special) {
      auto s = special(nid, ctx);
      if (s) {
        memo[key] = *s;
        return *s;
      }
    }
    const Node& node = b.nodes[nid];
    const std::string& op = node.op;
    std::string v;
    if (op == "input") {
      v = leaf(std::stoi(node.name.substr(1)), ctx);
      memo[key] = v;
      return v;
    }
    if (op == "const") {
      v = f32_literal(node.scalar_value ? node.value : node.values.at(0));
      memo[key] = v;
      return v;
    }
    if (op == "reshape") {
      v = value(node.inputs[0], ctx);
      memo[key] = v;
      return v;
    }
    if (op == "broadcast" || op == "transpose") {
      const Node& src = b.nodes[node.inputs[0]];
      if (src.op == "const") {
        v = value(src.id, ctx);
      } else {
        Gather g(node.shape, gather_strides(op, node.shape, src.shape, node.perm));
        v = value(src.id, child(ctx, g));
      }
      memo[key] = v;
      return v;
    }
    std::string expr;
    if (is_bin(op)) {
      std::string a = value(node.inputs[0], ctx);
      std::string c = value(node.inputs[1], ctx);
      expr = bin_fn(op) + "(" + a + ", " + c + ")";
    } else if (is_un(op)) {
      expr = un_fn(op) + "(" + value(node.inputs[0], ctx) + ")";
    } else {
      throw Error("fused codegen: no rule for '" + op + "'");
    }
    std::string name = "v" + std::to_string(counter++);
    lines.push_back("const float " + name + " = " + expr + ";");
    memo[key] = name;
    return name;
  }
};

static std::string join(const std::vector<std::string>& xs, const std::string& sep) {
  std::string s;
  for (size_t k = 0; k < xs.size(); ++k) s += (k ? sep : "") + xs[k];
  return s;
}

static Value num(i64 v) {
  Value x;
  x.kind = Value::Number;
  x.num = (double)v;
  x.integral = true;
  return x;
}
static Value boolean(bool v) {
  Value x;
  x.kind = Value::Bool;
  x.b = v;
  return x;
}
static Value str(const std::string& s) {
  Value x;
  x.kind = Value::String;
  x.str = s;
  return x;
}
static Value arr(std::initializer_list<Value> xs) {
  Value x;
  x.kind = Value::Array;
  x.arr = xs;
  return x;
}

static Call make_call(const std::string& name, std::array<i64, 3> grid, std::array<i64, 3> block, i64 smem = 0,
                      std::vector<i64> params = {}) {
  Call c;
  c.name = name;
  for (int k = 0; k < 3; ++k) {
    c.grid[k] = grid[k];
    c.block[k] = block[k];
  }
  c.smem = smem;
  c.params = std::move(params);
  return c;
}

static std::array<i64, 3> grid1d(i64 n, i64 per_thread = 4, i64 block = WG, i64 waves = 8) {
  i64 chunks = std::max<i64>(1, cdiv(n, per_thread));
  return {std::max<i64>(1, std::min<i64>(cdiv(chunks, block), (i64)SM_COUNT * waves)), 1, 1};
}

// ---------------------------------------------------------------- elementwise
struct EwLoads {
  std::string T;
  std::vector<std::string> fields, stmts, per_lane;
  std::map<std::pair<std::string, int>, std::string> seen;

  std::string leaf(int k, Ctx* ctx) {
    auto key = std::make_pair(ctx->key, k);
    auto it = seen.find(key);
    if (it != seen.end()) return it->second;
    std::string ptr = "reinterpret_cast<const float*>(a.in[" + std::to_string(k) + "])";
    std::string name = "x" + std::to_string(seen.size());
    const Gather& g = ctx->gather;
    std::string ref;
    if (!ctx->parent) {
      fields.push_back("float " + name + "[W];");
      stmts.push_back("tcb::load<W>(r." + name + ", " + ptr + " + i0);");
      ref = "r." + name + "[l]";
    } else if (!ctx->parent->parent && g.kind == "rowb" && g.P % 4 == 0) {
      fields.push_back("float " + name + "[W];");
      stmts.push_back("tcb::load<W>(r." + name + ", " + ptr + " + ((" + T + ")i0 % (" + T + ")" + std::to_string(g.P) +
                      "ull));");
      ref = "r." + name + "[l]";
    } else if (!ctx->parent->parent && (g.kind == "scalar" || (g.kind == "colb" && g.Q % 4 == 0))) {
      fields.push_back("float " + name + ";");
      stmts.push_back("r." + name + " = tcb::ld1(" + ptr + " + " + g.expr("(" + T + ")i0", T) + ");");
      ref = "r." + name;
    } else if (!ctx->parent->parent && g.vec4()) {
      fields.push_back("float " + name + "[W];");
      stmts.push_back("tcb::load<W>(r." + name + ", " + ptr + " + " + g.expr("(" + T + ")i0", T) + ");");
      ref = "r." + name + "[l]";
    } else {
      fields.push_back("float " + name + "[W];");
      per_lane.push_back("r." + name + "[l] = tcb::ld1(" + ptr + " + " +
                         chain_index(ctx, "((" + T + ")i0 + (" + T + ")l)", T) + ");");
      ref = "r." + name + "[l]";
    }
    seen[key] = ref;
    return ref;
  }
};

static std::string ew_body_struct(const Graph& body, int out_id, i64 n) {
  EwLoads loads;
  loads.T = idx_type(n);
  Emitter em(body);
  em.leaf = [&](int k, Ctx* c) { return loads.leaf(k, c); };
  Ctx base{"i", nullptr, Gather()};
  std::string out = em.value(out_id, &base);
  std::string fields = loads.fields.empty() ? "float unused_;" : join(loads.fields, "\n    ");
  std::string stmts = join(loads.stmts, "\n    ");
  std::string per_lane = loads.per_lane.empty()
                             ? ""
                             : "#pragma unroll\n    for (int l = 0; l < W; ++l) {\n      " +
                                   join(loads.per_lane, "\n      ") + "\n    }";
  std::string comp = join(em.lines, "\n      ");
  return "struct Body {\n"
         "  template <int W> struct Regs {\n"
         "    " + fields + "\n"
         "  };\n"
         "  template <int W> __device__ __forceinline__ static void load(const tcb::Args& a, u64 i0, Regs<W>& r) {\n"
         "    " + stmts + "\n"
         "    " + per_lane + "\n"
         "  }\n"
         "  template <int W> __device__ __forceinline__ static void compute(const Regs<W>& r, float (&o)[W]) {\n"
         "#pragma unroll\n"
         "    for (int l = 0; l < W; ++l) {\n"
         "      " + comp + "\n"
         "      o[l] = " + out + ";\n"
         "    }\n"
         "  }\n"
         "};\n";
}

static std::string elementwise_source(const Graph& body, int out_id, i64 n, const std::string& tag) {
  return "// " + tag + ": generated from a body of " + std::to_string(body.nodes.size()) + " nodes, " +
         std::to_string(n) + " elements\n#include \"tcb/common.cuh\"\n#define TCB_W 4\n" +
         ew_body_struct(body, out_id, n) + "#include \"tcb/elementwise.cuh\"\n";
}

static Launch ew_launch(const Graph& body, int out_id, i64 n, const std::string& kind, int node_id,
                        const std::string& op, const std::string* pattern, const std::vector<int>& inputs,
                        const std::string& sabotage, const std::string& tag) {
  Launch l;
  l.node = node_id;
  l.op = op;
  l.kind = kind;
  if (pattern) {
    l.pattern = *pattern;
    l.has_pattern = true;
  }
  l.inputs = inputs;
  l.code = elementwise_source(body, out_id, n, tag);
  i64 count = sabotage == "fused-bounds-off-by-one" ? n + 1 : n;
  l.calls.push_back(make_call("tcb_elementwise", grid1d(n), {WG, 1, 1}, 0, {count}));
  return l;
}

// ---------------------------------------------------------------- rowwise
struct Geo {
  i64 vec, tpr, groups, slots, items, block;
  bool cache;
};

static i64 pow2ceil(i64 x) {
  i64 p = 1;
  x = std::max<i64>(1, x);
  while (p < x) p <<= 1;
  return p;
}

static Geo rowwise_geometry(i64 R, i64 C, i64 n_leaves, i64 elems_per_thread = 16) {
  (void)R;
  Geo g;
  g.vec = C % 4 == 0 ? 4 : 1;
  g.tpr = std::min<i64>(1024, std::max<i64>(32, pow2ceil(cdiv(C, elems_per_thread))));
  g.groups = std::max<i64>(1, 256 / g.tpr);
  g.slots = cdiv(C, g.tpr * g.vec);
  g.items = g.slots * g.vec;
  g.cache = g.items <= 32 && g.items * std::max<i64>(1, n_leaves) <= 128;
  g.block = g.tpr * g.groups;
  return g;
}

struct ElemLoad {
  std::string name, kind, ptr, idx;
};

struct RowLoads {
  const Graph& body;
  i64 R, C;
  std::string T;
  i64 vec;
  bool cache;
  std::map<std::pair<std::string, int>, std::string> row, elem;
  std::vector<std::string> order_row;
  std::vector<ElemLoad> order_elem;
  std::vector<std::unique_ptr<Ctx>> roots;

  RowLoads(const Graph& b, i64 R_, i64 C_, std::string T_, i64 v, bool c) : body(b), R(R_), C(C_), T(T_), vec(v), cache(c) {}

  std::string leaf(int k, Ctx* ctx) {
    std::string ptr = "reinterpret_cast<const float*>(a.in[" + std::to_string(k) + "])";
    Ctx* root = ctx;
    while (root->parent) root = root->parent;
    if (root->key == "r") {
      auto key = std::make_pair(ctx->key, k);
      auto it = row.find(key);
      if (it == row.end()) {
        std::string name = "R" + std::to_string(row.size());
        row[key] = name;
        std::string idx = chain_index(ctx, "(" + T + ")r", T);
        order_row.push_back("const float " + name + " = active ? tcb::ld1(" + ptr + " + " + idx + ") : 0.0f;");
        return name;
      }
      return it->second;
    }
    const Gather& g = ctx->gather;
    if (ctx->parent && ctx->parent->key == "e" && g.kind == "colb" && g.Q == C) {
      roots.push_back(std::make_unique<Ctx>(Ctx{"r", nullptr, Gather()}));
      return leaf(k, roots.back().get());
    }
    auto key = std::make_pair(ctx->key, k);
    auto it = elem.find(key);
    if (it != elem.end()) return it->second;
    std::string name = "L" + std::to_string(elem.size());
    std::string kind, idx;
    if (ctx->key == "e") {
      kind = "vec";
      idx = "e";
    } else if (ctx->parent && ctx->parent->key == "e" && g.kind == "rowb" && g.P % 4 == 0) {
      kind = "vec";
      idx = "(e % (" + T + ")" + std::to_string(g.P) + "ull)";
    } else if (ctx->parent && ctx->parent->key == "e" && (g.kind == "scalar" || (g.kind == "colb" && g.Q % 4 == 0))) {
      kind = "one";
      idx = g.expr("e", T);
    } else {
      kind = "lane";
      idx = chain_index(ctx, "(e + (" + T + ")l)", T);
    }
    if (vec == 1 && kind == "vec") {
      kind = "lane";
      idx = idx != "e" ? idx : "(e + l)";
    }
    order_elem.push_back({name, kind, ptr, idx});
    std::string ref = cache ? name + "[q]" : name + "[l]";
    elem[key] = ref;
    return ref;
  }

  std::vector<std::string> load_stmts(const std::string& slot_var) const {
    std::vector<std::string> out;
    std::string V = std::to_string(vec);
    for (auto& e : order_elem) {
      std::string dst = cache ? e.name + "[" + slot_var + " * " + V + " + l]" : e.name + "[l]";
      if (e.kind == "vec") {
        out.push_back("{ float t_[" + V + "]; tcb::load<" + V + ">(t_, " + e.ptr + " + " + e.idx + ");" +
                      " _Pragma(\"unroll\") for (int l = 0; l < " + V + "; ++l) " + dst + " = t_[l]; }");
      } else if (e.kind == "one") {
        out.push_back("{ const float t_ = tcb::ld1(" + e.ptr + " + " + e.idx + ");" +
                      " _Pragma(\"unroll\") for (int l = 0; l < " + V + "; ++l) " + dst + " = t_; }");
      } else {
        out.push_back("_Pragma(\"unroll\") for (int l = 0; l < " + V + "; ++l) " + dst + " = tcb::ld1(" + e.ptr + " + " +
                      e.idx + ");");
      }
    }
    return out;
  }
};

struct Phase {
  std::vector<std::string> row_lines, elem_lines;
  int k;
  std::string init, comb, red;
};

struct RowOut {
  std::vector<std::string> row_lines, elem_lines;
  std::string ov;
  bool out_row;
};

static void rowwise_walk(const Graph& body, RowLoads& loads, const std::vector<const Node*>& reductions, int out_id,
                         const std::function<bool(int)>& row_tier, const std::string& pattern,
                         const std::string& sabotage, i64 TPR, i64 GROUPS, std::vector<Phase>* phases, RowOut* outp) {
  std::map<int, std::string> reduced;
  Emitter em(body);
  em.leaf = [&](int k, Ctx* c) { return loads.leaf(k, c); };
  Ctx E{"e", nullptr, Gather()}, ROW{"r", nullptr, Gather()};
  Ctx ROWV{"r", nullptr, Gather()};
  std::function<std::string(int)> row_value = [&](int nid) -> std::string {
    auto key = std::make_pair(std::string("r"), nid);
    auto it = em.memo.find(key);
    if (it != em.memo.end()) return it->second;
    std::vector<std::string> saved;
    std::swap(saved, em.lines);
    std::string v = em.value(nid, &ROWV);
    em.row_lines.insert(em.row_lines.end(), em.lines.begin(), em.lines.end());
    std::swap(saved, em.lines);
    return v;
  };
  em.special = [&](int nid, Ctx* ctx) -> std::optional<std::string> {
    const Node& node = body.nodes[nid];
    auto it = reduced.find(nid);
    if (it != reduced.end()) return it->second;
    if (ctx->key == "e" && row_tier(nid)) return row_value(nid);
    if (ctx->key == "e" && node.op == "broadcast") {
      const Node& src = body.nodes[node.inputs[0]];
      if (row_tier(src.id) && src.op != "input" && src.op != "const") return row_value(src.id);
    }
    return std::nullopt;
  };
  for (size_t k = 0; k < reductions.size(); ++k) {
    const Node* rd = reductions[k];
    em.forget_unless_row();
    em.lines.clear();
    em.row_lines.clear();
    std::string v = em.value(rd->inputs[0], &E);
    bool is_max = rd->op == "max";
    std::string ks = std::to_string(k);
    std::string red = "tcb::group_reduce<" + std::to_string(TPR) + ", " + std::to_string(GROUPS) + ", " +
                      (is_max ? "true" : "false") + ">(acc" + ks + ", red)";
    if (sabotage == "layernorm-tree-short" && pattern == "layernorm") red = "acc" + ks;
    if (sabotage == "softmax-no-max" && is_max && (pattern == "softmax" || pattern == "log-softmax"))
      red = "((void)" + red + ", 0.0f)";
    phases->push_back({em.row_lines, em.lines, (int)k, is_max ? "-__int_as_float(0x7f800000)" : "0.0f",
                       is_max ? "tcb::op_max(acc" + ks + ", " + v + ")" : "tcb::op_add(acc" + ks + ", " + v + ")", red});
    reduced[rd->id] = "red" + ks;
    em.memo[std::make_pair(std::string("r"), rd->id)] = "red" + ks;
  }
  em.forget_unless_row();
  em.lines.clear();
  em.row_lines.clear();
  bool out_row = row_tier(out_id);
  std::string ov = em.value(out_id, out_row ? &ROW : &E);
  *outp = {em.row_lines, em.lines, ov, out_row};
}

static std::string lines_at(const std::vector<std::string>& xs, int ind) {
  return join(xs, "\n" + std::string(ind, ' '));
}

static std::string rowwise_source(const Graph& body, int out_id, const std::string& pattern, const std::string& sabotage,
                                  Geo* geo_out, i64* R_out, i64* C_out) {
  std::vector<const Node*> reductions;
  for (auto& n : body.nodes)
    if (n.op == "sum" || n.op == "max") reductions.push_back(&n);
  if (reductions.empty()) throw Error("rowwise body without a reduction");
  const std::vector<i64>& S = body.nodes[reductions[0]->inputs[0]].shape;
  i64 C = S.back();
  i64 R = size_of(S) / C;
  std::string T = idx_type(R * C);
  auto row_tier = [&](int nid) {
    i64 s = size_of(body.nodes[nid].shape);
    return s == R && s != R * C;
  };
  Geo geo = rowwise_geometry(R, C, 1);
  {
    RowLoads dry(body, R, C, T, geo.vec, true);
    std::vector<Phase> ph;
    RowOut ro;
    rowwise_walk(body, dry, reductions, out_id, row_tier, pattern, "", geo.tpr, geo.groups, &ph, &ro);
    geo = rowwise_geometry(R, C, (i64)dry.order_elem.size());
  }
  i64 V = geo.vec, TPR = geo.tpr, GROUPS = geo.groups, SLOTS = geo.slots, ITEMS = geo.items;
  bool CACHE = geo.cache;
  RowLoads loads(body, R, C, T, V, CACHE);
  std::vector<Phase> phases;
  RowOut ro;
  rowwise_walk(body, loads, reductions, out_id, row_tier, pattern, sabotage, TPR, GROUPS, &phases, &ro);
  std::string Vs = std::to_string(V), Cs = std::to_string(C), TPRs = std::to_string(TPR);

  auto item_loop = [&](const std::vector<std::string>& elem_lines, const std::vector<std::string>& tail, bool store) {
    std::string head, foot, qdef;
    if (CACHE) {
      head = "_Pragma(\"unroll\")\n      for (int s = 0; s < " + std::to_string(SLOTS) + "; ++s) {\n"
             "        const u32 c = (u32)(s * " + TPRs + " + t) * " + Vs + ";\n"
             "        if (active && c < " + Cs + "u) {\n"
             "          const " + T + " e = (" + T + ")r * (" + T + ")" + Cs + " + c; (void)e;";
      foot = "        }\n      }";
      qdef = "const int q = s * " + Vs + " + l; (void)q;";
    } else {
      std::vector<std::string> decl;
      for (auto& e : loads.order_elem) decl.push_back("float " + e.name + "[" + Vs + "];");
      head = "for (u32 c = (u32)t * " + Vs + "; active && c < " + Cs + "u; c += " + std::to_string(TPR * V) + "u) {\n"
             "        {\n"
             "          const " + T + " e = (" + T + ")r * (" + T + ")" + Cs + " + c; (void)e;\n"
             "          " + join(decl, " ") + "\n"
             "          " + lines_at(loads.load_stmts("0"), 10);
      foot = "        }\n      }";
      qdef = "";
    }
    std::vector<std::string> all = elem_lines;
    all.insert(all.end(), tail.begin(), tail.end());
    std::string body_ = "\n          " + std::string(store ? "float o_[" + Vs + "];" : "") + "\n"
                        "          _Pragma(\"unroll\")\n"
                        "          for (int l = 0; l < " + Vs + "; ++l) {\n"
                        "            " + qdef + "\n"
                        "            " + lines_at(all, 12) + "\n"
                        "          }\n"
                        "          " + std::string(store ? "tcb::store<" + Vs + ">(out + e, o_);" : "") + "\n";
    return head + body_ + foot;
  };

  std::vector<std::string> parts;
  for (auto& ph : phases) {
    std::string ks = std::to_string(ph.k);
    parts.push_back(lines_at(ph.row_lines, 6));
    parts.push_back("float acc" + ks + " = " + ph.init + ";");
    parts.push_back(item_loop(ph.elem_lines, {"acc" + ks + " = " + ph.comb + ";"}, false));
    parts.push_back("const float red" + ks + " = " + ph.red + ";");
  }
  parts.push_back(lines_at(ro.row_lines, 6));
  if (ro.out_row) parts.push_back("if (active && t == 0) out[r] = " + ro.ov + ";");
  else parts.push_back(item_loop(ro.elem_lines, {"o_[l] = " + ro.ov + ";"}, true));
  std::string cache_decl, cache_load;
  if (CACHE && !loads.order_elem.empty()) {
    std::vector<std::string> d, z;
    for (auto& e : loads.order_elem) {
      d.push_back("float " + e.name + "[" + std::to_string(ITEMS) + "];");
      z.push_back(e.name + "[s * " + Vs + " + l] = 0.0f;");
    }
    cache_decl = join(d, " ");
    cache_load = "_Pragma(\"unroll\")\n    for (int s = 0; s < " + std::to_string(SLOTS) + "; ++s) {\n"
                 "      const u32 c = (u32)(s * " + TPRs + " + t) * " + Vs + ";\n"
                 "      const " + T + " e = (" + T + ")r * (" + T + ")" + Cs + " + c; (void)e;\n"
                 "      if (active && c < " + Cs + "u) {\n"
                 "        " + lines_at(loads.load_stmts("s"), 8) + "\n"
                 "      } else {\n"
                 "        _Pragma(\"unroll\") for (int l = 0; l < " + Vs + "; ++l) { " + join(z, " ") + " }\n"
                 "      }\n"
                 "    }";
  }
  std::vector<std::string> nonempty;
  for (auto& p : parts)
    if (!p.empty()) nonempty.push_back(p);
  i64 nw = std::max<i64>(1, TPR / 32);
  std::string Rs = std::to_string(R), Gs = std::to_string(GROUPS);
  std::string src =
      "// rowwise (" + pattern + "): R=" + Rs + " C=" + Cs + ", " + TPRs + " threads per row, " + Gs +
      " rows per CTA, vec " + Vs + ", " + (CACHE ? "cached" : "streamed") + "\n"
      "#include \"tcb/common.cuh\"\n"
      "#include \"tcb/rowwise.cuh\"\n"
      "extern \"C\" __global__ void __launch_bounds__(" + std::to_string(TPR * GROUPS) + ") tcb_rowwise(const tcb::Args a) {\n"
      "  tcb::grid_dependency_sync();\n"
      "  __shared__ float red[" + std::to_string(GROUPS * nw) + "];\n"
      "  float* __restrict__ out = reinterpret_cast<float*>(a.out);\n"
      "  const int g = threadIdx.x / " + TPRs + ";\n"
      "  const int t = threadIdx.x % " + TPRs + ";\n"
      "  for (u64 row0 = (u64)blockIdx.x * " + Gs + "; row0 < " + Rs + "ull; row0 += (u64)gridDim.x * " + Gs + ") {\n"
      "    const u64 r = row0 + g;\n"
      "    const bool active = r < " + Rs + "ull;\n"
      "    " + lines_at(loads.order_row, 4) + "\n"
      "    " + cache_decl + "\n"
      "    " + cache_load + "\n"
      "      " + lines_at(nonempty, 6) + "\n"
      "  }\n"
      "}\n";
  *geo_out = geo;
  *R_out = R;
  *C_out = C;
  return src;
}

static Launch rowwise_launch(const Graph& body, int out_id, int node_id, const std::string& pattern,
                             const std::vector<int>& inputs, const std::string& sabotage) {
  Geo geo;
  i64 R, C;
  Launch l;
  l.code = rowwise_source(body, out_id, pattern, sabotage, &geo, &R, &C);
  i64 ctas = std::max<i64>(1, std::min<i64>(cdiv(R, geo.groups), (i64)SM_COUNT * std::max<i64>(1, 2048 / geo.block) * 4));
  l.calls.push_back(make_call("tcb_rowwise", {ctas, 1, 1}, {geo.block, 1, 1}));
  l.node = node_id;
  l.op = "fused";
  l.kind = "fused-rowwise";
  l.pattern = pattern;
  l.has_pattern = true;
  l.inputs = inputs;
  l.info = {{"R", num(R)}, {"C", num(C)}, {"vec", num(geo.vec)}, {"tpr", num(geo.tpr)}, {"groups", num(geo.groups)},
            {"slots", num(geo.slots)}, {"items", num(geo.items)}, {"cache", boolean(geo.cache)}, {"block", num(geo.block)}};
  return l;
}

// ---------------------------------------------------------------- plain reduce
struct ReduceGeo {
  i64 outer, n, inner, split;
};

static std::string reduce_source(const std::string& op, const std::vector<i64>& in_shape, int axis, ReduceGeo* g) {
  i64 outer = size_of(std::vector<i64>(in_shape.begin(), in_shape.begin() + axis));
  i64 n = in_shape[axis];
  i64 inner = size_of(std::vector<i64>(in_shape.begin() + axis + 1, in_shape.end()));
  i64 outs = outer * inner;
  i64 split = 1;
  if (inner > 1 && outs < 2 * SM_COUNT * 256 && n >= 64)
    split = std::max<i64>(1, std::min({cdiv(n, 32), cdiv((i64)SM_COUNT * 2048, std::max<i64>(1, outs)), (i64)65535}));
  std::string shape = "[";
  for (size_t k = 0; k < in_shape.size(); ++k) shape += (k ? ", " : "") + std::to_string(in_shape[k]);
  shape += "]";
  *g = {outer, n, inner, split};
  return "// " + op + " over axis " + std::to_string(axis) + " of " + shape + ": outer " + std::to_string(outer) + ", n " +
         std::to_string(n) + ", inner " + std::to_string(inner) + ", split " + std::to_string(split) + "\n"
         "#include \"tcb/common.cuh\"\n"
         "#define TCB_OUTER " + std::to_string(outer) + "\n"
         "#define TCB_N " + std::to_string(n) + "\n"
         "#define TCB_INNER " + std::to_string(inner) + "\n"
         "#define TCB_SPLIT " + std::to_string(split) + "\n"
         "#define TCB_IS_MAX " + std::string(op == "max" ? "1" : "0") + "\n"
         "#include \"tcb/reduce.cuh\"\n";
}

static Launch reduce_launch(const std::string& op, const std::vector<i64>& in_shape, int axis) {
  ReduceGeo g;
  Launch l;
  l.code = reduce_source(op, in_shape, axis, &g);
  i64 outs = g.outer * g.inner;
  if (g.inner == 1) {
    l.calls.push_back(make_call("tcb_reduce_rows", {std::max<i64>(1, std::min<i64>(cdiv(g.outer * 32, 256), SM_COUNT * 8)), 1, 1},
                                {256, 1, 1}));
  } else {
    i64 gx = std::max<i64>(1, std::min<i64>(cdiv(outs, 256), SM_COUNT * 8));
    l.calls.push_back(make_call("tcb_reduce_cols", {gx, g.split, 1}, {256, 1, 1}));
    if (g.split > 1) {
      l.calls.push_back(make_call("tcb_reduce_finish", {std::max<i64>(1, std::min<i64>(cdiv(outs, 32), SM_COUNT * 8)), 1, 1},
                                  {256, 1, 1}));
      l.scratch_bytes = g.split * outs * 4;
    }
  }
  l.node = -1;
  l.op = op;
  l.kind = op;
  l.info = {{"outer", num(g.outer)}, {"n", num(g.n)}, {"inner", num(g.inner)}, {"split", num(g.split)}};
  return l;
}

// ---------------------------------------------------------------- matmul epilogue
static i64 kpad(i64 K) { return (K + KPAD - 1) / KPAD * KPAD; }
static i64 gemm_stage_bytes(i64 bn, i64 bk) { return 2 * GEMM_BM * bk * 4 + 2 * bn * bk * 4; }
static i64 gemm_stages(i64 bn, i64 bk) {
  return std::max<i64>(2, std::min<i64>(6, (SMEM_LIMIT - 2048 - GEMM_STAGING) / gemm_stage_bytes(bn, bk)));
}
static i64 gemm_smem(i64 bn, i64 bk) { return gemm_stages(bn, bk) * gemm_stage_bytes(bn, bk) + 1024 + GEMM_STAGING + 1024; }
static bool tma_store_ok(i64 N) { return N % 4 == 0; }
static i64 gemm_bk(i64 bn) { return bn == 256 ? 16 : 32; }
static i64 gemm_bn(i64 N) { return N >= 256 ? 256 : N <= 64 ? 64 : 128; }
static i64 split_bytes(i64 batch, i64 M, i64 K, i64 N, std::pair<bool, bool> fs) {
  i64 Kp = kpad(K);
  return (fs.first ? 0 : 2 * batch * M * Kp * 4) + (fs.second ? 0 : 2 * batch * N * Kp * 4);
}
static std::pair<i64, i64> splitk_plan(i64 batch, i64 M, i64 K, i64 N, i64 bn, std::pair<bool, bool> fs) {
  i64 tiles = batch * cdiv(M, GEMM_BM) * cdiv(N, bn);
  i64 kb = kpad(K) / 32;
  i64 s = 1;
  if (tiles < SM_COUNT && SM_COUNT / tiles > 8 && kb >= 8) {
    s = std::max<i64>(1, std::min<i64>((i64)SM_COUNT / tiles, kb / 4));
    s = cdiv(kb, cdiv(kb, s));
  }
  return {s, split_bytes(batch, M, K, N, fs) + 256};
}
static i64 ctrl_bytes(i64 rem) { return (16 + 16 * rem + 63) / 64 * 64; }

struct TailPlan {
  i64 grid, tail, rem, tail_off, scratch_end;
};

static TailPlan tail_plan(i64 batch, i64 M, i64 K, i64 N, i64 bn, i64 bk, i64 splitk, std::pair<bool, bool> fs) {
  i64 tiles = batch * cdiv(M, GEMM_BM) * cdiv(N, bn) * splitk;
  i64 kbs = kpad(K) / bk;
  i64 grid, rem, tail;
  if (splitk == 1 && tiles < SM_COUNT) {
    tail = std::min<i64>({(i64)SM_COUNT / tiles, kbs / 4, (i64)8});
    if (tail < 2) return {tiles, 1, 0, 0, 0};
    grid = tiles * tail;
    rem = tiles;
  } else {
    grid = std::min<i64>(SM_COUNT, tiles);
    rem = tiles % grid;
    tail = 1;
    if (splitk == 1 && rem && 2 * rem <= grid && kbs >= TAIL_MIN_KB) tail = std::min<i64>({grid / rem, kbs / 4, (i64)8});
    if (tail < 2) return {grid, 1, 0, 0, 0};
  }
  i64 tail_off = split_bytes(batch, M, K, N, fs) + std::max<i64>(256, (ctrl_bytes(rem) + 255) / 256 * 256);
  return {grid, tail, rem, tail_off, tail_off + rem * tail * GEMM_BM * bn * 4};
}

static std::pair<bool, bool> fused_split_plan(i64 batch, i64 M, i64 K, i64 N, i64 bn, bool a_t, bool b_t) {
  (void)batch;
  bool ea = a_t ? M % 4 == 0 : K % 4 == 0;
  bool eb = b_t ? K % 4 == 0 : N % 4 == 0;
  return {ea && cdiv(N, bn) <= FS_MAX_REREAD, eb && cdiv(M, GEMM_BM) <= FS_MAX_REREAD};
}

struct Mnk {
  i64 batch, M, K, N;
};

static std::string epilogue_source(const Graph& body, int out_id, const std::string& sabotage, bool tc, i64 bn, bool a_t,
                                   bool b_t, Mnk* mnk, bool cross_ba = false) {
  const Node* root = nullptr;
  for (auto& n : body.nodes)
    if (n.op == "matmul") {
      root = &n;
      break;
    }
  if (!root) throw Error("epilogue body without a matmul");
  int ia = std::stoi(body.nodes[root->inputs[0]].name.substr(1));
  int ib = std::stoi(body.nodes[root->inputs[1]].name.substr(1));
  const auto& a_s = body.nodes[root->inputs[0]].shape;
  const auto& b_s = body.nodes[root->inputs[1]].shape;
  i64 batch = size_of(std::vector<i64>(a_s.begin(), a_s.end() - 2));
  i64 M = a_s[a_s.size() - 2], K = a_s.back(), N = b_s.back();
  const Node* bias_add = nullptr;
  if (sabotage == "epilogue-before-bias") {
    for (auto& n : body.nodes) {
      bool uses = std::find(n.inputs.begin(), n.inputs.end(), root->id) != n.inputs.end();
      bool all_root = std::all_of(n.inputs.begin(), n.inputs.end(), [&](int i) { return i == root->id; });
      if (n.op == "add" && uses && !all_root) {
        if (n.id != out_id) bias_add = &n;
        break;
      }
    }
  }
  Emitter em(body);
  std::map<std::pair<std::string, int>, std::string> seen;
  em.leaf = [&](int k, Ctx* ctx) {
    auto key = std::make_pair(ctx->key, k);
    auto it = seen.find(key);
    if (it != seen.end()) return it->second;
    std::string name = "x" + std::to_string(seen.size());
    seen[key] = name;
    em.lines.push_back("const float " + name + " = tcb::ld1(reinterpret_cast<const float*>(a.in[" + std::to_string(k) +
                       "]) + " + chain_index(ctx, "i", "u64") + ");");
    return name;
  };
  em.special = [&](int nid, Ctx* ctx) -> std::optional<std::string> {
    if (ctx->key == "i" && (nid == root->id || (bias_add && nid == bias_add->id))) return std::string("acc");
    return std::nullopt;
  };
  Ctx base{"i", nullptr, Gather()};
  std::string out = em.value(out_id, &base);
  if (bias_add) {
    int other = -1;
    for (int i : bias_add->inputs)
      if (i != root->id) {
        other = i;
        break;
      }
    out = "tcb::op_add(" + out + ", " + em.value(other, &base) + ")";
  }
  std::string code = join(em.lines, "\n    ");
  std::string tc_defs;
  if (tc) {
    auto fs = fused_split_plan(batch, M, K, N, bn, a_t, b_t);
    auto [splitk, part_off] = splitk_plan(batch, M, K, N, bn, fs);
    i64 bk = gemm_bk(bn);
    TailPlan tp = tail_plan(batch, M, K, N, bn, bk, splitk, fs);
    tc_defs = "#define TCB_KP " + std::to_string(kpad(K)) + "\n#define TCB_BN " + std::to_string(bn) +
              "\n#define TCB_BK " + std::to_string(bk) + "\n" + "#define TCB_FS_A " + std::to_string((int)fs.first) +
              "\n#define TCB_FS_B " + std::to_string((int)fs.second) + "\n" + "#define TCB_TMA_STORE " +
              std::to_string((int)tma_store_ok(N)) + "\n" + "#define TCB_SPLIT_B_OFFSET " +
              std::to_string(fs.first ? 0 : 2 * batch * M * kpad(K) * 4) + "ull\n" + "#define TCB_STAGES " +
              std::to_string(gemm_stages(bn, bk)) + "\n" + "#define TCB_SPLITK " + std::to_string(splitk) +
              "\n#define TCB_PART_OFFSET " + std::to_string(part_off) + "ull\n" + "#define TCB_GRID " +
              std::to_string(tp.grid) + "\n#define TCB_TAIL_SPLIT " + std::to_string(tp.tail) + "\n" +
              "#define TCB_TAIL_OFFSET " + std::to_string(tp.tail_off) + "ull\n" + "#define TCB_A_T " +
              std::to_string((int)a_t) + "\n#define TCB_B_T " + std::to_string((int)b_t) + "\n" +
              (cross_ba ? "#define TCB_CROSS_BA 1\n" : "");
  }
  *mnk = {batch, M, K, N};
  std::string kernel = tc ? "tcgen05" : "simt";
  return "// matmul epilogue (" + kernel + "): batch " + std::to_string(batch) + ", [" + std::to_string(M) + "," +
         std::to_string(K) + "] x [" + std::to_string(K) + "," + std::to_string(N) + "]\n"
         "#include \"tcb/common.cuh\"\n"
         "#define TCB_M " + std::to_string(M) + "\n"
         "#define TCB_N " + std::to_string(N) + "\n"
         "#define TCB_K " + std::to_string(K) + "\n"
         "#define TCB_BATCH " + std::to_string(batch) + "\n"
         "#define TCB_IA " + std::to_string(ia) + "\n"
         "#define TCB_IB " + std::to_string(ib) + "\n" +
         tc_defs + "struct Epi {\n"
         "  __device__ __forceinline__ static float apply(const tcb::Args& a, float acc, u64 i, u64 row, u64 col, u64 b) {\n"
         "    (void)row; (void)col; (void)b;\n"
         "    " + code + "\n"
         "    return " + out + ";\n"
         "  }\n"
         "};\n"
         "#include \"tcb/" + std::string(tc ? "gemm_tc" : "matmul") + ".cuh\"\n";
}

static const Node& matmul_root(const Graph& body) {
  for (auto& n : body.nodes)
    if (n.op == "matmul") return n;
  throw Error("epilogue body without a matmul");
}

static bool uses_tensor_cores(const std::vector<i64>& a_shape, const std::string& matmul) {
  return matmul == "tiled" && a_shape.back() >= TC_MIN_K;
}

static Launch tc_epilogue_launch(const Graph& body, int out_id, int node_id, const std::string& op, const std::string& kind,
                                 const std::string* pattern, const std::vector<int>& inputs, const std::string& sabotage,
                                 bool a_t, bool b_t, bool cross_ba = false) {
  const Node& root = matmul_root(body);
  i64 bn = gemm_bn(body.nodes[root.inputs[1]].shape.back());
  Mnk m;
  Launch l;
  l.code = epilogue_source(body, out_id, sabotage, true, bn, a_t, b_t, &m, cross_ba);
  i64 batch = m.batch, M = m.M, K = m.K, N = m.N;
  if (batch > 65535 || cdiv(M, GEMM_BM) > 65535) throw Error("matmul grid too large");
  i64 Kp = kpad(K);
  auto fs = fused_split_plan(batch, M, K, N, bn, a_t, b_t);
  i64 err_off = split_bytes(batch, M, K, N, fs);
  auto [splitk, part_off] = splitk_plan(batch, M, K, N, bn, fs);
  i64 bk = gemm_bk(bn);
  TailPlan tp = tail_plan(batch, M, K, N, bn, bk, splitk, fs);
  i64 scratch = std::max<i64>(err_off + 256 + (splitk > 1 ? splitk * batch * M * N * 4 : 0), tp.scratch_end);
  Call gemm = make_call("tcb_gemm_tc", {tp.grid, 1, 1}, {(fs.first || fs.second) ? 320 : 192, 1, 1}, gemm_smem(bn, bk));
  gemm.err_offset = err_off;
  i64 a_bytes = fs.first ? 0 : batch * M * Kp * 4;
  i64 b_off = 2 * a_bytes;
  i64 b_bytes = batch * N * Kp * 4;
  int ia = std::stoi(body.nodes[root.inputs[0]].name.substr(1));
  int ib = std::stoi(body.nodes[root.inputs[1]].name.substr(1));
  std::vector<Map> maps;
  if (fs.first) {
    Map ra = a_t ? Map{"in", ia, M, K, batch, M * 4, K * M * 4, 32 | TMA_ATOM32, bk}
                 : Map{"in", ia, K, M, batch, K * 4, M * K * 4, bk, GEMM_BM};
    maps = {ra, ra};
  } else {
    maps = {Map{"scratch", 0, Kp, M, batch, Kp * 4, M * Kp * 4, bk, GEMM_BM},
            Map{"scratch", a_bytes, Kp, M, batch, Kp * 4, M * Kp * 4, bk, GEMM_BM}};
  }
  if (fs.second) {
    Map rb = b_t ? Map{"in", ib, K, N, batch, K * 4, N * K * 4, bk, bn}
                 : Map{"in", ib, N, K, batch, N * 4, K * N * 4, 32 | TMA_ATOM32, bk};
    maps.push_back(rb);
    maps.push_back(rb);
  } else {
    maps.push_back(Map{"scratch", b_off, Kp, N, batch, Kp * 4, N * Kp * 4, bk, bn});
    maps.push_back(Map{"scratch", b_off + b_bytes, Kp, N, batch, Kp * 4, N * Kp * 4, bk, bn});
  }
  if (tma_store_ok(N))
    maps.push_back(splitk == 1 ? Map{"out", 0, N, M, batch, N * 4, M * N * 4, 32, 32}
                               : Map{"scratch", part_off, N, M, splitk * batch, N * 4, M * N * 4, 32, 32});
  gemm.tma = maps;
  gemm.has_tma = true;
  Call first = fs.first ? make_call("tcb_gemm_prep", {1, 1, 1}, {128, 1, 1})
                        : make_call("tcb_split_a", a_t ? std::array<i64, 3>{Kp / 32, cdiv(M, 32), batch}
                                                       : grid1d(batch * M * Kp, 4), {256, 1, 1});
  first.err_offset = err_off;
  l.calls.push_back(first);
  if (!fs.second)
    l.calls.push_back(make_call("tcb_split_b", b_t ? grid1d(batch * N * Kp, 4) : std::array<i64, 3>{Kp / 32, cdiv(N, 32), batch},
                                {256, 1, 1}));
  l.calls.push_back(gemm);
  if (splitk > 1) l.calls.push_back(make_call("tcb_splitk_finish", grid1d(batch * M * N, 1), {256, 1, 1}));
  l.node = node_id;
  l.op = op;
  l.kind = kind;
  if (pattern) {
    l.pattern = *pattern;
    l.has_pattern = true;
  }
  l.inputs = inputs;
  l.scratch_bytes = scratch;
  l.info = {{"mnk", arr({num(batch), num(M), num(K), num(N)})}, {"bn", num(bn)}, {"bk", num(bk)},
            {"stages", num(gemm_stages(bn, bk))}, {"splitk", num(splitk)}, {"tail_split", num(tp.tail)},
            {"ctrl_bytes", num(ctrl_bytes(tp.rem))}, {"fused_split", arr({boolean(fs.first), boolean(fs.second)})},
            {"path", str("tcgen05-3xtf32")}, {"a_t", boolean(a_t)}, {"b_t", boolean(b_t)}, {"ia", num(ia)},
            {"ib", num(ib)}, {"kp", num(Kp)}};
  return l;
}

static Launch epilogue_launch(const Graph& body, int out_id, int node_id, const std::string& op, const std::string& kind,
                              const std::string* pattern, const std::vector<int>& inputs, const std::string& matmul,
                              const std::string& sabotage, bool a_t, bool b_t, bool cross_ba = false) {
  const Node& root = matmul_root(body);
  if (uses_tensor_cores(body.nodes[root.inputs[0]].shape, matmul))
    return tc_epilogue_launch(body, out_id, node_id, op, kind, pattern, inputs, sabotage, a_t, b_t, cross_ba);
  if (a_t || b_t) throw Error("transposed operands are folded only on the tensor-core path");
  Mnk m;
  Launch l;
  l.code = epilogue_source(body, out_id, sabotage, false, 0, false, false, &m);
  if (m.batch > 65535) throw Error("matmul batch above 65535");
  l.calls.push_back(make_call("tcb_matmul", {cdiv(m.N, 128), cdiv(m.M, 128), m.batch}, {256, 1, 1}));
  l.node = node_id;
  l.op = op;
  l.kind = kind;
  if (pattern) {
    l.pattern = *pattern;
    l.has_pattern = true;
  }
  l.inputs = inputs;
  l.info = {{"mnk", arr({num(m.batch), num(m.M), num(m.K), num(m.N)})}};
  return l;
}

// ---------------------------------------------------------------- plain launches
static Launch plain_uncached(const Node& node, const std::vector<std::vector<i64>>& shapes, const std::string& matmul) {
  int out;
  auto body = one_op_body(node, shapes, &out);
  i64 n = size_of(body->nodes[out].shape);
  const std::string& op = node.op;
  if (op == "sum" || op == "max") return reduce_launch(op, shapes[0], node.axis);
  if (op == "matmul") return epilogue_launch(*body, out, -1, "matmul", "matmul-" + matmul, nullptr, {}, matmul, "", false, false);
  if (is_bin(op) || is_un(op))
    return ew_launch(*body, out, n, op == "stopGradient" ? "copy" : op, -1, op, nullptr, {}, "", "plain " + op);
  if (op == "broadcast" || op == "transpose" || op == "reshape")
    return ew_launch(*body, out, n, "gather", -1, op, nullptr, {}, "", "plain " + op + " (gather)");
  throw Error("no lowering for '" + op + "'");
}

static std::string shapes_key(const Node& node, const Graph& g, const std::string& matmul) {
  std::string k = node.op + "|" + matmul + "|";
  for (int i : node.inputs) {
    for (i64 d : g.nodes[i].shape) k += std::to_string(d) + ",";
    k += ";";
  }
  k += "|" + std::to_string(node.axis) + (node.keepDims ? "k" : "") + "|";
  for (int p : node.perm) k += std::to_string(p) + ",";
  k += "|";
  for (i64 d : node.attr_shape) k += std::to_string(d) + ",";
  return k;
}

static Launch plain_launch(Lowering& L, const Node& node, const std::string& matmul) {
  const Graph& g = *L.graph;
  std::string key = shapes_key(node, g, matmul);
  auto it = L.plain_cache.find(key);
  if (it == L.plain_cache.end()) {
    std::vector<std::vector<i64>> shapes;
    for (int i : node.inputs) shapes.push_back(g.nodes[i].shape);
    it = L.plain_cache.emplace(key, plain_uncached(node, shapes, matmul)).first;
  }
  Launch l = it->second;
  l.node = node.id;
  l.op = node.op;
  l.has_pattern = false;
  l.pattern.clear();
  l.inputs = node.inputs;
  return l;
}

static i64 launch_bytes(const Graph& g, const Launch& l) {
  std::set<int> seen;
  i64 b = 0;
  for (int i : l.inputs)
    if (seen.insert(i).second) b += size_of(g.nodes[i].shape) * 4;
  return b + size_of(g.nodes[l.node].shape) * 4;
}

// ---------------------------------------------------------------- transposes folded into GEMM operands
static bool is_last2_swap(const Node& n) {
  const auto& p = n.perm;
  int r = (int)p.size();
  if (r < 2) return false;
  for (int i = 0; i < r - 2; ++i)
    if (p[i] != i) return false;
  return p[r - 2] == r - 1 && p[r - 1] == r - 2;
}

static bool matmul_operands(const Graph& g, const Node& node, std::pair<int, int>* ab) {
  if (node.op == "matmul") {
    *ab = {node.inputs[0], node.inputs[1]};
    return true;
  }
  if (node.op == "fused" && node.kind == "epilogue") {
    const Graph& b = *node.body;
    const Node& root = matmul_root(b);
    int ia = std::stoi(b.nodes[root.inputs[0]].name.substr(1));
    int ib = std::stoi(b.nodes[root.inputs[1]].name.substr(1));
    std::map<int, int> uses;
    for (auto& n : b.nodes)
      for (int i : n.inputs) uses[i]++;
    if (uses[root.inputs[0]] != 1 || uses[root.inputs[1]] != 1 || root.inputs[0] == root.inputs[1]) return false;
    *ab = {node.inputs[ia], node.inputs[ib]};
    return true;
  }
  (void)g;
  return false;
}

static std::set<int> foldable_transposes(const Graph& g, const std::string& matmul, const std::set<int>& keep) {
  std::map<int, std::vector<int>> consumers;
  for (auto& n : g.nodes)
    for (int i : n.inputs) consumers[i].push_back(n.id);
  std::set<int> folds;
  // readers come after what they read: from the end, every reader's verdict is known (a reader that is a
  // folded transposeLast2 is fine: the GEMMs behind it read through the chain)
  for (auto it = g.nodes.rbegin(); it != g.nodes.rend(); ++it) {
    const Node& t = *it;
    if (t.op != "transpose" || keep.count(t.id) || !is_last2_swap(t) || !consumers.count(t.id)) continue;
    bool ok = true;
    for (int c : consumers[t.id]) {
      if (folds.count(c)) continue;
      std::pair<int, int> ab;
      if (!matmul_operands(g, g.nodes[c], &ab) || (ab.first != t.id && ab.second != t.id) ||
          !uses_tensor_cores(g.nodes[ab.first].shape, matmul)) {
        ok = false;
        break;
      }
    }
    if (ok) folds.insert(t.id);
  }
  return folds;
}

static std::string sab_or_empty(const std::string& s) {
  static const char* k[] = {"epilogue-before-bias", "layernorm-tree-short", "softmax-no-max", "fused-bounds-off-by-one"};
  for (auto* x : k)
    if (s == x) return s;
  return "";
}

static Launch folded_launch(Lowering& L, const Node& node, const std::string& matmul, const std::string& sabotage,
                            const std::set<int>& folds) {
  const Graph& g = *L.graph;
  std::pair<int, int> ab;
  matmul_operands(g, node, &ab);
  // a slot read through a chain of folded transposes: its source, transposed when the chain is odd
  auto unfold = [&](int i, bool* t) {
    *t = false;
    while (folds.count(i)) { i = g.nodes[i].inputs[0]; *t = !*t; }
    return i;
  };
  bool a_t = false, b_t = false;
  unfold(ab.first, &a_t);
  unfold(ab.second, &b_t);
  Launch l;
  if (node.op == "matmul") {
    std::vector<std::vector<i64>> shapes;
    for (int i : node.inputs) shapes.push_back(g.nodes[i].shape);
    int out;
    auto body = one_op_body(node, shapes, &out);
    l = epilogue_launch(*body, out, node.id, "matmul", "matmul-" + matmul, nullptr, node.inputs, matmul, "", a_t, b_t);
  } else {
    l = epilogue_launch(*node.body, node.output, node.id, "fused", "fused-epilogue", &node.pattern, node.inputs, matmul,
                        sab_or_empty(sabotage), a_t, b_t);
  }
  l.inputs.clear();
  bool t;
  for (int i : node.inputs) l.inputs.push_back(unfold(i, &t));
  return l;
}

// A plain tensor-core matmul read only by a transposeLast2 (that does not itself fold into a GEMM):
// the pair becomes one GEMM computing the transposed product, (A.B)^T = B^T.A^T.
static std::map<int, int> transposed_products(const Graph& g, const std::string& matmul, const std::set<int>& keep,
                                              const std::set<int>& folds) {
  std::map<int, std::vector<int>> consumers;
  for (auto& n : g.nodes)
    for (int i : n.inputs) consumers[i].push_back(n.id);
  std::map<int, int> out;
  for (auto& T : g.nodes) {
    if (T.op != "transpose" || !is_last2_swap(T) || folds.count(T.id)) continue;
    const Node& M = g.nodes[T.inputs[0]];
    if (M.op != "matmul" || keep.count(M.id) || consumers[M.id] != std::vector<int>{T.id} ||
        !uses_tensor_cores(g.nodes[M.inputs[0]].shape, matmul))
      continue;
    out[T.id] = M.id;
  }
  return out;
}

static Launch transposed_product_launch(Lowering& L, const Node& T, const Node& M, const std::string& matmul,
                                        const std::set<int>& folds) {
  const Graph& g = *L.graph;
  auto unfold = [&](int i, bool* t) {
    *t = false;
    while (folds.count(i)) { i = g.nodes[i].inputs[0]; *t = !*t; }
    return i;
  };
  bool a_t = false, b_t = false;
  int a_src = unfold(M.inputs[0], &a_t), b_src = unfold(M.inputs[1], &b_t);
  std::vector<i64> sa = g.nodes[M.inputs[0]].shape, sb = g.nodes[M.inputs[1]].shape;
  std::swap(sa[sa.size() - 1], sa[sa.size() - 2]);
  std::swap(sb[sb.size() - 1], sb[sb.size() - 2]);
  int out;
  auto body = one_op_body(M, {sb, sa}, &out);
  Launch l = epilogue_launch(*body, out, T.id, "matmul", "matmul-" + matmul, nullptr, {b_src, a_src}, matmul, "", !b_t,
                             !a_t, true);
  l.inputs = {b_src, a_src};
  l.bytes = launch_bytes(g, l);
  return l;
}

// ---------------------------------------------------------------- elementwise + column sum
static bool elementwise_producer(const Node& n) {
  if (n.op == "fused") return n.kind == "elementwise";
  return is_bin(n.op) || is_un(n.op);
}

static std::map<int, std::pair<int, bool>> colsum_fusions(const Graph& g, const std::set<int>& keep) {
  std::map<int, std::vector<int>> consumers;
  for (auto& n : g.nodes)
    for (int i : n.inputs) consumers[i].push_back(n.id);
  std::map<int, std::pair<int, bool>> out;
  std::set<int> taken;
  for (auto& S : g.nodes) {
    if (S.op != "sum" || S.axis != 0) continue;
    const Node& P = g.nodes[S.inputs[0]];
    if (taken.count(P.id) || P.shape.size() < 2 ||
        size_of(std::vector<i64>(P.shape.begin() + 1, P.shape.end())) <= 1 || !elementwise_producer(P))
      continue;
    out[S.id] = {P.id, keep.count(P.id) > 0 || consumers[P.id].size() > 1};
    taken.insert(P.id);
  }
  return out;
}

static Launch colsum_launch(const Graph& g, const Node& P, const Node& S, bool write) {
  std::shared_ptr<Graph> owned;
  const Graph* body;
  int out_id;
  if (P.op == "fused") {
    body = P.body.get();
    out_id = P.output;
  } else {
    std::vector<std::vector<i64>> shapes;
    for (int i : P.inputs) shapes.push_back(g.nodes[i].shape);
    owned = one_op_body(P, shapes, &out_id);
    body = owned.get();
  }
  i64 R = P.shape[0], C = size_of(std::vector<i64>(P.shape.begin() + 1, P.shape.end()));
  ReduceGeo rg;
  reduce_source("sum", P.shape, 0, &rg);
  i64 split = rg.split;
  i64 W = (C % 4 == 0 && (C / 4) * split >= (i64)SM_COUNT * 1024) ? 4 : 1;
  Launch l;
  l.code = "// elementwise (" + P.op + ") + column sum over axis 0 of [" + std::to_string(R) + ", " + std::to_string(C) +
           "], split " + std::to_string(split) + ", value " + (write ? "stored" : "not stored") + "\n"
           "#include \"tcb/common.cuh\"\n"
           "#define TCB_OUTER 1\n"
           "#define TCB_N " + std::to_string(R) + "\n"
           "#define TCB_INNER " + std::to_string(C) + "\n"
           "#define TCB_SPLIT " + std::to_string(split) + "\n"
           "#define TCB_IS_MAX 0\n"
           "#define TCB_W " + std::to_string(W) + "\n"
           "#define TCB_WRITE " + std::to_string((int)write) + "\n" +
           ew_body_struct(*body, out_id, R * C) + "#include \"tcb/colsum.cuh\"\n";
  i64 groups = C / W;
  i64 block = std::min<i64>(256, std::max<i64>(32, cdiv(groups, 32) * 32));
  Call main = make_call("tcb_ew_colsum", {std::max<i64>(1, std::min<i64>(cdiv(groups, block), SM_COUNT * 8)), split, 1},
                        {block, 1, 1});
  if (write && split == 1) main.ptr_params = {{14, S.id}};
  l.calls.push_back(main);
  if (split > 1) {
    Call fin = make_call("tcb_reduce_finish", {std::max<i64>(1, std::min<i64>(cdiv(C, 32), SM_COUNT * 8)), 1, 1}, {256, 1, 1});
    if (write) fin.out_node = S.id;
    l.calls.push_back(fin);
  }
  l.node = write ? P.id : S.id;
  l.op = "fused";
  l.kind = "fused-colsum";
  l.pattern = "elementwise+colsum";
  l.has_pattern = true;
  l.inputs = P.inputs;
  l.scratch_bytes = split > 1 ? split * C * 4 : 0;
  l.info = {{"R", num(R)}, {"C", num(C)}, {"split", num(split)}, {"write", boolean(write)}, {"producer", num(P.id)},
            {"sum", num(S.id)}};
  if (write) l.nodes = {P.id, S.id};
  std::set<int> seen;
  i64 nb = 0;
  for (int i : P.inputs)
    if (seen.insert(i).second) nb += size_of(g.nodes[i].shape) * 4;
  l.bytes = nb + C * 4 + (write ? R * C * 4 : 0);
  return l;
}

// ---------------------------------------------------------------- elementwise + row sum
static const i64 ROWSUM_MIN_ROWS = (i64)SM_COUNT * 8;

static std::map<int, std::pair<int, bool>> rowsum_fusions(const Graph& g, const std::set<int>& keep,
                                                          const std::set<int>& exclude) {
  std::map<int, std::vector<int>> consumers;
  for (auto& n : g.nodes)
    for (int i : n.inputs) consumers[i].push_back(n.id);
  std::map<int, std::pair<int, bool>> out;
  std::set<int> taken;
  for (auto& S : g.nodes) {
    if (S.op != "sum" || exclude.count(S.id)) continue;
    const Node& P = g.nodes[S.inputs[0]];
    if (P.shape.size() < 2 || S.axis != (int)P.shape.size() - 1 || taken.count(P.id) || exclude.count(P.id) ||
        size_of(std::vector<i64>(P.shape.begin(), P.shape.end() - 1)) < ROWSUM_MIN_ROWS || !elementwise_producer(P))
      continue;
    out[S.id] = {P.id, keep.count(P.id) > 0 || consumers[P.id].size() > 1};
    taken.insert(P.id);
  }
  return out;
}

static Launch rowsum_launch(const Graph& g, const Node& P, const Node& S, bool write) {
  std::shared_ptr<Graph> owned;
  const Graph* body;
  int out_id;
  if (P.op == "fused") {
    body = P.body.get();
    out_id = P.output;
  } else {
    std::vector<std::vector<i64>> shapes;
    for (int i : P.inputs) shapes.push_back(g.nodes[i].shape);
    owned = one_op_body(P, shapes, &out_id);
    body = owned.get();
  }
  i64 R = size_of(std::vector<i64>(P.shape.begin(), P.shape.end() - 1)), C = P.shape.back();
  Launch l;
  l.code = "// elementwise (" + P.op + ") + sum over the last axis of [" + std::to_string(R) + ", " + std::to_string(C) +
           "], value " + (write ? "stored" : "not stored") + "\n"
           "#include \"tcb/common.cuh\"\n"
           "#define TCB_OUTER " + std::to_string(R) + "\n"
           "#define TCB_N " + std::to_string(C) + "\n"
           "#define TCB_INNER 1\n"
           "#define TCB_SPLIT 1\n"
           "#define TCB_IS_MAX 0\n"
           "#define TCB_WRITE " + std::to_string((int)write) + "\n" +
           ew_body_struct(*body, out_id, R * C) + "#include \"tcb/rowsum.cuh\"\n";
  Call main = make_call("tcb_ew_rowsum", {std::max<i64>(1, std::min<i64>(cdiv(R * 32, 256), SM_COUNT * 8)), 1, 1},
                        {256, 1, 1});
  if (write) main.ptr_params = {{14, S.id}};
  l.calls.push_back(main);
  l.node = write ? P.id : S.id;
  l.op = "fused";
  l.kind = "fused-rowsum";
  l.pattern = "elementwise+rowsum";
  l.has_pattern = true;
  l.inputs = P.inputs;
  l.scratch_bytes = 0;
  l.info = {{"R", num(R)}, {"C", num(C)}, {"write", boolean(write)}, {"producer", num(P.id)}, {"sum", num(S.id)}};
  if (write) l.nodes = {P.id, S.id};
  std::set<int> seen;
  i64 nb = 0;
  for (int i : P.inputs)
    if (seen.insert(i).second) nb += size_of(g.nodes[i].shape) * 4;
  l.bytes = nb + R * 4 + (write ? R * C * 4 : 0);
  return l;
}

// ---------------------------------------------------------------- one pass, several elementwise outputs
static bool reads_directly(const Node& node, int k) {
  if (node.op != "fused") return true;
  const Graph& b = *node.body;
  int nid = -1;
  for (auto& n : b.nodes)
    if (n.op == "input" && n.name == "a" + std::to_string(k)) {
      nid = n.id;
      break;
    }
  for (auto& n : b.nodes)
    if (std::find(n.inputs.begin(), n.inputs.end(), nid) != n.inputs.end() && !is_bin(n.op) && !is_un(n.op)) return false;
  return true;
}

static std::vector<int> mo_operands(const Node& P, const Node& Q) {
  std::vector<int> ops;
  auto add = [&](int i) {
    if (std::find(ops.begin(), ops.end(), i) == ops.end()) ops.push_back(i);
  };
  for (int i : P.inputs) add(i);
  for (int i : Q.inputs)
    if (i != P.id) add(i);
  return ops;
}

static std::map<int, int> mo_fusions(const Graph& g, const std::set<int>& keep, const std::set<int>& exclude) {
  std::set<int> live;
  bool use_live = !keep.empty();
  if (use_live) {
    live = keep;
    for (int i = (int)g.nodes.size() - 1; i >= 0; --i)
      if (live.count(i))
        for (int j : g.nodes[i].inputs) live.insert(j);
  }
  std::map<int, std::vector<int>> consumers;
  for (auto& n : g.nodes)
    for (int i : n.inputs) consumers[i].push_back(n.id);
  std::set<int> used = exclude;
  std::map<int, int> out;
  for (auto& P : g.nodes) {
    if (used.count(P.id) || !elementwise_producer(P)) continue;
    for (int qid : consumers[P.id]) {
      const Node& Q = g.nodes[qid];
      if (used.count(qid) || !elementwise_producer(Q) || Q.shape != P.shape || (use_live && !live.count(qid))) continue;
      bool ready = true;
      for (int i : Q.inputs)
        if (i != P.id && !(g.nodes[i].op == "input" || g.nodes[i].op == "const" || i < P.id)) ready = false;
      if (!ready) continue;
      bool direct = true;
      for (size_t k = 0; k < Q.inputs.size(); ++k)
        if (Q.inputs[k] == P.id && !reads_directly(Q, (int)k)) direct = false;
      if (!direct) continue;
      if (mo_operands(P, Q).size() > 8) continue;
      out[P.id] = qid;
      used.insert(P.id);
      used.insert(qid);
      break;
    }
  }
  return out;
}

static Launch mo_launch(const Graph& g, const Node& P, const Node& Q) {
  std::vector<int> operands = mo_operands(P, Q);
  Graph body;
  std::map<int, int> slot;
  for (size_t k = 0; k < operands.size(); ++k) {
    Node in;
    in.id = (int)k;
    in.op = "input";
    in.name = "a" + std::to_string(k);
    in.shape = g.nodes[operands[k]].shape;
    in.attr_shape = in.shape;
    body.nodes.push_back(in);
    slot[operands[k]] = (int)k;
  }
  std::vector<int> outs;
  const Node* parts[2] = {&P, &Q};
  for (int w = 0; w < 2; ++w) {
    const Node& node = *parts[w];
    std::shared_ptr<Graph> owned;
    const Graph* b;
    int out_id;
    if (node.op == "fused") {
      b = node.body.get();
      out_id = node.output;
    } else {
      std::vector<std::vector<i64>> shapes;
      for (int i : node.inputs) shapes.push_back(g.nodes[i].shape);
      owned = one_op_body(node, shapes, &out_id);
      b = owned.get();
    }
    std::map<int, int> remap;
    for (auto& n : b->nodes) {
      if (n.op == "input") {
        int src = node.inputs[std::stoi(n.name.substr(1))];
        remap[n.id] = (w == 1 && src == P.id) ? outs[0] : slot[src];
      } else {
        Node c = n;
        c.id = (int)body.nodes.size();
        for (auto& i : c.inputs) i = remap[i];
        c.body.reset();
        body.nodes.push_back(c);
        remap[n.id] = c.id;
      }
    }
    outs.push_back(remap[out_id]);
  }
  i64 n = size_of(P.shape);
  // the source: the elementwise load plan and emitter over the merged body, one store per output
  EwLoads loads;
  loads.T = idx_type(n);
  Emitter em(body);
  em.leaf = [&](int k, Ctx* c) { return loads.leaf(k, c); };
  Ctx base{"i", nullptr, Gather()};
  std::vector<std::string> vals;
  for (int o : outs) vals.push_back(em.value(o, &base));
  std::string fields = loads.fields.empty() ? "float unused_;" : join(loads.fields, "\n    ");
  std::string per_lane = loads.per_lane.empty()
                             ? ""
                             : "#pragma unroll\n    for (int l = 0; l < W; ++l) {\n      " +
                                   join(loads.per_lane, "\n      ") + "\n    }";
  std::vector<std::string> stores;
  for (size_t k = 0; k < vals.size(); ++k) stores.push_back("o[" + std::to_string(k) + "][l] = " + vals[k] + ";");
  Launch l;
  l.code = "// elementwise, " + std::to_string(outs.size()) + " outputs: generated from a body of " +
           std::to_string(body.nodes.size()) + " nodes, " + std::to_string(n) + " elements\n"
           "#include \"tcb/common.cuh\"\n#define TCB_W 4\n#define TCB_NOUT " + std::to_string(outs.size()) + "\n"
           "struct Body {\n"
           "  template <int W> struct Regs {\n"
           "    " + fields + "\n"
           "  };\n"
           "  template <int W> __device__ __forceinline__ static void load(const tcb::Args& a, u64 i0, Regs<W>& r) {\n"
           "    " + join(loads.stmts, "\n    ") + "\n"
           "    " + per_lane + "\n"
           "  }\n"
           "  template <int W> __device__ __forceinline__ static void compute(const Regs<W>& r, float (&o)[TCB_NOUT][W]) {\n"
           "#pragma unroll\n"
           "    for (int l = 0; l < W; ++l) {\n"
           "      " + join(em.lines, "\n      ") + "\n"
           "      " + join(stores, "\n      ") + "\n"
           "    }\n"
           "  }\n"
           "};\n"
           "#include \"tcb/elementwise_mo.cuh\"\n";
  Call call = make_call("tcb_elementwise_mo", grid1d(n), {WG, 1, 1}, 0, {n});
  call.ptr_params = {{1, Q.id}};
  l.calls.push_back(call);
  l.node = P.id;
  l.nodes = {P.id, Q.id};
  l.op = "fused";
  l.kind = "fused-multi";
  l.pattern = "elementwise+reader";
  l.has_pattern = true;
  l.inputs = operands;
  l.info = {{"producer", num(P.id)}, {"reader", num(Q.id)}, {"outputs", num(2)}};
  i64 nb = 0;
  for (int i : operands) nb += size_of(g.nodes[i].shape) * 4;
  l.bytes = nb + 2 * n * 4;
  return l;
}

// ---------------------------------------------------------------- lower / lowerFused / fusedKernel
static Launch fused_kernel(const Node& node, const std::string& matmul, const std::string& sabotage) {
  const Graph& body = *node.body;
  std::string sab = sab_or_empty(sabotage);
  if (node.kind == "elementwise")
    return ew_launch(body, node.output, size_of(node.shape), "fused-elementwise", node.id, "fused", &node.pattern,
                     node.inputs, sab, "fused elementwise (" + std::to_string(node.inputs.size()) + " operands)");
  if (node.kind == "epilogue")
    return epilogue_launch(body, node.output, node.id, "fused", "fused-epilogue", &node.pattern, node.inputs, matmul, sab,
                           false, false);
  if (node.kind == "rowwise") return rowwise_launch(body, node.output, node.id, node.pattern, node.inputs, sab);
  throw Error("no fused kernel kind '" + node.kind + "'");
}

struct Options {
  bool fused = true;
  std::string matmul = "naive", sabotage;
  bool fold = false, colfuse = false, mofuse = false;
  std::set<int> keep;
};

static void lower_graph(Lowering& L, const Options& o) {
  const Graph& g = *L.graph;
  std::set<int> folds = o.fold ? foldable_transposes(g, o.matmul, o.keep) : std::set<int>();
  std::map<int, int> tprods = o.fold ? transposed_products(g, o.matmul, o.keep, folds) : std::map<int, int>();
  std::set<int> tmats;
  for (auto& kv : tprods) tmats.insert(kv.second);
  std::map<int, std::pair<int, bool>> cols = (o.fused && o.colfuse) ? colsum_fusions(g, o.keep)
                                                                     : std::map<int, std::pair<int, bool>>();
  std::map<int, std::pair<int, bool>> rows;
  if (o.fused && o.colfuse) {
    std::set<int> taken;
    for (auto& [sid, pw] : cols) { taken.insert(sid); taken.insert(pw.first); }
    rows = rowsum_fusions(g, o.keep, taken);
  }
  // sum id -> (producer id, write, row sum?)
  std::map<int, std::tuple<int, bool, bool>> sums;
  for (auto& [sid, pw] : cols) sums[sid] = {pw.first, pw.second, false};
  for (auto& [sid, pw] : rows) sums[sid] = {pw.first, pw.second, true};
  std::map<int, std::tuple<int, bool, bool>> producer_of;
  for (auto& [sid, t] : sums) producer_of[std::get<0>(t)] = {sid, std::get<1>(t), std::get<2>(t)};
  std::map<int, int> mos;
  if (o.fused && o.mofuse) {
    std::set<int> exclude(folds.begin(), folds.end());
    for (auto& kv : sums) exclude.insert(kv.first);
    for (auto& kv : producer_of) exclude.insert(kv.first);
    for (auto& kv : tprods) { exclude.insert(kv.first); exclude.insert(kv.second); }
    mos = mo_fusions(g, o.keep, exclude);
  }
  std::set<int> readers;
  for (auto& kv : mos) readers.insert(kv.second);
  for (auto& node : g.nodes) {
    if (node.op == "input" || node.op == "const" || folds.count(node.id) || readers.count(node.id) ||
        tmats.count(node.id))
      continue;
    if (tprods.count(node.id)) {  // a GEMM read only by a transpose: the transposed product
      L.launches.push_back(transposed_product_launch(L, node, g.nodes[tprods[node.id]], o.matmul, folds));
      continue;
    }
    if (mos.count(node.id)) {
      L.launches.push_back(mo_launch(g, node, g.nodes[mos[node.id]]));
      continue;
    }
    if (producer_of.count(node.id)) {
      auto [sid, write, row] = producer_of[node.id];
      if (write) L.launches.push_back(row ? rowsum_launch(g, node, g.nodes[sid], true) : colsum_launch(g, node, g.nodes[sid], true));
      continue;
    }
    if (sums.count(node.id)) {
      auto [pid, write, row] = sums[node.id];
      if (!write) L.launches.push_back(row ? rowsum_launch(g, g.nodes[pid], node, false) : colsum_launch(g, g.nodes[pid], node, false));
      continue;
    }
    std::pair<int, int> ab;
    Launch l;
    bool folded = !folds.empty() && matmul_operands(g, node, &ab) && (folds.count(ab.first) || folds.count(ab.second));
    if (folded) l = folded_launch(L, node, o.matmul, o.sabotage, folds);
    else if (o.fused && node.op == "fused") l = fused_kernel(node, o.matmul, o.sabotage);
    else if (node.op == "fused") throw Error("lower(): fused node " + std::to_string(node.id) + " (use the fused lowering)");
    else l = plain_launch(L, node, o.matmul);
    l.bytes = launch_bytes(g, l);
    L.launches.push_back(std::move(l));
  }
  L.folded.assign(folds.begin(), folds.end());
  L.transposed.assign(tprods.begin(), tprods.end());
}

// ---------------------------------------------------------------- records as JSON
static std::string to_json(const Value& v) {
  switch (v.kind) {
    case Value::Null: return "null";
    case Value::Bool: return v.b ? "true" : "false";
    case Value::Number: {
      char buf[40];
      if (v.integral) snprintf(buf, sizeof buf, "%lld", (long long)v.num);
      else snprintf(buf, sizeof buf, "%.17g", v.num);
      return buf;
    }
    case Value::String: return tcb_json::quote(v.str);
    case Value::Array: {
      std::string s = "[";
      for (size_t k = 0; k < v.arr.size(); ++k) s += (k ? "," : "") + to_json(v.arr[k]);
      return s + "]";
    }
    case Value::Object: {
      std::string s = "{";
      for (size_t k = 0; k < v.obj.size(); ++k) s += (k ? "," : "") + tcb_json::quote(v.obj[k].first) + ":" + to_json(v.obj[k].second);
      return s + "}";
    }
  }
  return "null";
}

static std::string ints_json(const std::vector<int>& xs) {
  std::string s = "[";
  for (size_t k = 0; k < xs.size(); ++k) s += (k ? "," : "") + std::to_string(xs[k]);
  return s + "]";
}

static std::string launch_json(const Launch& l) {
  std::string s = "{\"node\":" + std::to_string(l.node);
  if (!l.nodes.empty()) s += ",\"nodes\":" + ints_json(l.nodes);
  s += ",\"op\":" + tcb_json::quote(l.op) + ",\"kind\":" + tcb_json::quote(l.kind) +
       ",\"pattern\":" + (l.has_pattern ? tcb_json::quote(l.pattern) : std::string("null")) +
       ",\"inputs\":" + ints_json(l.inputs) + ",\"code\":" + tcb_json::quote(l.code) +
       ",\"scratch_bytes\":" + std::to_string(l.scratch_bytes) + ",\"bytes\":" + std::to_string(l.bytes) + ",\"calls\":[";
  for (size_t k = 0; k < l.calls.size(); ++k) {
    const Call& c = l.calls[k];
    s += std::string(k ? "," : "") + "{\"name\":" + tcb_json::quote(c.name) + ",\"grid\":[" + std::to_string(c.grid[0]) + "," +
         std::to_string(c.grid[1]) + "," + std::to_string(c.grid[2]) + "],\"block\":[" + std::to_string(c.block[0]) + "," +
         std::to_string(c.block[1]) + "," + std::to_string(c.block[2]) + "],\"smem\":" + std::to_string(c.smem) + ",\"params\":[";
    for (size_t j = 0; j < c.params.size(); ++j) s += (j ? "," : "") + std::to_string(c.params[j]);
    s += "],\"err_offset\":" + (c.err_offset >= 0 ? std::to_string(c.err_offset) : std::string("null")) +
         ",\"out_node\":" + (c.out_node >= 0 ? std::to_string(c.out_node) : std::string("null")) + ",\"ptr_params\":[";
    for (size_t j = 0; j < c.ptr_params.size(); ++j)
      s += std::string(j ? "," : "") + "[" + std::to_string(c.ptr_params[j].first) + "," + std::to_string(c.ptr_params[j].second) + "]";
    s += "],\"tma\":";
    if (!c.has_tma) {
      s += "null";
    } else {
      s += "[";
      for (size_t j = 0; j < c.tma.size(); ++j) {
        const Map& m = c.tma[j];
        s += std::string(j ? "," : "") + "[" + tcb_json::quote(m.region) + "," + std::to_string(m.off) + "," +
             std::to_string(m.cols) + "," + std::to_string(m.rows) + "," + std::to_string(m.batches) + "," +
             std::to_string(m.rs) + "," + std::to_string(m.bs) + "," + std::to_string(m.bc) + "," + std::to_string(m.br) + "]";
      }
      s += "]";
    }
    s += "}";
  }
  s += "],\"info\":{";
  for (size_t k = 0; k < l.info.size(); ++k) s += (k ? "," : "") + tcb_json::quote(l.info[k].first) + ":" + to_json(l.info[k].second);
  return s + "}}";
}

}  // namespace tcl


extern "C" {

int tc_lower_json(const char* graph_json, const char* opts_json, tc_lowered** out) {
  if (!graph_json || !out) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_lower_json: null argument");
  *out = nullptr;
  try {
    auto* l = new tc_lowered();
    std::unique_ptr<tc_lowered> guard(l);
    tcb_json::Value g = tcb_json::parse(graph_json);
    l->L.graph = tcl::graph_from_json(g);
    tcl::Options o;
    if (opts_json && *opts_json) {
      tcb_json::Value v = tcb_json::parse(opts_json);
      if (auto* x = v.find("fused")) o.fused = x->truthy();
      if (auto* x = v.find("matmul")) o.matmul = x->as_string();
      if (auto* x = v.find("sabotage"))
        if (x->is_string()) o.sabotage = x->as_string();
      if (auto* x = v.find("fold")) o.fold = x->truthy();
      if (auto* x = v.find("colfuse")) o.colfuse = x->truthy();
      if (auto* x = v.find("mofuse")) o.mofuse = x->truthy();
      if (auto* x = v.find("keep"))
        for (auto& k : x->arr) o.keep.insert((int)k.as_int());
    }
    if (o.matmul != "naive" && o.matmul != "tiled")
      return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_lower_json: matmul must be \"naive\" or \"tiled\"");
    tcl::lower_graph(l->L, o);
    *out = guard.release();
    return TC_OK;
  } catch (const std::exception& e) {
    return tcb_detail::fail_msg(TC_ERR_INVALID, std::string("tc_lower_json: ") + e.what());
  }
}

int tc_lowered_count(tc_lowered* l, int* n) {
  if (!l || !n) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_lowered_count: null argument");
  *n = (int)l->L.launches.size();
  return TC_OK;
}

int tc_lowered_json(tc_lowered* l, char* json, uint64_t cap, uint64_t* needed) {
  if (!l) return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_lowered_json: null lowering");
  if (l->json.empty()) {
    std::string s = "{\"launches\":[";
    for (size_t k = 0; k < l->L.launches.size(); ++k) s += (k ? "," : "") + tcl::launch_json(l->L.launches[k]);
    s += "],\"folded\":" + tcl::ints_json(l->L.folded) + ",\"transposed\":[";
    for (size_t k = 0; k < l->L.transposed.size(); ++k)
      s += (k ? ",[" : "[") + std::to_string(l->L.transposed[k].first) + "," + std::to_string(l->L.transposed[k].second) + "]";
    s += "]}";
    l->json = std::move(s);
  }
  if (needed) *needed = l->json.size() + 1;
  if (json && cap) {
    if (cap < l->json.size() + 1)
      return tcb_detail::fail_msg(TC_ERR_INVALID, "tc_lowered_json: buffer of " + std::to_string(cap) + " bytes, " +
                                                      std::to_string(l->json.size() + 1) + " needed");
    std::memcpy(json, l->json.c_str(), l->json.size() + 1);
  }
  return TC_OK;
}

int tc_lowered_free(tc_lowered* l) {
  delete l;
  return TC_OK;
}

}  // extern "C"
