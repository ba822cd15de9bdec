// Programs (src/FuryKernel/Program/Graph.hs), their builder (Build.hs), the
// Llama-shaped programs of this path, and the deterministic text form
// (Graph.hs:445-528) with its parser.
#include <cinttypes>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <sstream>
#include <tuple>

#include "fkh.h"

namespace fkh {

bool pointwise(const std::string& k) {
  return k == "Add" || k == "GeluMul" || k == "SiluMul" || k == "ScaleBy" || k == "Softcap" || k == "KvStore";
}

// ---------------------------------------------------------------------------
// The builder

std::string Builder::fresh(const std::string& base) {
  std::string n = base;
  for (int i = 1; names_.count(n); ++i) n = base + "_" + std::to_string(i);
  names_.insert(n);
  return n;
}

int Builder::source(const std::string& name, SourceKind k) {
  Source s;
  s.id = (int)p_.sources.size();
  s.name = name;
  s.kind = std::move(k);
  names_.insert(name);
  p_.sources.push_back(s);
  return s.id;
}

std::vector<int> Builder::node(const std::string& name, Op op,
                               const std::vector<std::tuple<std::string, Shape, std::string>>& outs) {
  std::vector<int> ids;
  std::string first;
  for (const auto& [vname, sh, t] : outs) {
    Value v;
    v.id = (int)p_.values.size();
    v.name = fresh(vname);
    v.shape = sh;
    v.type = t;
    if (ids.empty()) first = v.name;
    p_.values.push_back(v);
    ids.push_back(v.id);
  }
  Node n;
  n.id = (int)p_.nodes.size();
  n.name = ids.empty() ? fresh(name) : first;
  n.op = std::move(op);
  n.outputs = ids;
  p_.nodes.push_back(n);
  return ids;
}

int Builder::one(const std::string& name, Op op, Shape sh, const std::string& type) {
  return node(name, std::move(op), {{name, sh, type}})[0];
}

uint64_t Builder::rows_of(int src) const {
  const Source* s = p_.source(src);
  if (s && (s->kind.kind == SrcKind::Weight || s->kind.kind == SrcKind::Table) && !s->kind.dims.empty())
    return s->kind.dims[0];
  return 0;
}

int Builder::input(const std::string& name, Shape sh, const std::string& type) {
  SourceKind k;
  k.kind = SrcKind::Input;
  k.shape = sh;
  k.type = type;
  const int s = source(name, k);
  Value v;
  v.id = (int)p_.values.size();
  v.name = name;
  v.shape = sh;
  v.type = type;
  p_.values.push_back(v);
  Node n;
  n.id = (int)p_.nodes.size();
  n.name = name;
  n.op.kind = "Input";
  n.op.sources = {s};
  n.outputs = {v.id};
  p_.nodes.push_back(n);
  return v.id;
}

int Builder::row_ints(const std::string& name, uint64_t n, uint64_t bound) {
  SourceKind k;
  k.kind = SrcKind::RowInts;
  k.count = n;
  k.bound = bound;
  return source(name, k);
}

int Builder::weight(const std::string& name, std::vector<uint64_t> dims, const std::string& type) {
  SourceKind k;
  k.kind = SrcKind::Weight;
  k.layout = dims.size() == 2 ? "out_in" : "row_major";
  k.dims = std::move(dims);
  k.type = type;
  return source(name, k);
}

int Builder::cache(const std::string& name, Ring layout, const std::string& elem) {
  SourceKind k;
  k.kind = SrcKind::Cache;
  k.ring = true;
  k.r = layout;
  k.elem = elem;
  return source(name, k);
}

int Builder::cache(const std::string& name, Paged layout, const std::string& elem) {
  SourceKind k;
  k.kind = SrcKind::Cache;
  k.ring = false;
  k.pg = layout;
  k.elem = elem;
  return source(name, k);
}

int Builder::linear(const std::string& name, int w, uint64_t seg, int x) {
  const uint64_t n = rows_of(w);
  Op op;
  op.kind = "Linear";
  op.values = {x};
  op.sources = {w};
  op.segment = seg == 0 ? n : seg;
  return one(name, op, Shape{n, op.segment});
}

int Builder::rmsnorm(const std::string& name, double eps, std::optional<int> gamma, double factor, int x) {
  Op op;
  op.kind = "RmsNorm";
  op.values = {x};
  if (gamma) op.sources = {*gamma};
  op.eps = eps;
  op.factor = factor;
  op.gamma = gamma.has_value();
  return one(name, op, p_.values[x].shape);
}

int Builder::add(const std::string& name, int a, int b) {
  Op op;
  op.kind = "Add";
  op.values = {a, b};
  return one(name, op, p_.values[a].shape);
}

int Builder::silu_mul(const std::string& name, int a, int b) {
  Op op;
  op.kind = "SiluMul";
  op.values = {a, b};
  return one(name, op, p_.values[a].shape);
}

int Builder::rope(const std::string& name, RopeSpec r, int pos, int x) {
  Op op;
  op.kind = "Rope";
  op.values = {x};
  op.sources = {pos};
  op.rope = r;
  return one(name, op, p_.values[x].shape);
}

void Builder::kv_store(const std::string& name, int cache, int positions, int sequences, int x) {
  Op op;
  op.kind = "KvStore";
  op.values = {x};
  op.sources = {cache, positions, sequences};
  node(name, op, {});
}

int Builder::attend(const std::string& name, AttnSpec spec, int q, int keys, int vals, int positions,
                    int sequences) {
  Op op;
  op.kind = "Attend";
  op.values = {q};
  op.sources = {keys, vals, positions, sequences};
  if (spec.reach) op.sources.push_back(spec.reach->first);
  op.attn = spec;
  return one(name, op, p_.values[q].shape);
}

int Builder::gather(const std::string& name, int table, int tokens, double factor) {
  const Source* t = p_.source(table);
  const uint64_t width = t && t->kind.kind == SrcKind::Weight && t->kind.dims.size() == 2 ? t->kind.dims[1] : 0;
  Op op;
  op.kind = "Gather";
  op.sources = {table, tokens};
  op.f = factor;
  return one(name, op, whole_row(width));
}

int Builder::argmax(const std::string& name, int x) {
  Op op;
  op.kind = "ArgMax";
  op.values = {x};
  return one(name, op, whole_row(1), "u32");
}

int Builder::table(const std::string& name, uint64_t entries, std::vector<uint64_t> dims, const std::string& type) {
  SourceKind k;
  k.kind = SrcKind::Table;
  k.entries = entries;
  k.dims = std::move(dims);
  k.type = type;
  k.layout = "out_in";
  return source(name, k);
}

int Builder::linear_routed(const std::string& name, int table, int ids, int x) {
  const uint64_t n = rows_of(table);
  const uint64_t ranks = p_.values[ids].shape.width;
  Op op;
  op.kind = "LinearRouted";
  op.values = {ids, x};
  op.sources = {table};
  return one(name, op, Shape{ranks * n, n});
}

std::pair<int, int> Builder::route(const std::string& name, uint64_t k, std::optional<int> scale, int x) {
  Op op;
  op.kind = "Route";
  op.values = {x};
  op.route.k = k;
  op.route.expert_scale = scale;
  if (scale) op.sources = {*scale};
  const auto ids = node(name, op, {{name + "_ids", whole_row(k), "u32"}, {name + "_weights", whole_row(k), "f32"}});
  return {ids[0], ids[1]};
}

int Builder::gated_gelu(const std::string& name, int x) {
  const Shape in = p_.values[x].shape;
  Op op;
  op.kind = "GatedGelu";
  op.values = {x};
  return one(name, op, Shape{in.width / 2, in.segment / 2});
}

int Builder::combine_ranks(const std::string& name, int w, int x) {
  Op op;
  op.kind = "CombineRanks";
  op.values = {w, x};
  return one(name, op, whole_row(p_.values[x].shape.segment));
}

void Builder::output(const std::string& name, int v) { p_.outputs.push_back(Output{name, v}); }

// ---------------------------------------------------------------------------
// The Llama-shaped programs

Program layer_program(const LlamaShape& s, const std::string& name) {
  Builder b(name);
  const int x = b.input("x", whole_row(s.d_model));
  const int pos = b.row_ints("position", 1, s.positions);
  // A row's sequence: its slot of the ring, or its block table of the pool.
  const int slot = s.paged() ? b.row_ints("block_table", s.table_len(), s.blocks) : b.row_ints("slot", 1, s.slots);
  const int attn_norm = b.weight("attn_norm", {s.d_model}, s.weights);
  const int wq = b.weight("q_proj", {s.q_width(), s.d_model}, s.weights);
  const int wk = b.weight("k_proj", {s.kv_width(), s.d_model}, s.weights);
  const int wv = b.weight("v_proj", {s.kv_width(), s.d_model}, s.weights);
  const int wo = b.weight("o_proj", {s.d_model, s.q_width()}, s.weights);
  const int mlp_norm = b.weight("mlp_norm", {s.d_model}, s.weights);
  // The dense FFN's weights, or the router and the experts' tables.
  int wg = -1, wu = -1, wd = -1, router = -1, egu = -1, edn = -1;
  std::optional<int> expert_scale;
  if (s.experts) {
    router = b.weight("router", {s.experts, s.d_model}, s.weights);
    if (s.expert_scale) expert_scale = b.weight("expert_scale", {s.experts}, s.weights);
    egu = b.table("experts_gate_up", s.experts, {2 * s.ffn, s.d_model}, s.weights);
    edn = b.table("experts_down", s.experts, {s.d_model, s.ffn}, s.weights);
  } else {
    wg = b.weight("gate_proj", {s.ffn, s.d_model}, s.weights);
    wu = b.weight("up_proj", {s.ffn, s.d_model}, s.weights);
    wd = b.weight("down_proj", {s.d_model, s.ffn}, s.weights);
  }
  const Ring ring{s.slots, s.kv_heads, s.length, s.head_dim};
  const Paged pool{s.blocks, s.block_size, s.kv_heads, s.head_dim};
  const int kc = s.paged() ? b.cache("k_cache", pool, s.cache) : b.cache("k_cache", ring, s.cache);
  const int vc = s.paged() ? b.cache("v_cache", pool, s.cache) : b.cache("v_cache", ring, s.cache);
  const int a = b.rmsnorm("attn_in", s.eps, attn_norm, 1.0, x);
  const int q = b.linear("q", wq, s.head_dim, a);
  const int k = b.linear("k", wk, s.head_dim, a);
  const int v = b.linear("v", wv, s.head_dim, a);
  const RopeSpec rope{s.theta, s.head_dim / 2, 1};
  const int qr = b.rope("q_rotated", rope, pos, q);
  const int kr = b.rope("k_rotated", rope, pos, k);
  b.kv_store("store_k", kc, pos, slot, kr);
  b.kv_store("store_v", vc, pos, slot, v);
  AttnSpec spec;
  spec.heads = s.heads;
  spec.kv_heads = s.kv_heads;
  spec.head_dim = s.head_dim;
  spec.scale = 1.0 / std::sqrt((double)s.head_dim);
  const int o = b.attend("attended", spec, qr, kc, vc, pos, slot);
  const int out = b.linear("attn_out", wo, 0, o);
  const int x1 = b.add("x1", x, out);
  const int m = b.rmsnorm("mlp_in", s.eps, mlp_norm, 1.0, x1);
  int ffn_out;
  if (s.experts) {  // each row's top_k experts, GELU-gated, weighted by the route
    const int logits = b.linear("router_logits", router, 0, m);
    const auto [ids, ws] = b.route("route", s.top_k, expert_scale, logits);
    const int gu = b.linear_routed("experts_gu", egu, ids, m);
    const int act = b.gated_gelu("experts_act", gu);
    const int eo = b.linear_routed("experts_out", edn, ids, act);
    ffn_out = b.combine_ranks("experts_sum", ws, eo);
  } else {
    const int gate = b.linear("gate", wg, 0, m);
    const int up = b.linear("up", wu, 0, m);
    const int act = b.silu_mul("mlp_act", gate, up);
    ffn_out = b.linear("mlp_out", wd, 0, act);
  }
  const int x2 = b.add("x2", x1, ffn_out);
  b.output("x", x2);
  return b.done();
}

Program embed_program(const LlamaShape& s) {
  Builder b("embed");
  const int tok = b.row_ints("token", 1, s.vocab);
  const int table = b.weight("embed", {s.vocab, s.d_model}, s.weights);
  const int x = b.gather("x", table, tok, 1.0);
  b.output("x", x);
  return b.done();
}

Program head_program(const LlamaShape& s) {
  Builder b("head");
  const int x = b.input("x", whole_row(s.d_model));
  const int norm = b.weight("final_norm", {s.d_model}, s.weights);
  const int embed = b.weight("embed", {s.vocab, s.d_model}, s.weights);
  const int n = b.rmsnorm("final_normed", s.eps, norm, 1.0, x);
  const int logits = b.linear("logits", embed, 0, n);
  const int token = b.argmax("token", logits);
  b.output("token", token);
  return b.done();
}

// ---------------------------------------------------------------------------
// The text form

namespace {

std::string dbl(double d) {
  uint64_t bits;
  std::memcpy(&bits, &d, 8);
  char buf[40];
  std::snprintf(buf, sizeof buf, "f64:0x%" PRIx64, bits);
  return buf;
}

std::string shape_text(Shape sh) { return "[" + std::to_string(sh.width) + "/" + std::to_string(sh.segment) + "]"; }

std::string dims_text(const std::vector<uint64_t>& ds) {
  std::string s = "[";
  for (size_t i = 0; i < ds.size(); ++i) s += (i ? ", " : "") + std::to_string(ds[i]);
  return s + "]";
}

std::string kind_text(const SourceKind& k) {
  switch (k.kind) {
    case SrcKind::Input: return "input " + shape_text(k.shape) + " " + k.type;
    case SrcKind::RowInts: return "row_ints " + std::to_string(k.count) + " below " + std::to_string(k.bound);
    case SrcKind::Weight: return "weight " + dims_text(k.dims) + " " + k.type + " " + k.layout;
    case SrcKind::Table:
      return "table " + std::to_string(k.entries) + " x " + dims_text(k.dims) + " " + k.type + " " + k.layout;
    case SrcKind::Cache: {
      std::string t = k.ring ? "ring slots " + std::to_string(k.r.slots) + " heads " + std::to_string(k.r.kv_heads) +
                                   " length " + std::to_string(k.r.length) + " dim " + std::to_string(k.r.head_dim)
                             : "paged blocks " + std::to_string(k.pg.blocks) + " size " +
                                   std::to_string(k.pg.block_size) + " heads " + std::to_string(k.pg.kv_heads) +
                                   " dim " + std::to_string(k.pg.head_dim);
      return "cache " + t + " " + k.elem;
    }
  }
  return "?";
}

}  // namespace

std::string render_program(const Program& p) {
  auto val = [&](int v) {
    const Value* x = p.value(v);
    return x ? x->name : "%" + std::to_string(v);
  };
  auto src = [&](int s) {
    const Source* x = p.source(s);
    return x ? x->name : std::string("?");
  };
  auto op_text = [&](const Op& o) -> std::string {
    const std::string& k = o.kind;
    if (k == "Input") return "input(" + src(o.sources[0]) + ")";
    if (k == "Linear") return "linear(" + src(o.sources[0]) + ", " + val(o.values[0]) + ") segment " +
                              std::to_string(o.segment);
    if (k == "LinearRouted")
      return "linear_routed(" + src(o.sources[0]) + ", " + val(o.values[0]) + ", " + val(o.values[1]) + ")";
    if (k == "RmsNorm") {
      const std::string g = o.gamma ? ", gamma " + src(o.sources[0]) : "";
      return "rmsnorm(" + val(o.values[0]) + ", eps " + dbl(o.eps) + g + ", factor " + dbl(o.factor) + ")";
    }
    if (k == "Add" || k == "Concat")
      return std::string(k == "Add" ? "add" : "concat") + "(" + val(o.values[0]) + ", " + val(o.values[1]) + ")";
    if (k == "ScaleBy") return "scale_by(" + src(o.sources[0]) + ", " + val(o.values[0]) + ")";
    if (k == "GatedGelu") return "gated_gelu(" + val(o.values[0]) + ")";
    if (k == "GeluMul") return "gelu_mul(" + val(o.values[0]) + ", " + val(o.values[1]) + ")";
    if (k == "SiluMul") return "silu_mul(" + val(o.values[0]) + ", " + val(o.values[1]) + ")";
    if (k == "Rope") {
      const std::string axes = o.rope.axes == 1 ? "" : ", axes " + std::to_string(o.rope.axes);
      return "rope(" + val(o.values[0]) + ", " + src(o.sources[0]) + ", theta " + dbl(o.rope.theta) + ", rotated " +
             std::to_string(o.rope.rotated) + axes + ")";
    }
    if (k == "Softcap") return "softcap(" + val(o.values[0]) + ", " + dbl(o.f) + ")";
    if (k == "Route") {
      const std::string sc = o.route.expert_scale ? ", scale " + src(*o.route.expert_scale) : "";
      return "route(" + val(o.values[0]) + ", k " + std::to_string(o.route.k) + sc + ")";
    }
    if (k == "CombineRanks") return "combine_ranks(" + val(o.values[0]) + ", " + val(o.values[1]) + ")";
    if (k == "KvStore")
      return "kv_store(" + src(o.sources[0]) + ", " + src(o.sources[1]) + ", " + src(o.sources[2]) + ", " +
             val(o.values[0]) + ")";
    if (k == "Attend") {
      const AttnSpec& a = o.attn;
      const std::string w = a.window ? ", window " + std::to_string(*a.window) : "";
      const std::string reach =
          a.reach ? ", reach " + src(a.reach->first) + " ahead " + std::to_string(a.reach->second) : "";
      return "attend(" + val(o.values[0]) + ", " + src(o.sources[0]) + ", " + src(o.sources[1]) + ", " +
             src(o.sources[2]) + ", " + src(o.sources[3]) + ", heads " + std::to_string(a.heads) + "/" +
             std::to_string(a.kv_heads) + ", dim " + std::to_string(a.head_dim) + w + ", scale " + dbl(a.scale) +
             reach + ")";
    }
    if (k == "Gather") return "gather(" + src(o.sources[0]) + ", " + src(o.sources[1]) + ", factor " + dbl(o.f) + ")";
    if (k == "Standardize")
      return "standardize(" + val(o.values[0]) + ", " + src(o.sources[0]) + ", " + src(o.sources[1]) + ", factor " +
             dbl(o.f) + ")";
    if (k == "ArgMax") return "argmax(" + val(o.values[0]) + ")";
    throw Refusal("render: an operation of kind " + k + " has no text form.");
  };
  std::string out = "program " + p.name + "\n";
  for (const Source& s : p.sources) out += "  source " + s.name + " : " + kind_text(s.kind) + "\n";
  for (const Node& n : p.nodes) {
    std::string outs;
    for (size_t i = 0; i < n.outputs.size(); ++i) {
      const Value& v = p.values[n.outputs[i]];
      outs += (i ? ", " : "") + v.name + " : " + shape_text(v.shape) + " " + v.type;
    }
    out += "  " + outs + (n.outputs.empty() ? "" : " = ") + n.name + " " + op_text(n.op) + "\n";
  }
  for (const Output& o : p.outputs) out += "  output " + o.name + " = " + val(o.value) + "\n";
  return out;
}

// ---------------------------------------------------------------------------
// The parser of the text form: the program a text renders from.

namespace {

struct Cursor {
  std::string s;
  size_t i = 0;
  explicit Cursor(std::string t) : s(std::move(t)) {}
  bool at_end() const { return i >= s.size(); }
  bool peek(const std::string& t) const { return s.compare(i, t.size(), t) == 0; }
  void expect(const std::string& t) {
    if (!peek(t)) throw Refusal("parse: expected '" + t + "' at '" + s.substr(i, 40) + "'.");
    i += t.size();
  }
  bool accept(const std::string& t) {
    if (!peek(t)) return false;
    i += t.size();
    return true;
  }
  std::string word() {  // up to a space, comma, parenthesis, bracket or slash
    size_t j = i;
    while (j < s.size() && !std::strchr(" ,()[]/", s[j])) ++j;
    if (j == i) throw Refusal("parse: expected a word at '" + s.substr(i, 40) + "'.");
    std::string w = s.substr(i, j - i);
    i = j;
    return w;
  }
  uint64_t num() { return std::stoull(word()); }
  double dbl() {
    expect("f64:0x");
    const std::string h = word();
    uint64_t bits = std::stoull(h, nullptr, 16);
    double d;
    std::memcpy(&d, &bits, 8);
    return d;
  }
};

Shape parse_shape(Cursor& c) {
  c.expect("[");
  Shape sh;
  sh.width = c.num();
  c.expect("/");
  sh.segment = c.num();
  c.expect("]");
  return sh;
}

std::vector<uint64_t> parse_dims(Cursor& c) {
  std::vector<uint64_t> ds;
  c.expect("[");
  while (!c.accept("]")) {
    ds.push_back(c.num());
    c.accept(", ");
  }
  return ds;
}

}  // namespace

Program parse_program(const std::string& text) {
  Program p;
  std::map<std::string, int> srcs, vals;
  std::istringstream in(text);
  std::string line;
  bool first = true;
  while (std::getline(in, line)) {
    if (line.empty()) continue;
    Cursor c(line);
    if (first) {
      c.expect("program ");
      p.name = line.substr(c.i);
      first = false;
      continue;
    }
    c.expect("  ");
    if (c.accept("source ")) {
      Source s;
      s.id = (int)p.sources.size();
      s.name = c.word();
      c.expect(" : ");
      SourceKind& k = s.kind;
      const std::string what = c.word();
      c.expect(" ");
      if (what == "input") {
        k.kind = SrcKind::Input;
        k.shape = parse_shape(c);
        c.expect(" ");
        k.type = c.word();
      } else if (what == "row_ints") {
        k.kind = SrcKind::RowInts;
        k.count = c.num();
        c.expect(" below ");
        k.bound = c.num();
      } else if (what == "weight") {
        k.kind = SrcKind::Weight;
        k.dims = parse_dims(c);
        c.expect(" ");
        k.type = c.word();
        c.expect(" ");
        k.layout = c.word();
      } else if (what == "table") {
        k.kind = SrcKind::Table;
        k.entries = c.num();
        c.expect(" x ");
        k.dims = parse_dims(c);
        c.expect(" ");
        k.type = c.word();
        c.expect(" ");
        k.layout = c.word();
      } else if (what == "cache") {
        k.kind = SrcKind::Cache;
        if (c.accept("ring slots ")) {
          k.ring = true;
          k.r.slots = c.num();
          c.expect(" heads ");
          k.r.kv_heads = c.num();
          c.expect(" length ");
          k.r.length = c.num();
          c.expect(" dim ");
          k.r.head_dim = c.num();
        } else {
          c.expect("paged blocks ");
          k.ring = false;
          k.pg.blocks = c.num();
          c.expect(" size ");
          k.pg.block_size = c.num();
          c.expect(" heads ");
          k.pg.kv_heads = c.num();
          c.expect(" dim ");
          k.pg.head_dim = c.num();
        }
        c.expect(" ");
        k.elem = c.word();
      } else {
        throw Refusal("parse: a source of kind " + what + ".");
      }
      srcs[s.name] = s.id;
      p.sources.push_back(s);
      continue;
    }
    if (c.accept("output ")) {
      Output o;
      o.name = c.word();
      c.expect(" = ");
      o.value = vals.at(c.word());
      p.outputs.push_back(o);
      continue;
    }
    // A node: [outs = ]name op
    Node n;
    n.id = (int)p.nodes.size();
    const size_t eq = line.find(" = ");
    const size_t paren = line.find('(');
    if (eq != std::string::npos && eq < paren) {
      while (true) {
        Value v;
        v.id = (int)p.values.size();
        v.name = c.word();
        c.expect(" : ");
        v.shape = parse_shape(c);
        c.expect(" ");
        v.type = c.word();
        vals[v.name] = v.id;
        p.values.push_back(v);
        n.outputs.push_back(v.id);
        if (c.accept(" = ")) break;
        c.expect(", ");
      }
    }
    n.name = c.word();
    c.expect(" ");
    const std::string kind = c.word();
    c.expect("(");
    Op& o = n.op;
    auto V = [&]() { return vals.at(c.word()); };
    auto S = [&]() { return srcs.at(c.word()); };
    if (kind == "input") {
      o.kind = "Input";
      o.sources = {S()};
    } else if (kind == "linear") {
      o.kind = "Linear";
      o.sources = {S()};
      c.expect(", ");
      o.values = {V()};
      c.expect(") segment ");
      o.segment = c.num();
      p.nodes.push_back(n);
      continue;
    } else if (kind == "linear_routed") {
      o.kind = "LinearRouted";
      o.sources = {S()};
      c.expect(", ");
      const int ids = V();
      c.expect(", ");
      o.values = {ids, V()};
    } else if (kind == "rmsnorm") {
      o.kind = "RmsNorm";
      o.values = {V()};
      c.expect(", eps ");
      o.eps = c.dbl();
      if (c.accept(", gamma ")) {
        o.gamma = true;
        o.sources = {S()};
      }
      c.expect(", factor ");
      o.factor = c.dbl();
    } else if (kind == "add" || kind == "concat" || kind == "gelu_mul" || kind == "silu_mul" ||
               kind == "combine_ranks") {
      o.kind = kind == "add" ? "Add" : kind == "concat" ? "Concat" : kind == "gelu_mul" ? "GeluMul"
                               : kind == "silu_mul" ? "SiluMul" : "CombineRanks";
      const int a = V();
      c.expect(", ");
      o.values = {a, V()};
    } else if (kind == "scale_by") {
      o.kind = "ScaleBy";
      o.sources = {S()};
      c.expect(", ");
      o.values = {V()};
    } else if (kind == "gated_gelu") {
      o.kind = "GatedGelu";
      o.values = {V()};
    } else if (kind == "rope") {
      o.kind = "Rope";
      o.values = {V()};
      c.expect(", ");
      o.sources = {S()};
      c.expect(", theta ");
      o.rope.theta = c.dbl();
      c.expect(", rotated ");
      o.rope.rotated = c.num();
      if (c.accept(", axes ")) o.rope.axes = c.num();
    } else if (kind == "softcap") {
      o.kind = "Softcap";
      o.values = {V()};
      c.expect(", ");
      o.f = c.dbl();
    } else if (kind == "route") {
      o.kind = "Route";
      o.values = {V()};
      c.expect(", k ");
      o.route.k = c.num();
      if (c.accept(", scale ")) {
        const int s = S();
        o.route.expert_scale = s;
        o.sources = {s};
      }
    } else if (kind == "kv_store") {
      o.kind = "KvStore";
      const int cache = S();
      c.expect(", ");
      const int pos = S();
      c.expect(", ");
      const int seq = S();
      c.expect(", ");
      o.sources = {cache, pos, seq};
      o.values = {V()};
    } else if (kind == "attend") {
      o.kind = "Attend";
      o.values = {V()};
      for (int t = 0; t < 4; ++t) {
        c.expect(", ");
        o.sources.push_back(S());
      }
      c.expect(", heads ");
      o.attn.heads = c.num();
      c.expect("/");
      o.attn.kv_heads = c.num();
      c.expect(", dim ");
      o.attn.head_dim = c.num();
      if (c.accept(", window ")) o.attn.window = c.num();
      c.expect(", scale ");
      o.attn.scale = c.dbl();
      if (c.accept(", reach ")) {
        const int s = S();
        c.expect(" ahead ");
        o.attn.reach = std::make_pair(s, c.num());
        o.sources.push_back(s);
      }
    } else if (kind == "gather") {
      o.kind = "Gather";
      const int t = S();
      c.expect(", ");
      o.sources = {t, S()};
      c.expect(", factor ");
      o.f = c.dbl();
    } else if (kind == "standardize") {
      o.kind = "Standardize";
      o.values = {V()};
      c.expect(", ");
      const int b0 = S();
      c.expect(", ");
      o.sources = {b0, S()};
      c.expect(", factor ");
      o.f = c.dbl();
    } else if (kind == "argmax") {
      o.kind = "ArgMax";
      o.values = {V()};
    } else {
      throw Refusal("parse: an operation " + kind + ".");
    }
    c.expect(")");
    p.nodes.push_back(n);
  }
  return p;
}

}  // namespace fkh
