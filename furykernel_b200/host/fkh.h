// The host side of furykernel-cuda in C++: FuryKernel's programs
// (src/FuryKernel/Program/Graph.hs, Build.hs), the planner
// (src/FuryKernel/Program/Plan.hs) and the lowering of a plan's steps to
// launches of the CUDA target's kernel table. Internal to the host library;
// its C ABI is include/furykernel_host.h.
#pragma once

#include <cstdint>
#include <map>
#include <optional>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

namespace fkh {

// A refusal with the text the caller reports (the lowering's and the
// builder's errors).
struct Refusal : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// ---------------------------------------------------------------------------
// Programs (Graph.hs)

struct Shape {
  uint64_t width = 0, segment = 0;  // a row's elements, in segments (Graph.hs:88-100)
  bool operator==(const Shape& o) const { return width == o.width && segment == o.segment; }
};
inline Shape whole_row(uint64_t n) { return {n, n}; }

struct Ring {
  uint64_t slots = 0, kv_heads = 0, length = 0, head_dim = 0;
};
struct Paged {
  uint64_t blocks = 0, block_size = 0, kv_heads = 0, head_dim = 0;
};

enum class SrcKind { Input, RowInts, Weight, Table, Cache };

struct SourceKind {
  SrcKind kind = SrcKind::Input;
  Shape shape;                  // Input
  std::string type;             // Input, Weight, Table
  uint64_t count = 0, bound = 0;  // RowInts
  std::vector<uint64_t> dims;   // Weight, Table
  std::string layout;           // Weight, Table: "out_in" | "row_major"
  uint64_t entries = 0;         // Table
  bool ring = true;             // Cache: Ring or Paged
  Ring r;
  Paged pg;
  std::string elem;  // Cache element: "bf16", "f16", "f32"
};

struct Source {
  int id = 0;
  std::string name;
  SourceKind kind;
};

struct RopeSpec {
  double theta = 10000.0;
  uint64_t rotated = 0, axes = 1;
};

struct AttnSpec {
  uint64_t heads = 0, kv_heads = 0, head_dim = 0;
  std::optional<uint64_t> window;
  double scale = 1.0;
  std::optional<std::pair<int, uint64_t>> reach;  // (source, ahead)
};

struct RouteSpec {
  uint64_t k = 0;
  std::optional<int> expert_scale;
};

// One operation (Graph.hs:299-360): `kind` names the constructor; values and
// sources by id; the arguments the kind takes.
struct Op {
  std::string kind;
  std::vector<int> values, sources;
  double eps = 0, factor = 1, f = 0;  // RmsNorm (eps, factor); Gather/Softcap/Standardize (f)
  bool gamma = false;                 // RmsNorm
  uint64_t segment = 0;               // Linear
  RopeSpec rope;
  AttnSpec attn;
  RouteSpec route;
};

struct Value {
  int id = 0;
  std::string name;
  Shape shape;
  std::string type;
};

struct Node {
  int id = 0;
  std::string name;
  Op op;
  std::vector<int> outputs;
};

struct Output {
  std::string name;
  int value = 0;
};

struct Program {
  std::string name;
  std::vector<Source> sources;  // by id
  std::vector<Value> values;    // by id
  std::vector<Node> nodes;      // by id
  std::vector<Output> outputs;

  const Value* value(int id) const { return id >= 0 && id < (int)values.size() ? &values[id] : nullptr; }
  const Source* source(int id) const { return id >= 0 && id < (int)sources.size() ? &sources[id] : nullptr; }
  const Node* node(int id) const { return id >= 0 && id < (int)nodes.size() ? &nodes[id] : nullptr; }
};

bool pointwise(const std::string& kind);
std::string render_program(const Program& p);
Program parse_program(const std::string& text);

// The program builder (Build.hs): sources keep their names; values and nodes
// take a suffix where a name is taken.
class Builder {
 public:
  explicit Builder(std::string name) { p_.name = std::move(name); }
  Program done() const { return p_; }

  int input(const std::string& name, Shape sh, const std::string& type = "f32");
  int row_ints(const std::string& name, uint64_t n, uint64_t bound);
  int weight(const std::string& name, std::vector<uint64_t> dims, const std::string& type);
  int cache(const std::string& name, Ring layout, const std::string& elem);
  int cache(const std::string& name, Paged layout, const std::string& elem);
  int linear(const std::string& name, int w, uint64_t seg, int x);
  int rmsnorm(const std::string& name, double eps, std::optional<int> gamma, double factor, int x);
  int add(const std::string& name, int a, int b);
  int silu_mul(const std::string& name, int a, int b);
  int rope(const std::string& name, RopeSpec r, int pos, int x);
  void kv_store(const std::string& name, int cache, int positions, int sequences, int x);
  int attend(const std::string& name, AttnSpec spec, int q, int keys, int vals, int positions, int sequences);
  int gather(const std::string& name, int table, int tokens, double factor);
  int argmax(const std::string& name, int x);
  int table(const std::string& name, uint64_t entries, std::vector<uint64_t> dims, const std::string& type);
  int linear_routed(const std::string& name, int table, int ids, int x);
  std::pair<int, int> route(const std::string& name, uint64_t k, std::optional<int> scale, int x);
  int gated_gelu(const std::string& name, int x);
  int combine_ranks(const std::string& name, int w, int x);
  void output(const std::string& name, int v);

  const Program& program() const { return p_; }

 private:
  std::string fresh(const std::string& base);
  int source(const std::string& name, SourceKind k);
  std::vector<int> node(const std::string& name, Op op,
                        const std::vector<std::tuple<std::string, Shape, std::string>>& outs);
  int one(const std::string& name, Op op, Shape sh, const std::string& type = "f32");
  uint64_t rows_of(int src) const;

  Program p_;
  std::set<std::string> names_;
};

// The Llama-shaped programs of this path (one decoder layer, the embedding,
// the head): f32 activations; f32 or bf16 weights and KV caches
// (tests/restated/llama.py states them too).
struct LlamaShape {
  uint64_t d_model = 4096, heads = 32, kv_heads = 32, head_dim = 128, ffn = 11008, vocab = 32000, layers = 32;
  double theta = 10000.0, eps = 1e-5;
  uint64_t slots = 1, length = 4096, positions = 4096;
  std::string weights = "f32", cache = "f32";  // element types: "f32", "bf16" or "f16"
  // Routed experts in place of the dense FFN: `experts` of ffn each, every
  // row taking its top_k (experts 0: the dense SiLU-gated FFN).
  uint64_t experts = 0, top_k = 2;
  // Each chosen expert's weight times its own scale (the route's expert
  // scale, RouteSpec, Graph.hs:249-257): a weight [experts] of the
  // weights' type after the router.
  bool expert_scale = false;
  // A paged cache (Graph.hs:144-152) instead of the ring: a pool of `blocks`
  // blocks of `block_size` positions a layer, each row's block table of
  // table_len() entries. block_size 0: the ring of `slots` and `length`.
  uint64_t blocks = 0, block_size = 0;
  bool paged() const { return block_size > 0; }
  uint64_t table_len() const { return paged() ? (positions + block_size - 1) / block_size : 0; }
  uint64_t weight_bytes() const { return weights == "f32" ? 4 : 2; }
  uint64_t cache_bytes() const { return cache == "f32" ? 4 : 2; }
  uint64_t q_width() const { return heads * head_dim; }
  uint64_t kv_width() const { return kv_heads * head_dim; }
};
Program layer_program(const LlamaShape& s, const std::string& name = "layer");
Program embed_program(const LlamaShape& s);
Program head_program(const LlamaShape& s);

// ---------------------------------------------------------------------------
// Plans (Plan.hs)

struct Work {
  std::string kind;  // Anchor, Recompute, Epilogue, Combine, Effect, Stage, Land
  int node = 0;
  bool operator==(const Work& o) const { return kind == o.kind && node == o.node; }
};

// A value in memory between steps: its elements of a type, attention's
// partials, or a staged store's values for a cache.
struct Stored {
  int value = 0;
  std::string form;  // "elements" | "partials" | "staged"
  std::string type;  // elements
  int cache = -1;    // staged
  bool operator==(const Stored& o) const {
    return value == o.value && form == o.form && type == o.type && cache == o.cache;
  }
};

struct Step {
  int index = 0;
  std::string name;
  std::vector<Work> work;
  std::vector<Stored> stores, reads;
  std::vector<int> caches;
};

struct Plan {
  Program program;
  std::vector<Step> steps;
};

struct PlanOptions {
  bool horizontal = true, gated = false, store_gelus = false;
  uint64_t sequence_rows = 1;
};

Plan plan(const PlanOptions& o, const Program& p);
std::string render_plan(const Plan& pl);
// A plan step's name: s, one or more digits, _, something
// (src/FuryKernel/Program/Plan.hs:162-165).
bool is_step_name(const std::string& t);

// ---------------------------------------------------------------------------
// Lowering: a step as one launch of the target's kernel table.

struct Launch {
  std::string kernel;
  std::vector<std::pair<std::string, double>> params;  // by name, in the table's order of declaration
  std::vector<uint64_t> bufs;                           // addresses, in declaration order
  double param(const std::string& n) const;
  bool has(const std::string& n) const;
  void set(const std::string& n, double v);
};

// A stored value on the device: its buffer, its first column and the
// buffer's row stride (elements).
struct View {
  uint64_t base = 0;
  uint64_t col = 0, ld = 0, width = 0;
  uint64_t ptr() const { return base + 4 * col; }
};

struct Binding {
  std::map<std::string, uint64_t> weights;  // source name -> address
  std::map<std::string, uint64_t> ints;     // source name -> address of [m] u32
  std::map<std::string, uint64_t> caches;   // source name -> address of the layer's Ring
  std::map<std::string, View> values;       // value name -> View
  uint64_t m = 1;
};

struct AttnBufs {
  uint64_t chunk = 32, max_splits = 1;
  uint64_t partials[3] = {0, 0, 0};
};

Launch lower_step(const Program& p, const Step& step, const Binding& b, uint64_t cos_t, uint64_t sin_t,
                  const AttnBufs& attn);
// A step as its launches: the routed-experts steps as several, any other
// as lower_step's one.
std::vector<Launch> lower_steps(const Program& p, const Step& step, const Binding& b, uint64_t cos_t, uint64_t sin_t,
                                const AttnBufs& attn);

// A kernel's element-type form: the f32 entry's name, or with the suffix of
// its 16-bit weights (_wbf16, _wf16) or 16-bit KV caches (_kvbf16, _kvf16).
// weight_form / cache_form: the suffix for weights or caches of element
// type t ("f32": none); they throw Refusal, naming `what`, for a type no
// kernel reads.
std::string weight_form(const std::string& t, const std::string& what);
std::string cache_form(const std::string& t, const std::string& what);
std::pair<std::string, std::string> kernel_form(const std::string& kernel);

// The whole decode step of the Llama engine (furykernel_b200/engine.py):
// every address the launches bind, the shape and the choices.
struct LlamaLaunchDesc {
  LlamaShape full;  // the whole model
  uint64_t batch = 1, rank = 0, world = 1, sms = 148, chunk = 32;
  bool gate_up_interleaved = true, peer_exchange = false, fuse_attention = false;
  // the weight arena: layers (layer_elems floats each, q k v o gate up down attn_norm mlp_norm), then the
  // whole embedding and the final norm
  uint64_t arena = 0, kbase = 0, vbase = 0;
  uint64_t cos_t = 0, sin_t = 0;
  uint64_t tokens = 0, pos = 0, slot = 0;
  uint64_t x = 0, x1 = 0, qkv = 0, att = 0, gu = 0, act = 0, logits = 0, out_ids = 0;
  uint64_t partial = 0, pairs = 0, pairs_all = 0;
  uint64_t part[3] = {0, 0, 0};
  // A committed selection's split-K for each GEMV shape (n, k), for every
  // batch alike; shapes it does not list take the default.
  std::map<std::pair<uint64_t, uint64_t>, uint64_t> splits;
  // Routed experts: the normed row, the router's logits, the route's ids
  // and weights, the experts' gate/up rows, their gate, their outputs.
  uint64_t mlp_in = 0, router_logits = 0, route_ids = 0, route_weights = 0, experts_gu = 0, experts_act = 0,
           experts_out = 0;
  // The layer's plan options beyond the defaults (PlanOptions, Plan.hs:243-268):
  // a route in a step of its own, gelus stored by their own step.
  bool gated = false, store_gelus = false;
};

std::vector<Launch> llama_launches(const LlamaLaunchDesc& d);
// This rank's shard of the model (heads, KV heads and ffn over the ranks),
// refused when the model does not split evenly.
LlamaShape shard_of(const LlamaLaunchDesc& d);
// A layer's floats in the weight arena, and the addresses of its weights
// (q k v o gate up down attn_norm mlp_norm, in that order).
uint64_t layer_elems(const LlamaShape& s);
std::map<std::string, uint64_t> layer_weights(const LlamaShape& s, uint64_t arena, uint64_t l);
uint64_t split_for(uint64_t n_rows, uint64_t k, uint64_t sms);

// The prompt prefill of up to `rows` rows in front of a decode step
// (furykernel_b200/prefill.py): its row buffers, the weights' TF32 halves
// (two arenas laid out as the weight arena) and its choices.
struct PrefillDesc {
  uint64_t rows = 1, chunk = 32, positions = 1;
  bool one_slot = false;  // every run's rows in one slot: the query-tiled prompt attention
  uint64_t w_hi = 0, w_lo = 0;
  uint64_t tokens = 0, pos = 0, slot = 0;
  uint64_t x = 0, a = 0, a_hi = 0, a_lo = 0, qkv = 0, att = 0, tmp = 0, x1 = 0, gu = 0, act = 0;
  uint64_t part[3] = {0, 0, 0};
  // Routed experts: the rows' router logits, route ids and weights, the
  // experts' gate/up rows, their gate and their outputs.
  uint64_t router_logits = 0, route_ids = 0, route_weights = 0, experts_gu = 0, experts_act = 0, experts_out = 0;
};

std::vector<Launch> prefill_launches(const LlamaLaunchDesc& decode, const PrefillDesc& p, uint64_t m);

}  // namespace fkh
