// The planner (src/FuryKernel/Program/Plan.hs): a program as steps, each one
// kernel launch, and the cut points where steps meet. No threadgroup waits
// for another inside a kernel: a value is stored once the step that writes
// it has finished. Anchors (linear layers, attention) set a step's grid;
// cheap operations are recomputed before them from stored values or run as
// epilogues on a linear layer's tile; light steps hold cache stores,
// attention's combine and outputs no anchor makes. The rules, the state
// machine and the names are the reference's, so that the launch lists the
// target runs are the reference's plans.
#include <algorithm>
#include <functional>

#include "fkh.h"

namespace fkh {
namespace {

enum Cost { CHEAP = 0, PASS = 1, EXPENSIVE = 2 };  // Plan.hs:196-206, ordered

// Where a value is (Plan.hs:166-181 and the planner's bookkeeping): stored
// by step a (-1: an input), attention's partials of step a, on step a's tile
// of anchor b, or not yet computed (virtual) at cost a.
struct Avail {
  enum K { Stored, Partials, Tile, Virtual } k = Stored;
  int a = -1, b = -1;
};

struct StepB {
  int index = 0;
  std::vector<Work> work;
  std::vector<Stored> stores;
  std::string family;  // "", "Gemv", "Attention"
  std::set<int> writes;
};

std::string anchor_family(const Op& op) {
  if (op.kind == "Linear" || op.kind == "LinearRouted") return "Gemv";
  if (op.kind == "Attend") return "Attention";
  return "";
}

int node_cost(const Program& p, const Op& op) {  // Plan.hs:214-223
  if (op.kind == "RmsNorm" || op.kind == "Route" || op.kind == "ArgMax") return PASS;
  if (op.kind == "Gather") {
    const Source* s = p.source(op.sources[1]);
    if (s && s->kind.kind == SrcKind::RowInts && s->kind.count > 1) return EXPENSIVE;
  }
  return CHEAP;
}

uint64_t ring_room(uint64_t length, std::optional<uint64_t> window, uint64_t bound) {  // Plan.hs:270-281
  const uint64_t seen = window ? *window : bound;
  return seen > length ? 0 : length - seen + 1;
}

Stored elements(int v, const std::string& type) { return Stored{v, "elements", type, -1}; }

template <typename T>
bool contains(const std::vector<T>& xs, const T& x) {
  return std::find(xs.begin(), xs.end(), x) != xs.end();
}

class Planner {
 public:
  Planner(const PlanOptions& o, const Program& p) : o_(o), p_(p) {
    for (const Node& n : p.nodes) {
      for (int v : n.outputs) producer_[v] = n.id;
      for (int v : n.op.values) consumers_[v].push_back(n.id);
    }
    for (const Output& out : p.outputs) output_values_.insert(out.value);
    staged_ = compute_staged();
  }

  Plan run() {
    for (const Node& n : p_.nodes) node(n);
    outputs();
    land_rest();
    close_open();
    Plan pl;
    pl.program = p_;
    for (const StepB& sb : closed_) pl.steps.push_back(finish(sb));
    return pl;
  }

 private:
  // -- the program's facts
  const Op& op_of(int n) const { return p_.nodes[n].op; }
  std::string type_of(int v) const {
    const Value* val = p_.value(v);
    return val ? val->type : "f32";
  }
  std::vector<int> outs_of(int n) const { return n >= 0 && n < (int)p_.nodes.size() ? p_.nodes[n].outputs : std::vector<int>{}; }
  const Node* producer(int v) const {
    auto it = producer_.find(v);
    return it == producer_.end() ? nullptr : &p_.nodes[it->second];
  }
  std::vector<int> consumers(int v) const {
    auto it = consumers_.find(v);
    return it == consumers_.end() ? std::vector<int>{} : it->second;
  }
  uint64_t position_bound(int s) const {
    const Source* src = p_.source(s);
    return src && src->kind.kind == SrcKind::RowInts ? src->kind.bound : 0;
  }

  std::set<int> compute_staged() const {
    std::set<int> out;
    const auto& nodes = p_.nodes;
    for (size_t i = 0; i < nodes.size(); ++i) {
      const Node& n = nodes[i];
      if (n.op.kind != "KvStore") continue;
      const int c = n.op.sources[0];
      const Source* src = p_.source(c);
      if (!src || src->kind.kind != SrcKind::Cache || !src->kind.ring) continue;
      const uint64_t length = src->kind.r.length;
      for (size_t j = i + 1; j < nodes.size(); ++j) {
        const Node& r = nodes[j];
        if (r.op.kind == "Attend" && (r.op.sources[0] == c || r.op.sources[1] == c)) {
          if (o_.sequence_rows > ring_room(length, r.op.attn.window, position_bound(r.op.sources[2]))) {
            out.insert(n.id);
            break;
          }
        }
      }
    }
    return out;
  }

  std::optional<int> staged_into(int c) const {
    for (const Node& n : p_.nodes)
      if (n.op.kind == "KvStore" && n.op.sources[0] == c && staged_.count(n.id)) return n.id;
    return std::nullopt;
  }

  std::optional<int> last_reader(int c) const {
    std::optional<int> last;
    for (const Node& n : p_.nodes)
      if (n.op.kind == "Attend" && (n.op.sources[0] == c || n.op.sources[1] == c)) last = n.id;
    return last;
  }

  // -- availability
  Avail avail_of(int v) const {
    auto it = avail_.find(v);
    return it == avail_.end() ? Avail{} : it->second;
  }
  std::optional<int> open_index() const { return open_ ? std::optional<int>(open_->index) : std::nullopt; }
  bool is_open(int index) const { return open_ && open_->index == index; }

  // -- steps
  void close_open() {
    if (!open_) return;
    outputs_here();
    store_shared();
    StepB sb = *open_;
    std::set<int> in_step;
    for (const Work& w : sb.work) in_step.insert(w.node);
    std::vector<int> tiled;
    for (const Work& w : sb.work)
      if (w.kind == "Anchor" || w.kind == "Epilogue")
        for (int v : outs_of(w.node)) tiled.push_back(v);
    std::vector<Stored> stores;
    for (int v : tiled)
      for (const Stored& st : store_tile(sb, in_step, v)) stores.push_back(st);
    sb.stores.insert(sb.stores.end(), stores.begin(), stores.end());
    closed_.push_back(sb);
    open_.reset();
  }

  std::vector<Stored> store_tile(const StepB& sb, const std::set<int>& in_step, int v) {
    bool outside = false;
    for (int c : consumers(v))
      if (!in_step.count(c)) outside = true;
    if (!(outside || output_values_.count(v))) return {};
    const Node* n = producer(v);
    if (n && n->op.kind == "Attend") {
      avail_[v] = Avail{Avail::Partials, sb.index, -1};
      return {Stored{v, "partials", "", -1}};
    }
    avail_[v] = Avail{Avail::Stored, sb.index, -1};
    return {elements(v, type_of(v))};
  }

  void new_step(const std::string& fam) {
    close_open();
    StepB sb;
    sb.index = next_++;
    sb.family = fam;
    open_ = sb;
  }

  void light_step() {
    bool anchored = false;
    if (open_)
      for (const Work& w : open_->work)
        if (w.kind == "Anchor") anchored = true;
    if (!(open_ && open_->family.empty() && !anchored)) new_step("");
    const std::optional<int> i = open_index();
    std::vector<std::tuple<int, int, int>> due, rest;
    for (const auto& l : landing_) {
      if (i && *i > std::get<0>(l))
        due.push_back(l);
      else
        rest.push_back(l);
    }
    for (const auto& [s, n, c] : due) {
      add_work(Work{"Land", n});
      if (open_) open_->writes.insert(c);
    }
    landing_ = rest;
  }

  void land_rest() {
    if (!landing_.empty()) light_step();
  }

  void add_work(const Work& w) {
    if (!open_) return;
    for (const Work& x : open_->work)
      if (x.node == w.node) return;
    open_->work.push_back(w);
  }

  void add_store(const Stored& st) {
    if (open_ && !contains(open_->stores, st)) open_->stores.push_back(st);
  }

  bool planned(int node) const {
    if (!open_) return false;
    for (const Work& w : open_->work)
      if (w.node == node) return true;
    return false;
  }

  // -- chains
  void chain(int v) {
    const Avail a = avail_of(v);
    const std::optional<int> i = open_index();
    const Node* n = producer(v);
    if (a.k == Avail::Stored && (!i || a.a != *i)) return;
    if (a.k == Avail::Partials && n && (!i || a.a != *i)) {
      add_work(Work{"Combine", n->id});
      return;
    }
    if (n && !planned(n->id)) {
      for (int u : n->op.values) chain(u);
      add_work(Work{"Recompute", n->id});
    }
  }

  void outputs_here() {
    if (!open_) return;
    std::set<int> combined;
    for (const Work& w : open_->work)
      if (w.kind == "Combine") combined.insert(w.node);
    std::function<bool(int)> has = [&](int v) -> bool {
      const Avail a = avail_of(v);
      if (a.k == Avail::Stored) return true;
      if (a.k == Avail::Partials) {
        const Node* n = producer(v);
        return n && combined.count(n->id);
      }
      if (a.k == Avail::Virtual) {
        const Node* n = producer(v);
        if (n) {
          for (int u : n->op.values)
            if (!has(u)) return false;
          return true;
        }
      }
      return false;
    };
    if (open_->family.empty() && !combined.empty())
      for (const Output& o : p_.outputs)
        if (avail_of(o.value).k == Avail::Virtual && has(o.value)) materialize(o.value);
  }

  void store_shared() {
    if (!open_) return;
    std::set<int> in_step;
    for (const Work& w : open_->work) in_step.insert(w.node);
    auto needed = [&](int v) {
      for (int c : consumers(v))
        if (!in_step.count(c)) return true;
      return output_values_.count(v) > 0;
    };
    const int index = open_->index;
    auto store = [&](int v) {
      add_store(elements(v, type_of(v)));
      avail_[v] = Avail{Avail::Stored, index, -1};
    };
    const std::vector<Work> work = open_->work;
    for (const Work& w : work)
      if (w.kind == "Recompute")
        for (int v : outs_of(w.node)) {
          const Avail a = avail_of(v);
          if (a.k == Avail::Virtual && a.a >= PASS && needed(v)) store(v);
        }
    for (const Work& w : work)
      if (w.kind == "Combine")
        for (int v : outs_of(w.node))
          if (avail_of(v).k == Avail::Partials && needed(v)) store(v);
  }

  void materialize(int v) {
    light_step();
    chain(v);
    const std::optional<int> i = open_index();
    if (i) {
      add_store(elements(v, type_of(v)));
      avail_[v] = Avail{Avail::Stored, *i, -1};
    }
  }

  // -- nodes
  void node(const Node& n) {
    if (n.op.kind == "Input") {
      for (int v : n.outputs) avail_[v] = Avail{Avail::Stored, -1, -1};
    } else if (!anchor_family(n.op).empty()) {
      anchor(n, anchor_family(n.op));
    } else if (n.op.kind == "KvStore") {
      effect(n);
    } else {
      light(n);
    }
  }

  void anchor(const Node& n, const std::string& fam) {
    const Op& op = n.op;
    const std::vector<int> ins = op.values;
    for (int v : ins)
      if (touches_open(v)) {
        close_open();
        break;
      }
    for (int v : ins)
      if (expensive(v) || stored_gelu(v)) materialize(v);
    if (op.kind == "LinearRouted" && o_.gated)
      if (avail_of(op.values[0]).k != Avail::Stored) materialize(op.values[0]);
    bool reads_caches = false;
    if (open_)
      for (int c : op.sources)
        if (open_->writes.count(c)) reads_caches = true;
    const bool gated_here = op.kind == "LinearRouted" && o_.gated;
    const bool joins = open_ && o_.horizontal && open_->family == fam && !reads_caches && !gated_here;
    if (!joins) new_step(fam);
    for (int v : ins) chain(v);
    add_work(Work{"Anchor", n.id});
    const std::optional<int> s = open_index();
    if (s) {
      for (int v : n.outputs)
        avail_[v] = op.kind == "Attend" ? Avail{Avail::Partials, *s, -1} : Avail{Avail::Tile, *s, n.id};
      if (op.kind == "Attend") {
        std::vector<int> kv = {op.sources[0]};
        if (op.sources[1] != op.sources[0]) kv.push_back(op.sources[1]);
        for (int c : kv) {
          const std::optional<int> store = staged_into(c);
          if (last_reader(c) == std::optional<int>(n.id) && store) landing_.emplace_back(*s, *store, c);
        }
      }
    }
  }

  bool touches_open(int v0) const {
    const std::optional<int> i = open_index();
    std::set<int> seen;
    std::vector<int> todo = {v0};
    while (!todo.empty()) {
      const int v = todo.front();
      todo.erase(todo.begin());
      if (seen.count(v)) continue;
      seen.insert(v);
      const Avail a = avail_of(v);
      if ((a.k == Avail::Tile || a.k == Avail::Partials) && i && a.a == *i) return true;
      if (a.k == Avail::Virtual) {
        const Node* n = producer(v);
        if (n) todo.insert(todo.begin(), n->op.values.begin(), n->op.values.end());
      }
    }
    return false;
  }

  bool stored_gelu(int v) const {
    if (!o_.store_gelus) return false;
    const Node* n = producer(v);
    return n && (n->op.kind == "GeluMul" || n->op.kind == "GatedGelu") && avail_of(v).k == Avail::Virtual;
  }

  bool expensive(int v) const {
    const Avail a = avail_of(v);
    return a.k == Avail::Partials || (a.k == Avail::Virtual && a.a >= EXPENSIVE);
  }

  int input_cost(int v) const {
    const Avail a = avail_of(v);
    if (a.k == Avail::Virtual) return a.a;
    if (a.k == Avail::Partials) return EXPENSIVE;
    return CHEAP;
  }

  void light(const Node& n) {
    const Op& op = n.op;
    const std::vector<int> ins = op.values;
    std::vector<Avail> avails;
    for (int v : ins) avails.push_back(avail_of(v));
    const std::optional<int> i = open_index();
    std::vector<int> anchors, tiled_vals;
    for (size_t j = 0; j < ins.size(); ++j) {
      const Avail& a = avails[j];
      if (a.k == Avail::Tile && i && a.a == *i) {
        tiled_vals.push_back(ins[j]);
        if (!contains(anchors, a.b)) anchors.push_back(a.b);
      }
    }
    auto other = [&](int v, const Avail& a) {
      if (a.k == Avail::Stored) return true;
      if (a.k == Avail::Virtual && a.a == CHEAP) return !touches_open(v);
      return false;
    };
    bool others_ok = true;
    for (size_t j = 0; j < ins.size(); ++j)
      if (!contains(tiled_vals, ins[j]) && !other(ins[j], avails[j])) others_ok = false;
    if (anchors.size() == 1 && pointwise(op.kind) && others_ok) {
      for (size_t j = 0; j < ins.size(); ++j)
        if (avails[j].k == Avail::Virtual) chain(ins[j]);
      add_work(Work{"Epilogue", n.id});
      if (i)
        for (int v : n.outputs) avail_[v] = Avail{Avail::Tile, *i, anchors[0]};
    } else {
      int c = node_cost(p_, op);
      for (int v : ins) c = std::max(c, input_cost(v));
      for (int v : n.outputs) avail_[v] = Avail{Avail::Virtual, c, -1};
      if (o_.gated && (feeds_routed(n) || routes_output(n))) {
        for (int v : ins)
          if (touches_open(v)) {
            close_open();
            break;
          }
        if (!n.outputs.empty()) materialize(n.outputs[0]);
      }
    }
  }

  bool feeds_routed(const Node& r) const {
    if (r.op.kind != "Route" || r.outputs.empty()) return false;
    const int v = r.outputs[0];
    for (int c : consumers(v)) {
      const Op& op = op_of(c);
      if (op.kind == "LinearRouted" && op.values[0] == v) return true;
    }
    return false;
  }

  bool routes_output(const Node& r) const {
    return r.op.kind == "Route" && !r.outputs.empty() && output_values_.count(r.outputs[0]);
  }

  void effect(const Node& n) {
    const Op& op = n.op;
    const std::vector<int> ins = op.values;
    if (staged_.count(n.id)) {
      light_step();
      for (int v : ins) chain(v);
      add_work(Work{"Stage", n.id});
      add_store(Stored{op.values[0], "staged", "", op.sources[0]});
      return;
    }
    const std::optional<int> i = open_index();
    size_t on_tile = 0;
    for (int v : ins) {
      const Avail a = avail_of(v);
      if (a.k == Avail::Tile && i && a.a == *i) ++on_tile;
    }
    if (on_tile && pointwise(op.kind) && on_tile == ins.size()) {
      add_work(Work{"Epilogue", n.id});
    } else {
      light_step();
      for (int v : ins) chain(v);
      add_work(Work{"Effect", n.id});
    }
    if (open_) open_->writes.insert(op.sources[0]);
  }

  void outputs() {
    for (const Output& o : p_.outputs) {
      const Avail::K k = avail_of(o.value).k;
      if (k == Avail::Virtual || k == Avail::Partials) materialize(o.value);
    }
  }

  // -- the steps as the plan gives them
  Step finish(const StepB& sb) const {
    Step s;
    s.index = sb.index;
    s.name = name(sb);
    s.work = sb.work;
    std::stable_sort(s.work.begin(), s.work.end(), [](const Work& a, const Work& b) { return a.node < b.node; });
    s.stores = sb.stores;
    std::stable_sort(s.stores.begin(), s.stores.end(),
                     [](const Stored& a, const Stored& b) { return a.value < b.value; });
    s.reads = reads_of(sb);
    std::stable_sort(s.reads.begin(), s.reads.end(),
                     [](const Stored& a, const Stored& b) { return a.value < b.value; });
    for (const Work& w : sb.work)
      for (int c : caches(w))
        if (!contains(s.caches, c)) s.caches.push_back(c);
    return s;
  }

  std::vector<int> caches(const Work& w) const {
    if (w.kind == "Stage" || w.kind == "Combine") return {};
    const Op& op = op_of(w.node);
    if (op.kind == "KvStore") return {op.sources[0]};
    if (op.kind == "Attend") return {op.sources[0], op.sources[1]};
    return {};
  }

  std::vector<Stored> reads_of(const StepB& sb) const {
    std::set<int> in_step;
    for (const Work& w : sb.work)
      if (w.kind == "Combine" || w.kind == "Anchor" || w.kind == "Recompute" || w.kind == "Epilogue")
        for (int v : outs_of(w.node)) in_step.insert(v);
    auto wanted = [](const Work& w, const Stored& st) {
      return w.kind == "Combine" ? st.form == "partials" : st.form == "elements";
    };
    auto stages_read = [&](const Work& w) -> std::vector<int> {
      const Op& op = op_of(w.node);
      if (w.kind == "Anchor" && op.kind == "Attend") {
        std::vector<int> r = {op.sources[0]};
        if (op.sources[1] != op.sources[0]) r.push_back(op.sources[1]);
        return r;
      }
      if (w.kind == "Land" && op.kind == "KvStore") return {op.sources[0]};
      return {};
    };
    auto reads_of_work = [&](const Work& w) -> std::vector<int> {
      if (w.kind == "Combine") return outs_of(w.node);
      if (w.kind == "Land") return {};
      std::vector<int> r;
      for (int v : op_of(w.node).values)
        if (!in_step.count(v)) r.push_back(v);
      return r;
    };
    std::vector<Stored> out;
    for (const Work& w : sb.work)
      for (int v : reads_of_work(w))
        for (const Stored& st : stored_before(sb.index, v))
          if (wanted(w, st) && !contains(out, st)) out.push_back(st);
    for (const Work& w : sb.work)
      for (int c : stages_read(w))
        for (const Stored& st : staged_before(sb.index, c))
          if (!contains(out, st)) out.push_back(st);
    return out;
  }

  std::vector<Stored> stored_before(int s, int v) const {
    std::vector<Stored> out;
    for (const StepB& sb : closed_)
      if (sb.index < s)
        for (const Stored& st : sb.stores)
          if (st.value == v) out.push_back(st);
    const Node* n = producer(v);
    if (n && n->op.kind == "Input") out.push_back(elements(v, type_of(v)));
    return out;
  }

  std::vector<Stored> staged_before(int s, int c) const {
    std::vector<Stored> out;
    for (const StepB& sb : closed_)
      if (sb.index < s)
        for (const Stored& st : sb.stores)
          if (st.form == "staged" && st.cache == c) out.push_back(st);
    return out;
  }

  std::string name(const StepB& sb) const {
    const std::string pre = "s" + std::to_string(sb.index) + "_";
    std::vector<std::string> words;
    for (const Work& w : sb.work)
      if (w.kind == "Anchor") {
        const std::string word = op_of(w.node).kind == "Attend" ? "attend" : "gemv";
        if (!contains(words, word)) words.push_back(word);
      }
    if (!words.empty()) {
      std::string s = pre;
      for (size_t i = 0; i < words.size(); ++i) s += (i ? "_" : "") + words[i];
      return s;
    }
    for (const Work& w : sb.work) {
      if (w.kind == "Effect" || w.kind == "Stage") return pre + "store";
      if (w.kind == "Combine") return pre + "combine";
      if (w.kind == "Recompute")
        for (const Stored& st : sb.stores)
          if (st.form == "elements") return pre + p_.values[st.value].name;
    }
    for (const Work& w : sb.work)
      if (w.kind == "Land") return pre + "land";
    return pre + "light";
  }

  const PlanOptions o_;
  const Program& p_;
  std::map<int, Avail> avail_;
  std::vector<StepB> closed_;
  std::optional<StepB> open_;
  int next_ = 0;
  std::vector<std::tuple<int, int, int>> landing_;  // (step, store node, cache)
  std::map<int, int> producer_;
  std::map<int, std::vector<int>> consumers_;
  std::set<int> output_values_;
  std::set<int> staged_;
};

}  // namespace

Plan plan(const PlanOptions& o, const Program& p) { return Planner(o, p).run(); }

bool is_step_name(const std::string& t) {
  if (t.empty() || t[0] != 's') return false;
  size_t i = 1;
  while (i < t.size() && t[i] >= '0' && t[i] <= '9') ++i;
  return i > 1 && i + 1 < t.size() && t[i] == '_';
}

std::string render_plan(const Plan& pl) {
  const Program& p = pl.program;
  auto stored = [&](const Stored& st) -> std::string {
    const std::string name = p.values[st.value].name;
    if (st.form == "elements") return name + " " + st.type;
    if (st.form == "partials") return name + " partials";
    return name + " staged for " + p.sources[st.cache].name;
  };
  std::string out = "plan " + p.name + "\n";
  for (const Step& s : pl.steps) {
    out += "  step " + s.name + "\n";
    for (const Work& w : s.work) {
      std::string k = w.kind;
      std::transform(k.begin(), k.end(), k.begin(), ::tolower);
      out += "    " + k + " " + p.nodes[w.node].name + "\n";
    }
    for (const Stored& st : s.reads) out += "    reads " + stored(st) + "\n";
    for (const Stored& st : s.stores) out += "    stores " + stored(st) + "\n";
  }
  return out;
}

}  // namespace fkh
