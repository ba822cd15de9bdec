// A plan's steps as launches of the CUDA target's kernel table (the step
// shapes of the Llama-shaped programs), and the whole decode step of the
// Llama engine: the embedding, every layer, the head, then the engine's
// rewrites (the SiLU-gate on interleaved gate/up tiles, tensor parallelism
// over peer memory or NCCL, the decode step's KV store folded into its
// attention) and the split-K of each GEMV.
#include <algorithm>

#include "fkh.h"

namespace fkh {

double Launch::param(const std::string& n) const {
  for (const auto& [k, v] : params)
    if (k == n) return v;
  throw Refusal(kernel + ": no parameter " + n + ".");
}
bool Launch::has(const std::string& n) const {
  for (const auto& kv : params)
    if (kv.first == n) return true;
  return false;
}
void Launch::set(const std::string& n, double v) {
  for (auto& kv : params)
    if (kv.first == n) {
      kv.second = v;
      return;
    }
  params.emplace_back(n, v);
}

namespace {

std::string work_text(const Program& p, const Step& step) {
  std::string s;
  for (size_t i = 0; i < step.work.size(); ++i) {
    std::string k = step.work[i].kind;
    std::transform(k.begin(), k.end(), k.begin(), ::tolower);
    s += (i ? "; " : "") + k + " " + p.nodes[step.work[i].node].name;
  }
  return s;
}

template <typename M>
typename M::mapped_type at(const M& m, const std::string& key, const std::string& what) {
  auto it = m.find(key);
  if (it == m.end()) throw Refusal(what + ": nothing is bound to " + key + ".");
  return it->second;
}

std::string weight_suffix(const Step& step, const std::string& t) { return weight_form(t, step.name); }

std::string cache_suffix(const Step& step, const std::string& elem) { return cache_form(elem, step.name); }

}  // namespace

std::string weight_form(const std::string& t, const std::string& what) {
  if (t == "f32") return "";
  if (t == "bf16") return "_wbf16";
  if (t == "f16") return "_wf16";
  throw Refusal(what + ": no kernel reads " + t + " weights.");
}

std::string cache_form(const std::string& t, const std::string& what) {
  if (t == "f32") return "";
  if (t == "bf16") return "_kvbf16";
  if (t == "f16") return "_kvf16";
  throw Refusal(what + ": no kernel reads " + t + " caches.");
}

std::pair<std::string, std::string> kernel_form(const std::string& kernel) {
  for (const char* suffix : {"_wbf16", "_wf16", "_kvbf16", "_kvf16"}) {
    const size_t n = std::char_traits<char>::length(suffix);
    if (kernel.size() > n && kernel.compare(kernel.size() - n, n, suffix) == 0)
      return {kernel.substr(0, kernel.size() - n), suffix};
  }
  return {kernel, ""};
}

Launch lower_step(const Program& p, const Step& step, const Binding& b, uint64_t cos_t, uint64_t sin_t,
                  const AttnBufs& attn) {
  std::vector<const Node*> anchors, epilogues, effects;
  std::map<int, const Node*> recomputed;
  std::vector<std::string> kinds;
  for (const Work& w : step.work) {
    const Node* n = &p.nodes[w.node];
    kinds.push_back(w.kind);
    if (w.kind == "Anchor") anchors.push_back(n);
    if (w.kind == "Recompute") recomputed[n->outputs[0]] = n;
    if (w.kind == "Epilogue") epilogues.push_back(n);
    if (w.kind == "Effect") effects.push_back(n);
  }
  auto vname = [&](int v) { return p.values[v].name; };
  auto stored = [&](int v) -> View {
    auto it = b.values.find(vname(v));
    if (it == b.values.end()) throw Refusal(step.name + ": " + vname(v) + " is not stored where the step reads it.");
    return it->second;
  };
  auto src_name = [&](int s) { return p.sources[s].name; };
  auto recomputed_of = [&](int v) -> const Node* {
    auto it = recomputed.find(v);
    return it == recomputed.end() ? nullptr : it->second;
  };
  const double m = (double)b.m;

  bool all_linear = !anchors.empty();
  for (const Node* n : anchors)
    if (n->op.kind != "Linear") all_linear = false;
  if (all_linear) {
    const int x_id = anchors[0]->op.values[0];
    for (const Node* n : anchors)
      if (n->op.values[0] != x_id)
        throw Refusal(step.name + ": anchors of different inputs: " + work_text(p, step));
    const std::string& wtype = p.sources[anchors[0]->op.sources[0]].kind.type;
    for (const Node* n : anchors)
      if (p.sources[n->op.sources[0]].kind.type != wtype)
        throw Refusal(step.name + ": its anchors' weights differ in type.");
    const std::string wt = weight_suffix(step, wtype);
    const uint64_t esz = wt.empty() ? 4 : 2;
    const uint64_t w0 = at(b.weights, src_name(anchors[0]->op.sources[0]), step.name);
    uint64_t n_total = 0;
    const uint64_t k = p.sources[anchors[0]->op.sources[0]].kind.dims[1];
    uint64_t addr = w0;
    for (const Node* n : anchors) {  // the anchors' weights must lie adjacent
      const Source& w = p.sources[n->op.sources[0]];
      if (at(b.weights, w.name, step.name) != addr)
        throw Refusal(step.name + ": the weights of its anchors are not adjacent.");
      addr += esz * w.kind.dims[0] * k;
      n_total += w.kind.dims[0];
    }
    View y;
    int r_id = -1;
    if (!epilogues.empty()) {
      const Node* ep = epilogues[0];
      if (epilogues.size() != 1 || ep->op.kind != "Add" || anchors.size() != 1)
        throw Refusal(step.name + ": epilogue " + ep->name + " is not one residual add.");
      const int tile = anchors[0]->outputs[0];
      r_id = ep->op.values[1] == tile ? ep->op.values[0] : ep->op.values[1];
      y = stored(ep->outputs[0]);
    } else {
      y = at(b.values, vname(anchors[0]->outputs[0]), step.name);
      for (size_t i = 1; i < anchors.size(); ++i) {  // adjacent columns
        const View nxt = at(b.values, vname(anchors[i]->outputs[0]), step.name);
        if (nxt.base != y.base) throw Refusal(step.name + ": its anchors' outputs are not adjacent.");
      }
    }
    Launch L;
    L.params = {{"n", (double)n_total}, {"k", (double)k}, {"m", m}, {"split", 1.0}, {"ldy", (double)y.ld}};
    const Node* xn = recomputed_of(x_id);
    if (!xn) {
      const View x = stored(x_id);
      L.set("ldx", (double)x.ld);
      if (!epilogues.empty()) {
        const View r = stored(r_id);
        L.kernel = "gemv_add" + wt;
        L.set("ldr", (double)r.ld);
        L.bufs = {w0, x.ptr(), r.ptr(), y.ptr()};
        return L;
      }
      L.kernel = "gemv" + wt;
      L.bufs = {w0, x.ptr(), y.ptr()};
      return L;
    }
    if (xn->op.kind == "RmsNorm" && epilogues.empty()) {
      const View x = stored(xn->op.values[0]);
      if (p.sources[xn->op.sources[0]].kind.type != wtype)
        throw Refusal(step.name + ": the norm's gain and the weights differ in type.");
      const uint64_t gamma = at(b.weights, src_name(xn->op.sources[0]), step.name);
      L.kernel = "gemv_rmsnorm" + wt;
      L.set("ldx", (double)x.ld);
      L.set("eps", xn->op.eps);
      L.set("factor", xn->op.factor);
      L.bufs = {w0, x.ptr(), gamma, y.ptr()};
      return L;
    }
    if (xn->op.kind == "SiluMul") {
      const View g = stored(xn->op.values[0]), u = stored(xn->op.values[1]);
      if (g.base != u.base || g.ld != u.ld) throw Refusal(step.name + ": SiLU-gate's halves are not one row.");
      L.set("ldx", (double)g.ld);
      L.set("up_off", (double)(u.col - g.col));
      if (!epilogues.empty()) {
        const View r = stored(r_id);
        L.kernel = "gemv_silu_add" + wt;
        L.set("ldr", (double)r.ld);
        L.bufs = {w0, g.ptr(), r.ptr(), y.ptr()};
        return L;
      }
      L.kernel = "gemv_silu" + wt;
      L.bufs = {w0, g.ptr(), y.ptr()};
      return L;
    }
    throw Refusal(step.name + ": no kernel runs " + work_text(p, step));
  }

  if (anchors.size() == 1 && anchors[0]->op.kind == "Attend") {
    const Node* att = anchors[0];
    const AttnSpec& spec = att->op.attn;
    const Node* qn = recomputed_of(att->op.values[0]);
    if (!qn || qn->op.kind != "Rope") throw Refusal(step.name + ": attention without its query's rotation.");
    const View q = stored(qn->op.values[0]);
    const Source& kc = p.sources[att->op.sources[0]];
    Launch L;
    if (!kc.kind.ring) {  // through the rows' block tables
      L.kernel = "attend_split_paged" + cache_suffix(step, kc.kind.elem);
      L.params = {{"m", m},
                  {"heads", (double)spec.heads},
                  {"kv_heads", (double)spec.kv_heads},
                  {"d", (double)spec.head_dim},
                  {"block_size", (double)kc.kind.pg.block_size},
                  {"table_len", (double)p.sources[att->op.sources[3]].kind.count},
                  {"blocks", (double)kc.kind.pg.blocks},
                  {"rotated", (double)qn->op.rope.rotated},
                  {"chunk", (double)attn.chunk},
                  {"max_splits", (double)attn.max_splits},
                  {"ldq", (double)q.ld},
                  {"q_off", (double)q.col},
                  {"scale", spec.scale}};
    } else {
      L.kernel = "attend_split" + cache_suffix(step, kc.kind.elem);
      L.params = {{"m", m},
                  {"heads", (double)spec.heads},
                  {"kv_heads", (double)spec.kv_heads},
                  {"d", (double)spec.head_dim},
                  {"length", (double)kc.kind.r.length},
                  {"rotated", (double)qn->op.rope.rotated},
                  {"chunk", (double)attn.chunk},
                  {"max_splits", (double)attn.max_splits},
                  {"ldq", (double)q.ld},
                  {"q_off", (double)q.col},
                  {"scale", spec.scale}};
    }
    const uint64_t kaddr = at(b.caches, kc.name, step.name), vaddr = at(b.caches, src_name(att->op.sources[1]), step.name);
    L.bufs = {q.base, cos_t, sin_t, at(b.ints, src_name(att->op.sources[2]), step.name),
              at(b.ints, src_name(att->op.sources[3]), step.name)};
    // A ring's caches are buffers before the partials; a paged cache's
    // tables of block addresses come after every buffer.
    if (kc.kind.ring) L.bufs.insert(L.bufs.end(), {kaddr, vaddr});
    L.bufs.insert(L.bufs.end(), {attn.partials[0], attn.partials[1], attn.partials[2]});
    if (!kc.kind.ring) L.bufs.insert(L.bufs.end(), {kaddr, vaddr});
    return L;
  }

  if (kinds == std::vector<std::string>{"Combine"}) {
    const Node* att = &p.nodes[step.work[0].node];
    const AttnSpec& spec = att->op.attn;
    const View out = stored(att->outputs[0]);
    Launch L;
    L.kernel = "attend_combine";
    L.params = {{"m", m},
                {"heads", (double)spec.heads},
                {"d", (double)spec.head_dim},
                {"chunk", (double)attn.chunk},
                {"max_splits", (double)attn.max_splits},
                {"ldo", (double)out.ld}};
    L.bufs = {attn.partials[0], attn.partials[1], attn.partials[2],
              at(b.ints, src_name(att->op.sources[2]), step.name), out.ptr()};
    return L;
  }

  bool all_stores = !effects.empty();
  for (const Node* n : effects)
    if (n->op.kind != "KvStore") all_stores = false;
  if (all_stores && effects.size() == 2) {
    const Node* sk = effects[0];
    const Node* sv = effects[1];
    const Node* kn = recomputed_of(sk->op.values[0]);
    if (!kn || kn->op.kind != "Rope") throw Refusal(step.name + ": keys stored without their rotation.");
    const View kview = stored(kn->op.values[0]), vview = stored(sv->op.values[0]);
    if (kview.base != vview.base) throw Refusal(step.name + ": keys and values are not one row.");
    const Source& kc = p.sources[sk->op.sources[0]];
    Launch L;
    if (!kc.kind.ring) {  // through the rows' block tables
      L.kernel = "kv_store_paged" + cache_suffix(step, kc.kind.elem);
      L.params = {{"m", m},
                  {"kv_heads", (double)kc.kind.pg.kv_heads},
                  {"d", (double)kc.kind.pg.head_dim},
                  {"block_size", (double)kc.kind.pg.block_size},
                  {"table_len", (double)p.sources[sk->op.sources[2]].kind.count},
                  {"blocks", (double)kc.kind.pg.blocks},
                  {"rotated", (double)kn->op.rope.rotated},
                  {"ldq", (double)kview.ld},
                  {"k_off", (double)kview.col},
                  {"v_off", (double)vview.col}};
    } else {
      L.kernel = "kv_store_ring" + cache_suffix(step, kc.kind.elem);
      L.params = {{"m", m},
                  {"kv_heads", (double)kc.kind.r.kv_heads},
                  {"d", (double)kc.kind.r.head_dim},
                  {"length", (double)kc.kind.r.length},
                  {"rotated", (double)kn->op.rope.rotated},
                  {"ldq", (double)kview.ld},
                  {"k_off", (double)kview.col},
                  {"v_off", (double)vview.col}};
    }
    L.bufs = {kview.base,
              cos_t,
              sin_t,
              at(b.ints, src_name(sk->op.sources[1]), step.name),
              at(b.ints, src_name(sk->op.sources[2]), step.name),
              at(b.caches, kc.name, step.name),
              at(b.caches, src_name(sv->op.sources[0]), step.name)};
    return L;
  }

  if (kinds == std::vector<std::string>{"Recompute"}) {
    const Node* n = &p.nodes[step.work[0].node];
    if (n->op.kind == "Gather") {
      const Source& table = p.sources[n->op.sources[0]];
      const Source& tok = p.sources[n->op.sources[1]];
      const View y = stored(n->outputs[0]);
      Launch L;
      L.kernel = "gather" + weight_suffix(step, table.kind.type);
      L.params = {{"width", (double)table.kind.dims[1]}, {"m", m}, {"factor", n->op.f}};
      L.bufs = {at(b.weights, table.name, step.name), at(b.ints, tok.name, step.name), y.ptr()};
      return L;
    }
    if (n->op.kind == "ArgMax") {
      const View x = stored(n->op.values[0]);
      const View y = stored(n->outputs[0]);
      Launch L;
      L.kernel = "argmax";
      L.params = {{"m", m}, {"n", (double)x.width}, {"ldx", (double)x.ld}};
      L.bufs = {x.ptr(), y.ptr()};
      return L;
    }
  }
  throw Refusal(step.name + ": no kernel runs " + work_text(p, step));
}

std::vector<Launch> lower_steps(const Program& p, const Step& step, const Binding& b, uint64_t cos_t, uint64_t sin_t,
                                const AttnBufs& attn) {
  std::vector<std::pair<std::string, std::string>> kinds;
  for (const Work& w : step.work) kinds.emplace_back(w.kind, p.nodes[w.node].op.kind);
  std::sort(kinds.begin(), kinds.end());
  auto node = [&](const std::string& kind) -> const Node& {
    for (const Work& w : step.work)
      if (p.nodes[w.node].op.kind == kind) return p.nodes[w.node];
    throw Refusal(step.name + ": no " + kind + ".");
  };
  auto stored = [&](int v) -> View {
    auto it = b.values.find(p.values[v].name);
    if (it == b.values.end())
      throw Refusal(step.name + ": " + p.values[v].name + " is not stored where the step reads it.");
    return it->second;
  };
  auto weight = [&](const std::string& name) -> uint64_t {
    auto it = b.weights.find(name);
    if (it == b.weights.end()) throw Refusal(step.name + ": nothing is bound to " + name + ".");
    return it->second;
  };
  auto make = [](const std::string& kernel, std::vector<std::pair<std::string, double>> params,
                 std::vector<uint64_t> bufs) {
    Launch L;
    L.kernel = kernel;
    L.params = std::move(params);
    L.bufs = std::move(bufs);
    return L;
  };
  using KP = std::vector<std::pair<std::string, std::string>>;
  const double m = (double)b.m;
  bool norm_stored = false;
  if (kinds == KP{{"Anchor", "Linear"}, {"Recompute", "RmsNorm"}}) {
    const int v = node("RmsNorm").outputs[0];
    for (const Stored& st : step.stores)
      if (st.value == v) norm_stored = true;
  }
  if (norm_stored) {  // the norm's row is stored for a later step: the rows, then their GEMV
    const Node& nn = node("RmsNorm");
    const Node& lin = node("Linear");
    const View x = stored(nn.op.values[0]), y = stored(nn.outputs[0]), out = stored(lin.outputs[0]);
    if (x.ld != x.width || y.ld != y.width) throw Refusal(step.name + ": a stored norm of rows that are not whole.");
    const Source& w = p.sources[lin.op.sources[0]];
    const std::string wt = weight_form(w.kind.type, step.name);
    return {make("rmsnorm_rows" + wt,
                 {{"rows", m}, {"h", (double)x.width}, {"eps", nn.op.eps}, {"factor", nn.op.factor}},
                 {x.ptr(), weight(p.sources[nn.op.sources[0]].name), y.ptr()}),
            make("gemv" + wt,
                 {{"n", (double)w.kind.dims[0]}, {"k", (double)w.kind.dims[1]}, {"m", m}, {"split", 1.0},
                  {"ldx", (double)y.ld}, {"ldy", (double)out.ld}},
                 {weight(w.name), y.ptr(), out.ptr()})};
  }
  // Routed experts: the route, the GELU gate and the routed GEMV, each a
  // step of its own (the gated plan's, Plan.hs:246-251, with or without
  // stored gelus) or the route or the gate recomputed in the GEMV's step.
  const bool lone_route = kinds == KP{{"Recompute", "Route"}};
  const bool lone_gate = kinds == KP{{"Recompute", "GatedGelu"}};
  const bool lone_routed = kinds == KP{{"Anchor", "LinearRouted"}};
  const bool routed_route = kinds == KP{{"Anchor", "LinearRouted"}, {"Recompute", "Route"}};
  const bool routed_gate = kinds == KP{{"Anchor", "LinearRouted"}, {"Recompute", "GatedGelu"}};
  if (lone_route || lone_gate || lone_routed || routed_route || routed_gate) {
    std::vector<Launch> out;
    if (lone_route || routed_route) {
      const Node& r = node("Route");
      const View logits = stored(r.op.values[0]), ids = stored(r.outputs[0]), ws = stored(r.outputs[1]);
      const std::vector<std::pair<std::string, double>> params = {
          {"m", m}, {"n", (double)logits.width}, {"k", (double)ids.width}, {"ldx", (double)logits.ld}};
      if (r.op.route.expert_scale) {  // each expert's weight times its scale
        const Source& sc = p.sources[*r.op.route.expert_scale];
        out.push_back(make("route_topk_scaled" + weight_form(sc.kind.type, step.name), params,
                           {logits.ptr(), weight(sc.name), ids.ptr(), ws.ptr()}));
      } else {
        out.push_back(make("route_topk", params, {logits.ptr(), ids.ptr(), ws.ptr()}));
      }
    }
    if (lone_gate || routed_gate) {
      const Node& g = node("GatedGelu");
      const View gu = stored(g.op.values[0]), x = stored(g.outputs[0]);
      const uint64_t f = p.values[g.outputs[0]].shape.segment;
      if (gu.ld != gu.width || x.ld != x.width) throw Refusal(step.name + ": a gate of rows that are not whole.");
      if (f == 0 || x.width % f != 0) throw Refusal(step.name + ": a gate whose rows are not whole segments.");
      out.push_back(make("gated_gelu", {{"segments", m * (double)(x.width / f)}, {"f", (double)f}},
                         {gu.ptr(), x.ptr()}));
    }
    if (lone_routed || routed_route || routed_gate) {
      const Node& lr = node("LinearRouted");
      const Source& t = p.sources[lr.op.sources[0]];
      const std::string tsuf = weight_form(t.kind.type, step.name);
      const uint64_t n = t.kind.dims[0], kk = t.kind.dims[1];
      const View ids = stored(lr.op.values[0]), x = stored(lr.op.values[1]), y = stored(lr.outputs[0]);
      out.push_back(make("gemv_routed" + tsuf,
                         {{"entries", (double)t.kind.entries},
                          {"n", (double)n},
                          {"kk", (double)kk},
                          {"m", m},
                          {"k", (double)ids.width},
                          {"split", 1.0},
                          {"ldx", (double)x.ld},
                          {"ldy", (double)y.ld},
                          {"per_rank", x.width != kk ? 1.0 : 0.0}},
                         {weight(t.name), ids.ptr(), x.ptr(), y.ptr()}));
    }
    return out;
  }
  if (kinds == KP{{"Recompute", "Add"}, {"Recompute", "CombineRanks"}}) {
    const Node& c = node("CombineRanks");
    const Node& a = node("Add");
    const View ws = stored(c.op.values[0]), segs = stored(c.op.values[1]), y = stored(a.outputs[0]);
    const int r_id = a.op.values[1] == c.outputs[0] ? a.op.values[0] : a.op.values[1];
    const View r = stored(r_id);
    for (const View* v : {&ws, &segs, &y, &r})
      if (v->ld != v->width) throw Refusal(step.name + ": a combine of rows that are not whole.");
    return {make("combine_ranks_add", {{"m", m}, {"k", (double)ws.width}, {"d", (double)y.width}},
                 {r.ptr(), ws.ptr(), segs.ptr(), y.ptr()})};
  }
  return {lower_step(p, step, b, cos_t, sin_t, attn)};
}

uint64_t split_for(uint64_t n_rows, uint64_t k, uint64_t sms) {
  for (uint64_t s : {1, 2, 4, 8})
    if (n_rows * s >= sms * 48 || k / s < 1024) return s;
  return 8;
}

namespace {

// The [gate; up] step followed by the down step that recomputes
// silu(gate) * up from their stored rows becomes the [gate; up] GEMV on
// interleaved rows with the SiLU-gate epilogue, storing mlp_act, and the
// down GEMV reading it.
void silu_on_tiles(std::vector<Launch>& out, uint64_t f, uint64_t gu, uint64_t act) {
  for (size_t i = 0; i + 1 < out.size(); ++i) {
    Launch& a = out[i];
    Launch& b = out[i + 1];
    const auto [ab, asuf] = kernel_form(a.kernel);
    const auto [bb, bsuf] = kernel_form(b.kernel);
    if (ab == "gemv_rmsnorm" && a.bufs[3] == gu && a.param("n") == 2.0 * f &&
        (bb == "gemv_silu" || bb == "gemv_silu_add") && b.bufs[1] == gu && b.param("up_off") == f) {
      Launch na;
      na.kernel = "gemv_rmsnorm_silu" + asuf;
      na.params = a.params;
      na.set("ldy", (double)f);
      na.bufs = {a.bufs[0], a.bufs[1], a.bufs[2], act};
      Launch nb;
      for (const auto& kv : b.params)
        if (kv.first != "up_off") nb.params.push_back(kv);
      nb.set("ldx", (double)f);
      if (bb == "gemv_silu_add") {
        nb.kernel = "gemv_add" + bsuf;
        nb.bufs = {b.bufs[0], act, b.bufs[2], b.bufs[3]};
      } else {
        nb.kernel = "gemv" + bsuf;
        nb.bufs = {b.bufs[0], act, b.bufs[2]};
      }
      a = na;
      b = nb;
    }
  }
}

// Over NVLink peer memory: a row-parallel projection scatters its partial
// rows into every rank's exchange buffer (o: 0, down: 1) and leaves its
// residual epilogue to the next GEMV, whose prologue adds the ranks'
// partials in rank order to the residual, stores the new residual row and
// normalizes it; the greedy candidates travel the same way.
std::vector<Launch> tensor_parallel_peers(const std::vector<Launch>& in, const LlamaLaunchDesc& d,
                                          uint64_t vocab_local) {
  std::vector<Launch> out;
  struct Pending {
    int buf;
    uint64_t r, y;
    bool live;
  };
  std::optional<Pending> pending;
  const uint64_t dm = d.full.d_model;
  for (const Launch& L : in) {
    const auto [base, suf] = kernel_form(L.kernel);
    if (base == "gemv_add") {
      const int xbuf = !pending || pending->buf == 1 ? 0 : 1;
      if (L.param("ldy") != dm || L.param("ldr") != dm)
        throw Refusal("a row-parallel output that is not a whole row.");
      Launch s;
      s.kernel = "gemv_scatter" + suf;
      s.params = {{"n", L.param("n")}, {"k", L.param("k")}, {"m", L.param("m")}, {"split", L.param("split")},
                  {"ldx", L.param("ldx")}, {"xbuf", (double)xbuf}};
      s.bufs = {L.bufs[0], L.bufs[1]};
      out.push_back(s);
      pending = Pending{xbuf, L.bufs[2], L.bufs[3], true};
    } else if (pending && pending->live && (base == "gemv_rmsnorm" || base == "gemv_rmsnorm_silu") &&
               L.bufs[1] == pending->y) {
      Launch r;
      r.kernel = (base == "gemv_rmsnorm_silu" ? "gemv_reduce_rmsnorm_silu" : "gemv_reduce_rmsnorm") + suf;
      for (const auto& kv : L.params)
        if (kv.first != "ldx") r.params.push_back(kv);
      r.set("ldr", (double)dm);
      r.set("xbuf", (double)pending->buf);
      r.bufs = {L.bufs[0], pending->r, L.bufs[2], pending->y, L.bufs[3]};
      out.push_back(r);
      pending->live = false;  // consumed; the buffer alternates on
    } else if (L.kernel == "argmax") {
      Launch s;
      s.kernel = "argmax_scatter";
      s.params = L.params;
      s.set("offset", (double)(d.rank * vocab_local));
      s.bufs = {L.bufs[0]};
      out.push_back(s);
      Launch g;
      g.kernel = "argmax_gather_pick";
      g.params = {{"m", (double)d.batch}};
      g.bufs = {L.bufs[1]};
      out.push_back(g);
    } else {
      out.push_back(L);
    }
  }
  return out;
}

// With NCCL: the row-parallel projections' residual epilogues move after the
// allreduce of their partial sums, the experts' outputs (each rank's share
// of every expert's FFN) are summed before they are combined, and the greedy
// pick gathers the shards' candidates.
std::vector<Launch> tensor_parallel_nccl(const std::vector<Launch>& in, const LlamaLaunchDesc& d,
                                         uint64_t vocab_local) {
  std::vector<Launch> out;
  const uint64_t dm = d.full.d_model, m = d.batch;
  for (const Launch& L : in) {
    const auto [base, suf] = kernel_form(L.kernel);
    if (base == "gemv_add" || base == "gemv_silu_add") {
      if (L.param("ldy") != dm || L.param("ldr") != dm)
        throw Refusal("a row-parallel output that is not a whole row.");
      Launch g;
      g.kernel = base.substr(0, base.size() - 4) + suf;
      for (const auto& kv : L.params)
        if (kv.first != "ldr") g.params.push_back(kv);
      g.bufs = {L.bufs[0], L.bufs[1], d.partial};
      out.push_back(g);
      Launch ar;
      ar.kernel = "__allreduce__";
      ar.params = {{"count", (double)(m * dm)}};
      ar.bufs = {d.partial};
      out.push_back(ar);
      Launch add;
      add.kernel = "add";
      add.params = {{"n", (double)(m * dm)}};
      add.bufs = {L.bufs[2], d.partial, L.bufs[3]};
      out.push_back(add);
    } else if (L.kernel == "combine_ranks_add") {
      Launch ar;
      ar.kernel = "__allreduce__";
      ar.params = {{"count", L.param("m") * L.param("k") * L.param("d")}};
      ar.bufs = {L.bufs[2]};
      out.push_back(ar);
      out.push_back(L);
    } else if (L.kernel == "argmax") {
      Launch a;
      a.kernel = "argmax_pairs";
      a.params = L.params;
      a.set("offset", (double)(d.rank * vocab_local));
      a.bufs = {L.bufs[0], d.pairs};
      out.push_back(a);
      Launch g;
      g.kernel = "__allgather__";
      g.params = {{"count", (double)(2 * m)}};
      g.bufs = {d.pairs, d.pairs_all};
      out.push_back(g);
      Launch p;
      p.kernel = "argmax_pick";
      p.params = {{"shards", (double)d.world}, {"m", (double)m}};
      p.bufs = {d.pairs_all, L.bufs[1]};
      out.push_back(p);
    } else {
      out.push_back(L);
    }
  }
  return out;
}

// Each layer's KV store and split attention, when they bind the same row of
// q/k/v, positions, slots and caches, become one attend_decode launch.
// A paged cache's pair likewise becomes attend_decode_paged (the engine
// holds every block-table entry distinct).
std::vector<Launch> fuse_attention(const std::vector<Launch>& in) {
  std::vector<Launch> out;
  for (size_t i = 0; i < in.size(); ++i) {
    const auto kvf = kernel_form(in[i].kernel);
    const auto atf = i + 1 < in.size() ? kernel_form(in[i + 1].kernel) : std::pair<std::string, std::string>{};
    const bool ring = kvf.first == "kv_store_ring" && atf.first == "attend_split";
    const bool paged = kvf.first == "kv_store_paged" && atf.first == "attend_split_paged";
    if (i + 1 < in.size() && (ring || paged) && kvf.second == atf.second) {
      const Launch& kv = in[i];
      const Launch& at = in[i + 1];
      // The same q/k/v rows, positions, slots (block tables) and caches: a
      // ring's caches are the attention's buffers 5 and 6, a paged cache's
      // address tables its bindings 8 and 9 (after the partials).
      bool same = kv.bufs[0] == at.bufs[0] && std::equal(kv.bufs.begin() + 3, kv.bufs.begin() + 5, at.bufs.begin() + 3) &&
                  std::equal(kv.bufs.begin() + 5, kv.bufs.begin() + 7, at.bufs.begin() + (ring ? 5 : 8));
      const std::vector<const char*> keys =
          ring ? std::vector<const char*>{"ldq", "rotated", "d", "kv_heads", "length"}
               : std::vector<const char*>{"ldq", "rotated", "d", "kv_heads", "block_size", "table_len", "blocks"};
      for (const char* k : keys)
        if (kv.param(k) != at.param(k)) same = false;
      if (same) {
        Launch f;
        f.kernel = (ring ? "attend_decode" : "attend_decode_paged") + kvf.second;
        f.params = at.params;
        f.set("k_off", kv.param("k_off"));
        f.set("v_off", kv.param("v_off"));
        f.bufs = at.bufs;
        out.push_back(f);
        ++i;
        continue;
      }
    }
    out.push_back(in[i]);
  }
  return out;
}

}  // namespace

LlamaShape shard_of(const LlamaLaunchDesc& d) {
  const LlamaShape& full = d.full;
  if (d.world == 0 || full.heads % d.world || full.kv_heads % d.world || full.ffn % d.world ||
      full.vocab % d.world)
    throw Refusal("the model does not split over " + std::to_string(d.world) + " ranks.");
  LlamaShape s = full;  // this rank's shard
  s.heads = full.heads / d.world;
  s.kv_heads = full.kv_heads / d.world;
  s.ffn = full.ffn / d.world;
  return s;
}

namespace {

// A layer's weights in the arena, in order: q k v o, the dense FFN's gate
// up down (or the router and the experts' gate/up and down tables), the
// two norms.
// A layer's weights in the arena, in order: (name, elements).
std::vector<std::pair<const char*, uint64_t>> layer_layout(const LlamaShape& s) {
  const uint64_t dm = s.d_model, qw = s.q_width(), kvw = s.kv_width(), f = s.ffn, e = s.experts;
  std::vector<std::pair<const char*, uint64_t>> out = {
      {"q_proj", qw * dm}, {"k_proj", kvw * dm}, {"v_proj", kvw * dm}, {"o_proj", dm * qw}};
  if (e) {
    out.push_back({"router", e * dm});
    if (s.expert_scale) out.push_back({"expert_scale", e});
    out.insert(out.end(), {{"experts_gate_up", e * 2 * f * dm}, {"experts_down", e * dm * f}});
  } else {
    out.insert(out.end(), {{"gate_proj", f * dm}, {"up_proj", f * dm}, {"down_proj", dm * f}});
  }
  out.insert(out.end(), {{"attn_norm", dm}, {"mlp_norm", dm}});
  return out;
}

}  // namespace

uint64_t layer_elems(const LlamaShape& s) {
  uint64_t t = 0;
  for (const auto& [name, n] : layer_layout(s)) t += n;
  return t;
}

std::map<std::string, uint64_t> layer_weights(const LlamaShape& s, uint64_t arena, uint64_t l) {
  std::map<std::string, uint64_t> w;
  const uint64_t wb = s.weight_bytes();
  uint64_t at = arena + wb * l * layer_elems(s);
  for (const auto& [name, n] : layer_layout(s)) {
    w[name] = at;
    at += wb * n;
  }
  return w;
}

std::vector<Launch> llama_launches(const LlamaLaunchDesc& d) {
  const LlamaShape& full = d.full;
  const LlamaShape s = shard_of(d);
  const uint64_t m = d.batch, dm = s.d_model, qw = s.q_width(), kvw = s.kv_width(), f = s.ffn;
  const uint64_t vocab_local = full.vocab / d.world;
  const uint64_t wb = s.weight_bytes();
  const uint64_t embed_ptr = d.arena + wb * s.layers * layer_elems(s);
  const uint64_t final_norm_ptr = embed_ptr + wb * full.vocab * full.d_model;

  PlanOptions layer_opts;
  layer_opts.sequence_rows = s.slots == 1 ? m : 1;
  layer_opts.gated = d.gated;
  layer_opts.store_gelus = d.store_gelus;
  LlamaShape head_shape = full;
  head_shape.vocab = vocab_local;
  const Plan embed_plan = plan(PlanOptions{}, embed_program(full));
  const Plan layer_plan = plan(layer_opts, layer_program(s));
  const Plan head_plan = plan(PlanOptions{}, head_program(head_shape));

  AttnBufs attn;
  attn.chunk = d.chunk;
  attn.max_splits = (s.positions + d.chunk - 1) / d.chunk;
  for (int i = 0; i < 3; ++i) attn.partials[i] = d.part[i];
  // A row's sequence: its ring slot, or its block table of the paged pool.
  const std::map<std::string, uint64_t> ints = {
      {"token", d.tokens}, {"position", d.pos}, {s.paged() ? "block_table" : "slot", d.slot}};

  std::vector<Launch> out;
  {
    Binding eb;
    eb.weights = {{"embed", embed_ptr}};
    eb.ints = ints;
    eb.m = m;
    eb.values = {{"x", View{d.x, 0, dm, dm}}};
    for (const Step& st : embed_plan.steps)
      out.push_back(lower_step(embed_plan.program, st, eb, d.cos_t, d.sin_t, attn));
  }
  // A layer's caches: its ring's slots, or its pool's blocks.
  const uint64_t units = s.paged() ? s.blocks : s.slots, unit_len = s.paged() ? s.block_size : s.length;
  // A ring's layer is a slab of the arena; a paged cache's layer is its row
  // of the [layers, blocks] table of block addresses.
  const uint64_t per_cache = s.paged() ? 8 * s.blocks : s.cache_bytes() * units * s.kv_heads * unit_len * s.head_dim;
  for (uint64_t l = 0; l < s.layers; ++l) {
    Binding b;
    b.weights = layer_weights(s, d.arena, l);
    b.ints = ints;
    b.caches = {{"k_cache", d.kbase + l * per_cache}, {"v_cache", d.vbase + l * per_cache}};
    b.m = m;
    b.values = {{"x", View{d.x, 0, dm, dm}},
                {"q", View{d.qkv, 0, qw + 2 * kvw, qw}},
                {"k", View{d.qkv, qw, qw + 2 * kvw, kvw}},
                {"v", View{d.qkv, qw + kvw, qw + 2 * kvw, kvw}},
                {"attended", View{d.att, 0, qw, qw}},
                {"x1", View{d.x1, 0, dm, dm}},
                {"gate", View{d.gu, 0, 2 * f, f}},
                {"up", View{d.gu, f, 2 * f, f}},
                {"x2", View{d.x, 0, dm, dm}}};
    if (s.experts) {
      const uint64_t e = s.experts, k = s.top_k;
      const std::pair<const char*, std::pair<uint64_t, uint64_t>> moe[] = {
          {"mlp_in", {d.mlp_in, dm}},           {"router_logits", {d.router_logits, e}},
          {"route_ids", {d.route_ids, k}},      {"route_weights", {d.route_weights, k}},
          {"experts_gu", {d.experts_gu, k * 2 * f}}, {"experts_act", {d.experts_act, k * f}},
          {"experts_out", {d.experts_out, k * dm}}};
      for (const auto& [name, bw] : moe) b.values[name] = View{bw.first, 0, bw.second, bw.second};
    }
    for (const Step& st : layer_plan.steps)
      for (Launch& L : lower_steps(layer_plan.program, st, b, d.cos_t, d.sin_t, attn)) out.push_back(std::move(L));
  }
  {
    Binding hb;
    hb.weights = {{"embed", embed_ptr + wb * d.rank * vocab_local * full.d_model}, {"final_norm", final_norm_ptr}};
    hb.ints = ints;
    hb.m = m;
    hb.values = {{"x", View{d.x, 0, dm, dm}},
                 {"logits", View{d.logits, 0, vocab_local, vocab_local}},
                 {"token", View{d.out_ids, 0, 1, 1}}};
    for (const Step& st : head_plan.steps)
      out.push_back(lower_step(head_plan.program, st, hb, d.cos_t, d.sin_t, attn));
  }
  if (d.gate_up_interleaved) silu_on_tiles(out, f, d.gu, d.act);
  if (d.world > 1 && d.peer_exchange && s.experts)
    throw Refusal("routed experts over several ranks: their sums travel by NCCL, not peer memory.");
  if (d.world > 1)
    out = d.peer_exchange ? tensor_parallel_peers(out, d, vocab_local) : tensor_parallel_nccl(out, d, vocab_local);
  if (d.fuse_attention) out = fuse_attention(out);
  // The engine's greedy feedback: the ids become the next step's tokens and
  // the positions advance, so replays decode on their own.
  Launch adv;
  adv.kernel = "advance";
  adv.params = {{"m", (double)m}};
  adv.bufs = {d.out_ids, d.tokens, d.pos};
  out.push_back(adv);
  // Split-K a GEMV: a selection's pick for its shape, the same at every
  // batch (so that a row's bits do not depend on its batch); else one,
  // which the streaming and batched kernels keep (past 64 rows, the
  // chunked kernel's choice for the shape). The routed GEMV keeps the
  // lowering's split 1 (its `k` is the route's rank count).
  for (Launch& L : out) {
    if (L.kernel.rfind("gemv", 0) != 0 || L.kernel.rfind("gemv_routed", 0) == 0) continue;
    const uint64_t n = (uint64_t)L.param("n"), k = (uint64_t)L.param("k");
    auto it = d.splits.find({n, k});
    const uint64_t split = it != d.splits.end() ? it->second : m <= 64 ? 1 : split_for(n, k, d.sms);
    const std::string base = kernel_form(L.kernel).first;
    if (split != 1 && m > 4 && (base == "gemv_rmsnorm_silu" || base == "gemv_reduce_rmsnorm_silu"))
      throw Refusal(L.kernel + ": the row-pair kernels take split 1 past batch 4, not " + std::to_string(split) +
                    ".");
    L.set("split", (double)split);
  }
  return out;
}

}  // namespace fkh
