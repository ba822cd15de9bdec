// The C ABI of the host library (include/furykernel_host.h) over the fkh
// namespace: every entry catches the C++ side's refusals and returns their
// text.
#include <cstring>
#include <exception>
#include <memory>

#include "../../include/furykernel_host.h"
#include "fkh.h"
#include "fkh_select.h"

struct fkh_launches {
  std::vector<fkh::Launch> list;
};

namespace {

void put_err(char* err, size_t cap, const char* text) {
  if (!err || cap == 0) return;
  const size_t n = std::min(cap - 1, std::strlen(text));
  std::memcpy(err, text, n);
  err[n] = 0;
}

int put_text(const std::string& s, char* buf, size_t cap, size_t* len) {
  if (len) *len = s.size();
  if (!buf || cap < s.size() + 1) return FKH_ERR_SPACE;
  std::memcpy(buf, s.data(), s.size());
  buf[s.size()] = 0;
  return FKH_OK;
}

template <typename F>
int guarded(char* err, size_t err_cap, F&& f) {
  try {
    return f();
  } catch (const fkh::Refusal& e) {
    put_err(err, err_cap, e.what());
    return FKH_ERR_ARGUMENT;
  } catch (const std::exception& e) {
    put_err(err, err_cap, e.what());
    return FKH_ERR_INTERNAL;
  } catch (...) {
    put_err(err, err_cap, "an unknown failure.");
    return FKH_ERR_INTERNAL;
  }
}

fkh::LlamaShape shape_of(const fkh_llama_shape& s) {
  fkh::LlamaShape o;
  o.d_model = s.d_model;
  o.heads = s.heads;
  o.kv_heads = s.kv_heads;
  o.head_dim = s.head_dim;
  o.ffn = s.ffn;
  o.vocab = s.vocab;
  o.layers = s.layers;
  o.theta = s.theta;
  o.eps = s.eps;
  o.slots = s.slots;
  o.length = s.length;
  o.positions = s.positions;
  static const char* const types[] = {"f32", "bf16", "f16"};
  if (s.weights_type < 0 || s.weights_type > 2 || s.cache_type < 0 || s.cache_type > 2)
    throw fkh::Refusal("the shape's element types are " + std::to_string(s.weights_type) + " and " +
                       std::to_string(s.cache_type) + ", not 0 (f32), 1 (bf16) or 2 (f16).");
  o.weights = types[s.weights_type];
  o.cache = types[s.cache_type];
  o.expert_scale = s.expert_scale != 0;
  o.blocks = s.blocks;
  o.block_size = s.block_size;
  o.experts = s.experts;
  o.top_k = s.top_k;
  if (o.experts && (o.top_k == 0 || o.top_k > o.experts)) throw fkh::Refusal("top_k must be 1 to experts.");
  if (o.paged() && !o.blocks) throw fkh::Refusal("a paged cache of no blocks.");
  if (!o.heads || !o.kv_heads || o.heads % o.kv_heads || !o.head_dim || o.head_dim % 2 || !o.d_model ||
      !o.ffn || !o.vocab || !o.slots || !o.length || !o.positions)
    throw fkh::Refusal("the Llama shape has an empty or uneven dimension.");
  return o;
}

bool valid(const fkh_launches* l, size_t i) { return l && i < l->list.size(); }

fkh::LlamaLaunchDesc desc_of(const fkh_llama_desc& desc) {
  fkh::LlamaLaunchDesc d;
  d.full = shape_of(desc.full);
  d.batch = desc.batch;
  d.rank = desc.rank;
  d.world = desc.world;
  d.sms = desc.sms;
  d.chunk = desc.chunk;
  if (!d.batch || !d.world || d.rank >= d.world || !d.sms || !d.chunk)
    throw fkh::Refusal("batch, world, sms and chunk must be positive and rank below world.");
  d.gate_up_interleaved = desc.gate_up_interleaved != 0;
  d.peer_exchange = desc.peer_exchange != 0;
  d.fuse_attention = desc.fuse_attention != 0;
  d.arena = desc.arena;
  d.kbase = desc.kbase;
  d.vbase = desc.vbase;
  d.cos_t = desc.cos_t;
  d.sin_t = desc.sin_t;
  d.tokens = desc.tokens;
  d.pos = desc.pos;
  d.slot = desc.slot;
  d.x = desc.x;
  d.x1 = desc.x1;
  d.qkv = desc.qkv;
  d.att = desc.att;
  d.gu = desc.gu;
  d.act = desc.act;
  d.logits = desc.logits;
  d.out_ids = desc.out_ids;
  d.partial = desc.partial;
  d.pairs = desc.pairs;
  d.pairs_all = desc.pairs_all;
  for (int i = 0; i < 3; ++i) d.part[i] = desc.part[i];
  d.mlp_in = desc.mlp_in;
  d.router_logits = desc.router_logits;
  d.route_ids = desc.route_ids;
  d.route_weights = desc.route_weights;
  d.experts_gu = desc.experts_gu;
  d.experts_act = desc.experts_act;
  d.experts_out = desc.experts_out;
  d.gated = desc.gated != 0;
  d.store_gelus = desc.store_gelus != 0;
  if (desc.nsplits && !desc.splits) throw fkh::Refusal("nsplits without splits.");
  for (size_t i = 0; i < desc.nsplits; ++i) {
    const uint32_t s = desc.splits[3 * i + 2];
    if (s != 1 && s != 2 && s != 4 && s != 8) throw fkh::Refusal("a split of " + std::to_string(s) + ", not 1, 2, 4 or 8.");
    d.splits[{desc.splits[3 * i], desc.splits[3 * i + 1]}] = s;
  }
  return d;
}

}  // namespace

extern "C" {

int fkh_abi_version(void) { return FKH_ABI_VERSION; }

int fkh_llama_program_text(const fkh_llama_shape* shape, int which, char* buf, size_t cap, size_t* len, char* err,
                           size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!shape) throw fkh::Refusal("no shape.");
    const fkh::LlamaShape s = shape_of(*shape);
    fkh::Program p;
    switch (which) {
      case 0: p = fkh::embed_program(s); break;
      case 1: p = fkh::layer_program(s); break;
      case 2: p = fkh::head_program(s); break;
      default: throw fkh::Refusal("no program " + std::to_string(which) + ": 0 embed, 1 layer, 2 head.");
    }
    return put_text(fkh::render_program(p), buf, cap, len);
  });
}

int fkh_program_roundtrip(const char* program_text, char* buf, size_t cap, size_t* len, char* err, size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!program_text) throw fkh::Refusal("no program text.");
    return put_text(fkh::render_program(fkh::parse_program(program_text)), buf, cap, len);
  });
}

int fkh_plan_text(const char* program_text, const fkh_plan_options* opts, char* buf, size_t cap, size_t* len,
                  char* err, size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!program_text) throw fkh::Refusal("no program text.");
    fkh::PlanOptions o;
    if (opts) {
      o.horizontal = opts->horizontal != 0;
      o.gated = opts->gated != 0;
      o.store_gelus = opts->store_gelus != 0;
      o.sequence_rows = opts->sequence_rows;
    }
    if (o.sequence_rows == 0) throw fkh::Refusal("sequence_rows is 0.");
    return put_text(fkh::render_plan(fkh::plan(o, fkh::parse_program(program_text))), buf, cap, len);
  });
}

int fkh_llama_launches(const fkh_llama_desc* desc, fkh_launches** out, char* err, size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!desc || !out) throw fkh::Refusal("no descriptor or no place for the launches.");
    *out = nullptr;
    auto l = std::make_unique<fkh_launches>();
    l->list = fkh::llama_launches(desc_of(*desc));
    *out = l.release();
    return FKH_OK;
  });
}

int fkh_llama_prefill_launches(const fkh_llama_desc* desc, const fkh_prefill_desc* prefill, uint64_t m,
                               fkh_launches** out, char* err, size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!desc || !prefill || !out) throw fkh::Refusal("no descriptor or no place for the launches.");
    *out = nullptr;
    fkh::PrefillDesc p;
    p.rows = prefill->rows;
    p.chunk = prefill->chunk;
    p.positions = prefill->positions;
    if (!p.rows || !p.chunk || !p.positions) throw fkh::Refusal("prefill: rows, chunk and positions must be positive.");
    p.one_slot = prefill->one_slot != 0;
    p.w_hi = prefill->w_hi;
    p.w_lo = prefill->w_lo;
    p.tokens = prefill->tokens;
    p.pos = prefill->pos;
    p.slot = prefill->slot;
    p.x = prefill->x;
    p.a = prefill->a;
    p.a_hi = prefill->a_hi;
    p.a_lo = prefill->a_lo;
    p.qkv = prefill->qkv;
    p.att = prefill->att;
    p.tmp = prefill->tmp;
    p.x1 = prefill->x1;
    p.gu = prefill->gu;
    p.act = prefill->act;
    for (int i = 0; i < 3; ++i) p.part[i] = prefill->part[i];
    p.router_logits = prefill->router_logits;
    p.route_ids = prefill->route_ids;
    p.route_weights = prefill->route_weights;
    p.experts_gu = prefill->experts_gu;
    p.experts_act = prefill->experts_act;
    p.experts_out = prefill->experts_out;
    auto l = std::make_unique<fkh_launches>();
    l->list = fkh::prefill_launches(desc_of(*desc), p, m);
    *out = l.release();
    return FKH_OK;
  });
}

size_t fkh_launches_count(const fkh_launches* l) { return l ? l->list.size() : 0; }

const char* fkh_launch_kernel(const fkh_launches* l, size_t i) {
  return valid(l, i) ? l->list[i].kernel.c_str() : nullptr;
}

size_t fkh_launch_param_count(const fkh_launches* l, size_t i) { return valid(l, i) ? l->list[i].params.size() : 0; }

const char* fkh_launch_param_name(const fkh_launches* l, size_t i, size_t j) {
  return valid(l, i) && j < l->list[i].params.size() ? l->list[i].params[j].first.c_str() : nullptr;
}

double fkh_launch_param_value(const fkh_launches* l, size_t i, size_t j) {
  return valid(l, i) && j < l->list[i].params.size() ? l->list[i].params[j].second : 0.0;
}

size_t fkh_launch_buf_count(const fkh_launches* l, size_t i) { return valid(l, i) ? l->list[i].bufs.size() : 0; }

uint64_t fkh_launch_buf(const fkh_launches* l, size_t i, size_t j) {
  return valid(l, i) && j < l->list[i].bufs.size() ? l->list[i].bufs[j] : 0;
}

void fkh_launches_free(fkh_launches* l) { delete l; }

uint64_t fkh_split_for(uint64_t n_rows, uint64_t k, uint64_t sms) { return fkh::split_for(n_rows, k, sms); }

// ---- JSON, variant spaces, selections -------------------------------------

int fkh_json_roundtrip(const char* text, char* buf, size_t cap, size_t* len, char* err, size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!text) throw fkh::Refusal("no text.");
    return put_text(fkh::render_json(fkh::parse_json(text)), buf, cap, len);
  });
}

int fkh_selection_roundtrip(const char* text, char* buf, size_t cap, size_t* len, char* err, size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!text) throw fkh::Refusal("no text.");
    return put_text(fkh::render_selection(fkh::parse_selection(text)), buf, cap, len);
  });
}

namespace {

std::vector<fkh::VShape> gemv_classes(const uint32_t* classes, size_t count) {
  if (count && !classes) throw fkh::Refusal("no classes.");
  std::vector<fkh::VShape> out;
  for (size_t i = 0; i < count; ++i)
    out.push_back({{"n", classes[3 * i]}, {"k", classes[3 * i + 1]}, {"m", classes[3 * i + 2]}});
  return out;
}

// A space from its JSON description: {"family": ..., "axes": [{"name",
// "prefix", "values": [...], "order"}], "classes": [{dim: value, ...} or
// [[dim, value], ...]], "batch": [...]}; its points are all kept, each its
// own kernel.
fkh::Space space_of(const std::string& text) {
  const fkh::Json j = fkh::parse_json(text);
  auto get = [&](const fkh::Json& o, const std::string& k) -> const fkh::Json& {
    for (const auto& m : o.members)
      if (m.first == k) return m.second;
    throw fkh::Refusal("the space has no " + k + ".");
  };
  fkh::Space sp;
  sp.family = get(j, "family").s;
  for (const fkh::Json& a : get(j, "axes").items) {
    fkh::Axis ax{get(a, "name").s, get(a, "prefix").s, {}, get(a, "order").b};
    for (const fkh::Json& v : get(a, "values").items) ax.values.push_back((uint64_t)v.i);
    sp.axes.push_back(ax);
  }
  for (const fkh::Json& c : get(j, "classes").items) {  // an object, or a list of [dimension, value] pairs
    fkh::VShape s;
    if (c.kind == fkh::Json::Array) {
      for (const fkh::Json& dv : c.items)
        if (dv.kind == fkh::Json::Array && dv.items.size() == 2) s.emplace_back(dv.items[0].s, (uint64_t)dv.items[1].i);
    } else {
      for (const auto& [d, v] : c.members) s.emplace_back(d, (uint64_t)v.i);
    }
    sp.shapes.push_back(s);
  }
  for (const fkh::Json& b : get(j, "batch").items) sp.batch.push_back(b.s);
  sp.consider = [](const fkh::VShape& s, const fkh::Point& p, uint64_t) {
    fkh::Outcome o;
    o.kind = fkh::Outcome::Kept;
    o.hash = std::hash<std::string>{}(fkh::shape_key(s) + "/" + fkh::axis_key(p));
    return o;
  };
  return sp;
}

}  // namespace

int fkh_space_check(const char* space_json, char* buf, size_t cap, size_t* len, char* err, size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!space_json) throw fkh::Refusal("no space.");
    std::string out;
    for (const std::string& p : fkh::check_space(space_of(space_json))) out += p + "\n";
    return put_text(out, buf, cap, len);
  });
}

int fkh_space_parse_key(const char* space_json, const char* key, char* buf, size_t cap, size_t* len, char* err,
                        size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!space_json || !key) throw fkh::Refusal("no space or no key.");
    return put_text(fkh::axis_key(fkh::parse_axis_key(space_of(space_json).axes, key)), buf, cap, len);
  });
}

int fkh_space_names(const char* space_json, char* buf, size_t cap, size_t* len, char* err, size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!space_json) throw fkh::Refusal("no space.");
    const fkh::Space sp = space_of(space_json);
    std::string out;
    for (const fkh::VShape& s : sp.shapes)
      for (const fkh::Point& p : fkh::points(sp.axes)) {
        const std::string name = fkh::variant_name(sp, s, p);
        fkh::VShape back;
        fkh::Point pb;
        const bool ok = fkh::variant_of_name(sp, name, back, pb) && back == s && pb == p;
        out += name + (ok ? "" : " (does not read back)") + "\n";
      }
    return put_text(out, buf, cap, len);
  });
}

int fkh_split_join(const char* name, const char* right_prefix, char* buf, size_t cap, size_t* len, char* err,
                   size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!name || !right_prefix) throw fkh::Refusal("no name.");
    const std::string pre = right_prefix;
    // Valid: the prefix then one or more digits; with no prefix, a step's name.
    auto valid = [&](const std::string& r) {
      if (pre.empty()) return fkh::is_step_name(r);
      if (r.compare(0, pre.size(), pre) != 0 || r.size() == pre.size()) return false;
      for (size_t i = pre.size(); i < r.size(); ++i)
        if (r[i] < '0' || r[i] > '9') return false;
      return true;
    };
    std::string left, right;
    if (!fkh::split_join(valid, name, left, right)) return put_text("", buf, cap, len);
    return put_text(left + "\n" + right, buf, cap, len);
  });
}

int fkh_gemv_consider(uint32_t n, uint32_t k, uint32_t m, uint32_t split, uint32_t cores, int* kind, uint64_t* groups,
                      uint64_t* hash, char* reasons, size_t reasons_cap) {
  return guarded(reasons, reasons_cap, [&] {
    const fkh::Space sp = fkh::gemv_space({});
    const fkh::Outcome o = sp.consider({{"n", n}, {"k", k}, {"m", m}}, {{"s", split}}, cores);
    if (kind) *kind = (int)o.kind;
    if (groups) *groups = o.groups;
    if (hash) *hash = o.hash;
    std::string r;
    for (const std::string& x : o.reasons) r += (r.empty() ? "" : " ") + x;
    put_err(reasons, reasons_cap, r.c_str());
    return FKH_OK;
  });
}

int fkh_gemv_selection_render(const uint32_t* classes, const uint32_t* splits, size_t count, uint32_t cores,
                              char* buf, size_t cap, size_t* len, char* err, size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (count && !splits) throw fkh::Refusal("no splits.");
    const std::vector<fkh::VShape> cls = gemv_classes(classes, count);
    const fkh::Space sp = fkh::gemv_space(cls);
    fkh::Selection sel;
    sel.family = sp.family;
    sel.target = fkh::kTargetName;
    sel.cores = cores;
    for (size_t i = 0; i < count; ++i) {
      const fkh::Point p{{"s", splits[i]}};
      const fkh::Outcome o = sp.consider(cls[i], p, cores);
      if (o.kind != fkh::Outcome::Kept)
        throw fkh::Refusal(fkh::variant_name(sp, cls[i], p) + " is not a kept variant of its class.");
      sel.classes[fkh::shape_key(cls[i])] = fkh::Pick{fkh::axis_key(p), o.hash};
    }
    fkh::validate_selection(cores, fkh::kTargetName, sp, sel);
    return put_text(fkh::render_selection(sel), buf, cap, len);
  });
}

int fkh_gemv_selection_validate(const char* text, const uint32_t* classes, size_t count, uint32_t cores,
                                uint32_t* splits, char* err, size_t err_cap) {
  return guarded(err, err_cap, [&] {
    if (!text || (count && !splits)) throw fkh::Refusal("no selection or no place for the splits.");
    const fkh::Space sp = fkh::gemv_space(gemv_classes(classes, count));
    const std::vector<fkh::Point> picks = fkh::validate_selection(cores, fkh::kTargetName, sp,
                                                                  fkh::parse_selection(text));
    for (size_t i = 0; i < picks.size(); ++i) splits[i] = (uint32_t)picks[i][0].second;
    return FKH_OK;
  });
}

}  // extern "C"
