// The C ABI of the host library (include/furykernel_host.h) over the fkh
// namespace: every entry catches the C++ side's refusals and returns their
// text.
#include <cstring>
#include <exception>
#include <memory>

#include "../../include/furykernel_host.h"
#include "fkh.h"

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
  o.weights = s.weights_bf16 ? "bf16" : "f32";
  o.cache = s.cache_bf16 ? "bf16" : "f32";
  o.blocks = s.blocks;
  o.block_size = s.block_size;
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

}  // extern "C"
