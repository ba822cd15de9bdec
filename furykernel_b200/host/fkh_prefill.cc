// The prompt prefill's launch list: every prompt row through the layers at
// once, the decode layer's plan run over m rows with the linears as
// tcgen05 3xTF32 GEMM tiles (gemm_tf32x3) instead of GEMVs. The decode
// step's own launches are the templates of the gather, the KV stores and
// the attention (their shapes, tables and caches). A layer of routed
// experts runs its experts through the decode step's own kernels over the
// m rows (the router GEMV, the route, the expert-grouped routed GEMVs, the
// gate, the combine), so its arithmetic is the decode step's.
#include "fkh.h"

namespace fkh {

namespace {

Launch make(const std::string& kernel, std::vector<std::pair<std::string, double>> params,
            std::vector<uint64_t> bufs) {
  Launch L;
  L.kernel = kernel;
  L.params = std::move(params);
  L.bufs = std::move(bufs);
  return L;
}

// A launch's parameters with some replaced (the rest keep their order).
Launch with(const Launch& t, const std::vector<std::pair<std::string, double>>& changes, std::vector<uint64_t> bufs) {
  Launch L = t;
  for (const auto& [k, v] : changes) L.set(k, v);
  L.bufs = std::move(bufs);
  return L;
}

}  // namespace

std::vector<Launch> prefill_launches(const LlamaLaunchDesc& d, const PrefillDesc& p, uint64_t m) {
  if (m < 1 || m > p.rows)
    throw Refusal("prefill: " + std::to_string(m) + " rows, outside 1.." + std::to_string(p.rows) + ".");
  const LlamaShape s = shard_of(d);
  const uint64_t dm = s.d_model, qw = s.q_width(), kvw = s.kv_width(), f = s.ffn, nq = qw + 2 * kvw;
  const uint64_t max_splits = (p.positions + p.chunk - 1) / p.chunk;
  const std::vector<Launch> decode = llama_launches(d);

  // The decode launches by their f32 entries' names; the forms follow the
  // model's element types.
  std::map<std::string, std::vector<const Launch*>> by;
  for (const Launch& L : decode) by[kernel_form(L.kernel).first].push_back(&L);
  const std::string wsuf = weight_form(s.weights, "prefill");
  const std::string csuf = cache_form(s.cache, "prefill");
  auto need = [&](const std::string& k, uint64_t i) -> const Launch& {
    auto it = by.find(k);
    if (it == by.end() || it->second.size() <= i) throw Refusal("prefill: the decode step has no " + k + " launch.");
    return *it->second[i];
  };
  // Where the decode step folded each layer's store into its attention,
  // split the launches back into the two steps.
  std::vector<Launch> unfused;
  if (by.count("attend_decode")) {
    unfused.reserve(2 * by["attend_decode"].size());
    for (const Launch* L : by["attend_decode"]) {
      unfused.push_back(make("kv_store_ring" + csuf,
                             {{"m", L->param("m")},
                              {"kv_heads", L->param("kv_heads")},
                              {"d", L->param("d")},
                              {"length", L->param("length")},
                              {"rotated", L->param("rotated")},
                              {"ldq", L->param("ldq")},
                              {"k_off", L->param("k_off")},
                              {"v_off", L->param("v_off")}},
                             {L->bufs.begin(), L->bufs.begin() + 7}));
      std::vector<std::pair<std::string, double>> ap;
      for (const char* k : {"m", "heads", "kv_heads", "d", "length", "rotated", "chunk", "max_splits", "ldq", "q_off",
                            "scale"})
        ap.emplace_back(k, L->param(k));
      unfused.push_back(make("attend_split" + csuf, ap, {L->bufs.begin(), L->bufs.begin() + 10}));
    }
  }
  if (by.count("attend_decode_paged")) {  // likewise for a paged cache
    for (const Launch* L : by["attend_decode_paged"]) {
      std::vector<std::pair<std::string, double>> kp, ap;
      for (const char* k : {"m", "kv_heads", "d", "block_size", "table_len", "blocks", "rotated", "ldq", "k_off",
                            "v_off"})
        kp.emplace_back(k, L->param(k));
      for (const char* k : {"m", "heads", "kv_heads", "d", "block_size", "table_len", "blocks", "rotated", "chunk",
                            "max_splits", "ldq", "q_off", "scale"})
        ap.emplace_back(k, L->param(k));
      // The store: the attention's first five buffers and its two tables.
      unfused.push_back(make("kv_store_paged" + csuf, kp,
                             {L->bufs[0], L->bufs[1], L->bufs[2], L->bufs[3], L->bufs[4], L->bufs[8], L->bufs[9]}));
      unfused.push_back(make("attend_split_paged" + csuf, ap, {L->bufs.begin(), L->bufs.begin() + 10}));
    }
  }
  for (const Launch& L : unfused) by[kernel_form(L.kernel).first].push_back(&L);
  double eps = 0;
  bool have_eps = false;
  for (const Launch& L : decode)
    if (L.kernel.rfind("gemv", 0) == 0 && L.has("eps")) {
      eps = L.param("eps");
      have_eps = true;
      break;
    }
  if (!have_eps) throw Refusal("prefill: the decode step normalizes nothing.");

  // f32 weights: the GEMM reads them from the weight arena and splits them
  // into their TF32 halves itself (gemm_tf32x3w). 16-bit weights: their
  // widened halves are f32 arenas laid out as the weight arena (the low
  // half 0), read by gemm_tf32x3.
  const uint64_t wb = s.weight_bytes();
  const bool f32w = wb == 4;
  auto hi = [&](uint64_t w) { return p.w_hi + (w - d.arena) * 4 / wb; };
  auto lo = [&](uint64_t w) { return p.w_lo + (w - d.arena) * 4 / wb; };
  auto gemm = [&](uint64_t a, uint64_t K, uint64_t w, uint64_t N, uint64_t c, uint64_t ldc) {
    const std::vector<std::pair<std::string, double>> prm = {
        {"M", (double)m}, {"N", (double)N}, {"K", (double)K}, {"ldc", (double)ldc}};
    if (f32w) return make("gemm_tf32x3w", prm, {a, p.a_hi, p.a_lo, w, c});
    return make("gemm_tf32x3", prm, {a, p.a_hi, p.a_lo, hi(w), lo(w), c});
  };
  const double md = (double)m;

  std::vector<Launch> out;
  const Launch& g0 = need("gather", 0);
  out.push_back(with(g0, {{"m", md}}, {g0.bufs[0], p.tokens, p.x}));
  for (uint64_t l = 0; l < s.layers; ++l) {
    const auto w = layer_weights(s, d.arena, l);
    const bool paged = s.paged();
    const Launch& kv = need(paged ? "kv_store_paged" : "kv_store_ring", l);
    const Launch& at = need(paged ? "attend_split_paged" : "attend_split", l);
    const Launch& cb = need("attend_combine", l);
    out.push_back(make("rmsnorm_rows" + wsuf, {{"rows", md}, {"h", (double)dm}, {"eps", eps}, {"factor", 1.0}},
                       {p.x, w.at("attn_norm"), p.a}));
    out.push_back(gemm(p.a, dm, w.at("q_proj"), nq, p.qkv, nq));
    out.push_back(with(kv, {{"m", md}, {"ldq", (double)nq}},
                       {p.qkv, kv.bufs[1], kv.bufs[2], p.pos, p.slot, kv.bufs[5], kv.bufs[6]}));
    if (p.one_slot && paged) {
      out.push_back(make("attend_prompt_paged" + csuf,
                         {{"m", md},
                          {"heads", at.param("heads")},
                          {"kv_heads", at.param("kv_heads")},
                          {"d", at.param("d")},
                          {"block_size", at.param("block_size")},
                          {"table_len", at.param("table_len")},
                          {"blocks", at.param("blocks")},
                          {"rotated", at.param("rotated")},
                          {"ldq", (double)nq},
                          {"q_off", at.param("q_off")},
                          {"ldo", (double)qw},
                          {"max_pos", (double)(p.positions - 1)},
                          {"scale", at.param("scale")}},
                         {p.qkv, at.bufs[1], at.bufs[2], p.pos, p.slot, p.att, at.bufs[8], at.bufs[9]}));
    } else if (p.one_slot) {
      out.push_back(make("attend_prompt" + csuf,
                         {{"m", md},
                          {"heads", at.param("heads")},
                          {"kv_heads", at.param("kv_heads")},
                          {"d", at.param("d")},
                          {"length", at.param("length")},
                          {"rotated", at.param("rotated")},
                          {"ldq", (double)nq},
                          {"q_off", at.param("q_off")},
                          {"ldo", (double)qw},
                          {"max_pos", (double)(p.positions - 1)},
                          {"scale", at.param("scale")}},
                         {p.qkv, at.bufs[1], at.bufs[2], p.pos, p.slot, at.bufs[5], at.bufs[6], p.att}));
    } else {
      out.push_back(with(at,
                         {{"m", md}, {"ldq", (double)nq}, {"chunk", (double)p.chunk},
                          {"max_splits", (double)max_splits}},
                         paged ? std::vector<uint64_t>{p.qkv, at.bufs[1], at.bufs[2], p.pos, p.slot, p.part[0],
                                                       p.part[1], p.part[2], at.bufs[8], at.bufs[9]}
                               : std::vector<uint64_t>{p.qkv, at.bufs[1], at.bufs[2], p.pos, p.slot, at.bufs[5],
                                                       at.bufs[6], p.part[0], p.part[1], p.part[2]}));
      out.push_back(with(cb,
                         {{"m", md}, {"chunk", (double)p.chunk}, {"max_splits", (double)max_splits},
                          {"ldo", (double)qw}},
                         {p.part[0], p.part[1], p.part[2], p.pos, p.att}));
    }
    // The row-parallel projections' partial sums are added across the
    // ranks before the residual add.
    out.push_back(gemm(p.att, qw, w.at("o_proj"), dm, p.tmp, dm));
    if (d.world > 1) out.push_back(make("__allreduce__", {{"count", (double)(m * dm)}}, {p.tmp}));
    out.push_back(make("add", {{"n", (double)(m * dm)}}, {p.x, p.tmp, p.x1}));
    out.push_back(make("rmsnorm_rows" + wsuf, {{"rows", md}, {"h", (double)dm}, {"eps", eps}, {"factor", 1.0}},
                       {p.x1, w.at("mlp_norm"), p.a}));
    if (s.experts) {
      const uint64_t e = s.experts, k = s.top_k;
      out.push_back(make("gemv" + wsuf,
                         {{"n", (double)e}, {"k", (double)dm}, {"m", md}, {"split", 1.0}, {"ldx", (double)dm},
                          {"ldy", (double)e}},
                         {w.at("router"), p.a, p.router_logits}));
      const std::vector<std::pair<std::string, double>> rp = {
          {"m", md}, {"n", (double)e}, {"k", (double)k}, {"ldx", (double)e}};
      if (s.expert_scale)
        out.push_back(make("route_topk_scaled" + wsuf, rp,
                           {p.router_logits, w.at("expert_scale"), p.route_ids, p.route_weights}));
      else
        out.push_back(make("route_topk", rp, {p.router_logits, p.route_ids, p.route_weights}));
      auto routed = [&](uint64_t table, uint64_t n, uint64_t kk, uint64_t x, uint64_t ldx, uint64_t y, bool per_rank) {
        return make("gemv_routed" + wsuf,
                    {{"entries", (double)e},
                     {"n", (double)n},
                     {"kk", (double)kk},
                     {"m", md},
                     {"k", (double)k},
                     {"split", 1.0},
                     {"ldx", (double)ldx},
                     {"ldy", (double)(k * n)},
                     {"per_rank", per_rank ? 1.0 : 0.0}},
                    {table, p.route_ids, x, y});
      };
      out.push_back(routed(w.at("experts_gate_up"), 2 * f, dm, p.a, dm, p.experts_gu, false));
      out.push_back(make("gated_gelu", {{"segments", md * (double)k}, {"f", (double)f}}, {p.experts_gu, p.experts_act}));
      out.push_back(routed(w.at("experts_down"), dm, f, p.experts_act, k * f, p.experts_out, true));
      // Each rank ran its ffn slice of every expert: their outputs are summed first.
      if (d.world > 1) out.push_back(make("__allreduce__", {{"count", (double)(m * k * dm)}}, {p.experts_out}));
      out.push_back(make("combine_ranks_add", {{"m", md}, {"k", (double)k}, {"d", (double)dm}},
                         {p.x1, p.route_weights, p.experts_out, p.x}));
      continue;
    }
    if (d.gate_up_interleaved) {  // rows gate_0, up_0, ...: the GEMM's columns likewise
      out.push_back(gemm(p.a, dm, w.at("gate_proj"), 2 * f, p.gu, 2 * f));
      out.push_back(make("silu_pairs", {{"n", (double)(m * f)}}, {p.gu, p.act}));
    } else {  // gate rows, then up rows: a GEMM each, then the gate
      const uint64_t up = p.gu + 4 * m * f;
      out.push_back(gemm(p.a, dm, w.at("gate_proj"), f, p.gu, f));
      out.push_back(gemm(p.a, dm, w.at("up_proj"), f, up, f));
      out.push_back(make("silu_mul", {{"n", (double)(m * f)}}, {p.gu, up, p.act}));
    }
    out.push_back(gemm(p.act, f, w.at("down_proj"), dm, p.tmp, dm));
    if (d.world > 1) out.push_back(make("__allreduce__", {{"count", (double)(m * dm)}}, {p.tmp}));
    out.push_back(make("add", {{"n", (double)(m * dm)}}, {p.x1, p.tmp, p.x}));
  }
  return out;
}

}  // namespace fkh
