"""Test infrastructure: the Python restatement of the prompt prefill's
launch list (libfurykernel_host.so, fkh_llama_prefill_launches), which the
tests hold the C++ library to."""

from __future__ import annotations

from furykernel_b200 import _native as N
from furykernel_b200.engine import Launch, kernel_form
from furykernel_b200.target import CACHE_SUFFIX, WEIGHT_SUFFIX


def _hi(pre, ptr: int) -> int:
    return pre.w_hi.ptr + (ptr - pre.eng.arena.ptr) * 4 // pre.eng.wb


def _lo(pre, ptr: int) -> int:
    return pre.w_lo.ptr + (ptr - pre.eng.arena.ptr) * 4 // pre.eng.wb


def _gemm(pre, a, K: int, w: int, N: int, c, ldc: int) -> Launch:
    params = {"M": pre.m, "N": N, "K": K, "ldc": ldc}
    if pre.w_hi is None:
        return Launch("gemm_tf32x3w", params, [a, pre.a_hi.ptr, pre.a_lo.ptr, w, c])
    return Launch("gemm_tf32x3", params, [a, pre.a_hi.ptr, pre.a_lo.ptr, _hi(pre, w), _lo(pre, w), c])


def prefill_launches(pre, m: int) -> list:
    """A prefill's launch list over its first m rows in Python: the
    restatement the host library's fkh_llama_prefill_launches is checked
    against."""
    eng, s = pre.eng, pre.eng.s
    if not 1 <= m <= pre.R:
        raise N.Refused(N.FKC_ERR_ARGUMENT, f"prefill: {m} rows, outside 1..{pre.R}.")
    pre.m = m
    d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
    rs4 = 4 * pre.rs
    tok, pos, slot = pre.rows_buf.ptr, pre.rows_buf.ptr + rs4, pre.rows_buf.ptr + 2 * rs4
    # The decode step's own launches are the templates of the gather,
    # the KV stores and the attention (their shapes and tables).
    by = {}
    for L in eng.launches:
        by.setdefault(kernel_form(L.kernel)[0], []).append(L)
    wsuf = WEIGHT_SUFFIX[eng.s.weights]
    csuf = CACHE_SUFFIX[eng.s.cache]
    g0 = by["gather"][0]
    out = [Launch(g0.kernel, dict(g0.params, m=m), [g0.bufs[0], tok, pre.x.ptr])]
    if "attend_decode" in by:  # the decode step fused them: split its launches back into the two steps
        for L in by["attend_decode"]:
            p = L.params
            by.setdefault("kv_store_ring", []).append(Launch("kv_store_ring" + csuf, {
                "m": p["m"], "kv_heads": p["kv_heads"], "d": p["d"], "length": p["length"],
                "rotated": p["rotated"], "ldq": p["ldq"], "k_off": p["k_off"], "v_off": p["v_off"]},
                L.bufs[:7]))
            by.setdefault("attend_split", []).append(Launch("attend_split" + csuf, {
                k: p[k] for k in ("m", "heads", "kv_heads", "d", "length", "rotated", "chunk", "max_splits",
                                  "ldq", "q_off", "scale")}, L.bufs[:10]))
    for L in by.get("attend_decode_paged", []):  # likewise for a paged cache
        p = L.params
        by.setdefault("kv_store_paged", []).append(Launch("kv_store_paged" + csuf, {
            k: p[k] for k in ("m", "kv_heads", "d", "block_size", "table_len", "blocks", "rotated", "ldq",
                              "k_off", "v_off")}, L.bufs[:5] + L.bufs[8:10]))
        by.setdefault("attend_split_paged", []).append(Launch("attend_split_paged" + csuf, {
            k: p[k] for k in ("m", "heads", "kv_heads", "d", "block_size", "table_len", "blocks", "rotated",
                              "chunk", "max_splits", "ldq", "q_off", "scale")}, L.bufs[:10]))
    eps = None
    for L in eng.launches:
        if L.kernel.startswith("gemv") and "eps" in L.params:
            eps = L.params["eps"]
            break
    nq = qw + 2 * kvw
    for l in range(s.layers):
        w = eng.layer_weights(l)
        paged = "kv_store_paged" in by
        kv = by["kv_store_paged" if paged else "kv_store_ring"][l]
        at = by["attend_split_paged" if paged else "attend_split"][l]
        cb = by["attend_combine"][l]
        out.append(Launch("rmsnorm_rows" + wsuf, {"rows": m, "h": d, "eps": eps, "factor": 1.0},
                          [pre.x.ptr, w["attn_norm"], pre.a.ptr]))
        out.append(_gemm(pre, pre.a.ptr, d, w["q_proj"], nq, pre.qkv.ptr, nq))
        out.append(Launch(kv.kernel, dict(kv.params, m=m, ldq=nq),
                          [pre.qkv.ptr, kv.bufs[1], kv.bufs[2], pos, slot, kv.bufs[5], kv.bufs[6]]))
        if pre.one_slot and paged:
            ap = at.params
            out.append(Launch("attend_prompt_paged" + csuf, {
                "m": m, "heads": ap["heads"], "kv_heads": ap["kv_heads"], "d": ap["d"],
                "block_size": ap["block_size"], "table_len": ap["table_len"], "blocks": ap["blocks"],
                "rotated": ap["rotated"], "ldq": nq, "q_off": ap["q_off"], "ldo": qw,
                "max_pos": pre.positions - 1, "scale": ap["scale"]},
                [pre.qkv.ptr, at.bufs[1], at.bufs[2], pos, slot, pre.att.ptr, at.bufs[8], at.bufs[9]]))
        elif pre.one_slot:
            ap = at.params
            out.append(Launch("attend_prompt" + csuf, {
                "m": m, "heads": ap["heads"], "kv_heads": ap["kv_heads"], "d": ap["d"], "length": ap["length"],
                "rotated": ap["rotated"], "ldq": nq, "q_off": ap["q_off"], "ldo": qw,
                "max_pos": pre.positions - 1, "scale": ap["scale"]},
                [pre.qkv.ptr, at.bufs[1], at.bufs[2], pos, slot, at.bufs[5], at.bufs[6], pre.att.ptr]))
        else:
            out.append(Launch(at.kernel, dict(at.params, m=m, ldq=nq, chunk=pre.chunk,
                                                   max_splits=pre.max_splits),
                              [pre.qkv.ptr, at.bufs[1], at.bufs[2], pos, slot, pre.part[0].ptr, pre.part[1].ptr,
                               pre.part[2].ptr, at.bufs[8], at.bufs[9]] if paged else
                              [pre.qkv.ptr, at.bufs[1], at.bufs[2], pos, slot, at.bufs[5], at.bufs[6],
                               pre.part[0].ptr, pre.part[1].ptr, pre.part[2].ptr]))
            out.append(Launch("attend_combine", dict(cb.params, m=m, chunk=pre.chunk,
                                                     max_splits=pre.max_splits, ldo=qw),
                              [pre.part[0].ptr, pre.part[1].ptr, pre.part[2].ptr, pos, pre.att.ptr]))
        out.append(_gemm(pre, pre.att.ptr, qw, w["o_proj"], d, pre.tmp.ptr, d))
        if eng.world > 1:
            out.append(Launch("__allreduce__", {"count": m * d}, [pre.tmp.ptr]))
        out.append(Launch("add", {"n": m * d}, [pre.x.ptr, pre.tmp.ptr, pre.x1.ptr]))
        out.append(Launch("rmsnorm_rows" + wsuf, {"rows": m, "h": d, "eps": eps, "factor": 1.0},
                          [pre.x1.ptr, w["mlp_norm"], pre.a.ptr]))
        if s.experts:  # the decode step's kernels over the m rows
            e, k, b = s.experts, s.top_k, {n: v.ptr for n, v in pre.moe.items()}
            out.append(Launch("gemv" + wsuf, {"n": e, "k": d, "m": m, "split": 1, "ldx": d, "ldy": e},
                              [w["router"], pre.a.ptr, b["router_logits"]]))
            rp = {"m": m, "n": e, "k": k, "ldx": e}
            if s.expert_scale:
                out.append(Launch("route_topk_scaled" + wsuf, rp, [b["router_logits"], w["expert_scale"],
                                                                   b["route_ids"], b["route_weights"]]))
            else:
                out.append(Launch("route_topk", rp, [b["router_logits"], b["route_ids"], b["route_weights"]]))

            def routed(table, n, kk, x, ldx, y, per_rank):
                return Launch("gemv_routed" + wsuf, {"entries": e, "n": n, "kk": kk, "m": m, "k": k, "split": 1,
                                                     "ldx": ldx, "ldy": k * n, "per_rank": per_rank},
                              [table, b["route_ids"], x, y])

            out.append(routed(w["experts_gate_up"], 2 * f, d, pre.a.ptr, d, b["experts_gu"], 0))
            out.append(Launch("gated_gelu", {"segments": m * k, "f": f}, [b["experts_gu"], b["experts_act"]]))
            out.append(routed(w["experts_down"], d, f, b["experts_act"], k * f, b["experts_out"], 1))
            if eng.world > 1:  # each rank ran its ffn slice of every expert: their outputs summed first
                out.append(Launch("__allreduce__", {"count": m * k * d}, [b["experts_out"]]))
            out.append(Launch("combine_ranks_add", {"m": m, "k": k, "d": d},
                              [pre.x1.ptr, b["route_weights"], b["experts_out"], pre.x.ptr]))
            continue
        if eng.gate_up_interleaved:  # rows gate_0, up_0, ...: columns likewise
            out.append(_gemm(pre, pre.a.ptr, d, w["gate_proj"], 2 * f, pre.gu.ptr, 2 * f))
            out.append(Launch("silu_pairs", {"n": m * f}, [pre.gu.ptr, pre.act.ptr]))
        else:  # gate rows, then up rows: one GEMM each, then the gate
            up = pre.gu.ptr + 4 * m * f
            out.append(_gemm(pre, pre.a.ptr, d, w["gate_proj"], f, pre.gu.ptr, f))
            out.append(_gemm(pre, pre.a.ptr, d, w["up_proj"], f, up, f))
            out.append(Launch("silu_mul", {"n": m * f}, [pre.gu.ptr, up, pre.act.ptr]))
        out.append(_gemm(pre, pre.act.ptr, f, w["down_proj"], d, pre.tmp.ptr, d))
        if eng.world > 1:
            out.append(Launch("__allreduce__", {"count": m * d}, [pre.tmp.ptr]))
        out.append(Launch("add", {"n": m * d}, [pre.x1.ptr, pre.tmp.ptr, pre.x.ptr]))
    return out
