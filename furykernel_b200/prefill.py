"""Prompt prefill for the Llama engine: every prompt row through the layers
at once, the projections as tcgen05 3xTF32 GEMMs (`gemm_tf32x3w`), which
store each row's keys and values in the Ring caches; then the engine's
decode step continues from the last prompt row.

The plan is the decode layer's (src/FuryKernel/Program/Plan.hs: RMSNorm
before each anchor, the KV store before the attention, the residual Adds),
run over R rows with the linears as tiles instead of GEMVs:

    x  = gather(embed, tokens)
    per layer:
      a    = rmsnorm_rows(x, attn_norm)
      qkv  = a [q;k;v]^T                      (GEMM)
      kv_store_ring(qkv rows at their positions)
      att  = attend_split + attend_combine     (each row over positions <= its own)
      x1   = x + att o^T                       (GEMM, then add; TP: allreduce first)
      m    = rmsnorm_rows(x1, mlp_norm)
      act  = silu(m gate^T) * (m up^T)         (GEMM over the arena's gate/up rows)
      x    = x1 + act down^T                   (GEMM, then add; TP: allreduce first)

The GEMMs are 3xTF32 (a_hi b_hi + a_hi b_lo + a_lo b_hi, f32 accumulation
in TMEM), so prefill agrees with the binary32 contract within the f64
evaluator's bounds, not bit for bit; the decode steps after it are the
contract's bits given the caches prefill left. f32 weights are read from
the weight arena and split into their TF32 halves inside the GEMM
(`gemm_tf32x3w`); 16-bit weights are widened once into two arenas laid out
as the weight arena (`gemm_tf32x3`).

With tensor parallelism each rank runs its shard's GEMMs; the row-parallel
partials (o, down) are summed by an NCCL allreduce before the residual add.
"""

from __future__ import annotations

import numpy as np

from . import _native as N
from .engine import Launch, Llama
from .target import WEIGHT_SUFFIX


class Prefill:
    """Prefill of up to `rows` prompt rows for an engine (any batch, any
    rank). `run(tokens, positions, slots)` stores the rows' keys and values
    and leaves the last layer's rows in `x`."""

    def __init__(self, eng: Llama, rows: int, chunk: int | None = None, positions: int | None = None,
                 one_slot: bool = False):
        ctx, s = eng.ctx, eng.s
        self.eng, self.ctx, self.R = eng, ctx, rows
        d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
        for what, k in (("d_model", d), ("q width", qw), ("ffn", f)):
            if k % 32:
                raise N.Refused(N.FKC_ERR_ARGUMENT, f"prefill: the GEMM's K ({what} {k}) is not a multiple of 32.")
        # f32 weights: the GEMMs read the weight arena and split each slab
        # into its TF32 halves on the chip (gemm_tf32x3w). 16-bit weights:
        # the widened weights (the high halves; the low halves 0) in two
        # arenas laid out as the weight arena, a layer a launch.
        per = eng.layer_elems
        self.w_hi = self.w_lo = None
        if eng.wb != 4:
            self.w_hi = ctx.alloc(4 * s.layers * per)
            self.w_lo = ctx.alloc(4 * s.layers * per)
            split = "split_tf32" + WEIGHT_SUFFIX[eng.s.weights]
            for l in range(s.layers):
                at = 4 * l * per
                ctx.launch(split, {"n": per},
                           [eng.arena.ptr + eng.wb * l * per, self.w_hi.ptr + at, self.w_lo.ptr + at])
        R = rows
        kmax = max(d, qw, f)
        # Tokens, positions, then each row's slot or (paged) block table.
        self.rs = (R + 3) // 4 * 4
        self.seq = s.table_len if s.paged else 1
        self.rows_words = 2 * self.rs + (R * self.seq + 3) // 4 * 4
        self.rows_buf = ctx.zeros(self.rows_words, np.uint32)
        self.x = ctx.zeros((R, d))
        self.a = ctx.zeros((R, d))
        self.a_hi = ctx.zeros((R, kmax))
        self.a_lo = ctx.zeros((R, kmax))
        self.qkv = ctx.zeros((R, qw + 2 * kvw))
        self.att = ctx.zeros((R, qw))
        self.tmp = ctx.zeros((R, d))
        self.x1 = ctx.zeros((R, d))
        self.gu = ctx.zeros((R, 2 * f))
        self.act = ctx.zeros((R, f))
        # Routed experts over the rows, through the decode step's kernels:
        # the router's logits, the route, the experts' gate/up rows, their
        # gate, their outputs.
        self.moe = {}
        if s.experts:
            e, k = s.experts, s.top_k
            self.moe = {"router_logits": ctx.zeros((R, e)), "route_ids": ctx.zeros((R, k), np.uint32),
                        "route_weights": ctx.zeros((R, k)), "experts_gu": ctx.zeros((R, k * 2 * f)),
                        "experts_act": ctx.zeros((R, k * f)), "experts_out": ctx.zeros((R, k * d))}
        self.chunk = chunk or eng.chunk
        # Splits a row's attention can have: up to the largest position a
        # prefill here stores (the engine's positions unless given).
        self.positions = positions or s.positions
        self.max_splits = (self.positions + self.chunk - 1) // self.chunk
        # One prompt (one slot) a run: the attention tiled by queries
        # (attend_prompt), each round of keys shared by 64 rows, instead of
        # the decode attention over every row.
        span = s.table_len * s.block_size if s.paged else s.length
        self.one_slot = one_slot and self.positions <= span
        ms = R * s.heads * self.max_splits
        self.part = [ctx.zeros(ms), ctx.zeros(ms), ctx.zeros(ms * s.head_dim)]
        self.graphs: dict = {}

    def launches(self, m: int) -> list:
        """The launch list over the first m rows of the row buffers, from
        libfurykernel_host.so (fkh_llama_prefill_launches)."""
        from . import _host

        if not 1 <= m <= self.R:
            raise N.Refused(N.FKC_ERR_ARGUMENT, f"prefill: {m} rows, outside 1..{self.R}.")
        self.m = m
        addrs = {n: getattr(self, n).ptr for n in ("x", "a", "a_hi", "a_lo", "qkv", "att", "tmp", "x1", "gu", "act")}
        addrs.update(w_hi=self.w_hi.ptr if self.w_hi is not None else 0,
                     w_lo=self.w_lo.ptr if self.w_lo is not None else 0)
        rs4 = 4 * self.rs
        addrs.update(tokens=self.rows_buf.ptr, pos=self.rows_buf.ptr + rs4, slot=self.rows_buf.ptr + 2 * rs4,
                     part=[b.ptr for b in self.part])
        addrs.update({n: b.ptr for n, b in self.moe.items()})
        return [Launch(k, p, b) for k, p, b in _host.prefill_launches(
            self.eng.launch_args(), self.R, self.chunk, self.positions, self.one_slot, addrs, m)]

    def set_rows(self, tokens, positions, slots) -> int:
        """The rows of a run: tokens, positions, and each row's slot or,
        with a paged cache, its block table [m, table_len]."""
        tokens = np.asarray(tokens, np.uint32)
        m = len(tokens)
        slots = np.asarray(slots, np.uint32)
        if self.eng.s.paged and slots.shape != (m, self.seq):
            raise N.Refused(N.FKC_ERR_ARGUMENT, f"prefill: block tables of shape {slots.shape}, not ({m}, {self.seq}).")
        if m > self.R:
            raise N.Refused(N.FKC_ERR_ARGUMENT, f"prefill: {m} rows, more than {self.R}.")
        if m and int(np.max(positions)) >= self.positions:
            raise N.Refused(N.FKC_ERR_ARGUMENT,
                            f"prefill: position {int(np.max(positions))} is past the {self.positions} it was sized for.")
        self.eng.check_rows(tokens, positions, slots)
        if self.one_slot and m and len(np.unique(slots.reshape(m, -1), axis=0)) != 1:
            raise N.Refused(N.FKC_ERR_ARGUMENT, "prefill: a one-slot prefill's rows sit in more than one slot.")
        host = np.zeros(self.rows_words, np.uint32)
        host[:m] = tokens
        host[self.rs:self.rs + m] = np.asarray(positions, np.uint32)
        host[2 * self.rs:2 * self.rs + m * self.seq] = slots.reshape(-1)
        self.rows_buf.upload(host)
        return m

    def graph(self, m: int) -> N.Graph:
        """The captured prefill of m rows (one graph a row count)."""
        g = self.graphs.get(m)
        if g is None:
            launches = self.launches(m)
            self.ctx.set_pdl(False)
            self.ctx.capture_begin()
            try:
                for L in launches:
                    self.eng._run(L)
            finally:
                g = self.ctx.capture_end()
            self.graphs[m] = g
        return g

    def run(self, tokens, positions, slots) -> None:
        m = self.set_rows(tokens, positions, slots)
        self.graph(m).launch()

    def gemm_flops(self, rows: int) -> int:
        """Useful flops of the GEMMs over `rows` rows (2 a multiply-add); with
        routed experts only the attention's projections are GEMMs."""
        s = self.eng.s
        per = sum(self.eng.layer_sizes()[:4]) if s.experts else self.eng.layer_elems - 2 * s.d_model
        return 2 * rows * s.layers * per

    def close(self) -> None:
        """Destroys the graphs and frees the TF32 halves and scratch."""
        for g in self.graphs.values():
            g.destroy()
        self.graphs = {}
        bufs = [self.rows_buf, self.x, self.a, self.a_hi, self.a_lo, self.qkv, self.att, self.tmp, self.x1, self.gu,
                self.act] + self.part + list(self.moe.values())
        for b in bufs + [b for b in (self.w_hi, self.w_lo) if b is not None]:
            b.free()
        self.moe = {}


def prompt_rows(prompts, slots):
    """Every prompt's rows but its last: (tokens, positions, slots)."""
    prompts = [np.asarray(p, np.uint32) for p in prompts]
    toks = np.concatenate([p[:-1] for p in prompts])
    poss = np.concatenate([np.arange(len(p) - 1, dtype=np.uint32) for p in prompts])
    sl = np.concatenate([np.full(len(p) - 1, s, np.uint32) for p, s in zip(prompts, slots)])
    return toks, poss, sl


def prompt_chunks(pre: Prefill, toks, poss, sl) -> list:
    """The (start, rows) runs a prefill takes the rows in: R at a time, and
    for a one-slot prefill never across a slot."""
    out, i = [], 0
    while i < len(toks):
        j = min(i + pre.R, len(toks))
        if pre.one_slot:
            j = i + int(np.argmax(np.append(sl[i:j] != sl[i], True)))
        out.append((i, j - i))
        i = j
    return out


def prompt_then_decode(eng: Llama, pre: Prefill, prompts, slots) -> np.ndarray:
    """Prefill each prompt's rows but its last into its slot (R rows at a
    time; one prompt a run for a one-slot prefill), then one decode step over
    the batch from each prompt's last token: the first generated ids."""
    toks, poss, sl = prompt_rows(prompts, slots)
    for i, m in prompt_chunks(pre, toks, poss, sl):
        pre.run(toks[i:i + m], poss[i:i + m], sl[i:i + m])
    eng.set_rows([p[-1] for p in prompts], [len(p) - 1 for p in prompts], slots)
    return eng.step()
