"""The Llama engine on the device: a Llama-shaped model's weights, KV
arena and row buffers, its decode step's launch list, and that list captured
as one CUDA graph and replayed a step at a time (host token ids in, greedy
ids out).

The launch list comes from the C++ host library (libfurykernel_host.so,
fkh_llama_launches): the programs of the embedding, a layer and the head
(src/FuryKernel/Program/Build.hs), planned as the reference plans them
(src/FuryKernel/Program/Plan.hs), each step lowered to one launch of a
kernel in the target's table, then the engine's rewrites (the SiLU-gate on
interleaved gate/up tiles, tensor parallelism over peer memory or NCCL, the
fused decode attention) and the split-K choice. KV caches are Ring arenas
or paged pools per layer.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _native as N
from .shape import LlamaShape


@dataclass
class Launch:
    kernel: str
    params: dict
    bufs: list

    def run(self, ctx: N.Context) -> None:
        ctx.launch(self.kernel, self.params, self.bufs)


# A kernel's element-type form: the f32 entry's name, or with the suffix of
# its 16-bit weights or its 16-bit KV caches (target.WEIGHT_SUFFIX,
# target.CACHE_SUFFIX).
def kernel_form(kernel: str) -> tuple:
    """(the f32 entry's name, the suffix of the form)."""
    for suffix in ("_wbf16", "_wf16", "_kvbf16", "_kvf16"):
        if kernel.endswith(suffix):
            return kernel[:-len(suffix)], suffix
    return kernel, ""


class Llama:
    """A Llama-shaped model on one device, or one rank of a Megatron-style
    tensor-parallel group: the weights (seeded on the device, or given), the
    Ring KV arena, the plans of the embedding, a layer and the head, and the
    captured decode step. Activations are f32; the weights and the caches
    are f32, bf16 or f16, as the shape says (`weights`, `cache`).

    With `world` ranks, each holds heads/world query and KV heads with their
    rows of q/k/v and columns of o, ffn/world rows of gate and up with their
    columns of down (column then row parallel), and vocab/world rows of the
    tied LM head; the embedding table is whole on every rank. The
    row-parallel projections (o, down) leave partial sums that an NCCL
    allreduce adds before their residual epilogue runs; the head's greedy
    candidates, one a shard, are gathered and picked.
    """

    def __init__(self, ctx: N.Context, shape: LlamaShape, batch: int, seed: int = 2026, chunk: int = 32,
                 pdl: bool = True, prefill_kv: float | None = None, rank: int = 0, world: int = 1,
                 host_weights=None, peer_exchange: bool = True, fuse_attention: bool | None = None,
                 selection: str | None = None, gated: bool = False, store_gelus: bool = False,
                 prefetch_attention: int = 0, prefetch_gemv: int | None = None):
        import dataclasses

        full = shape
        for what, n in (("heads", full.heads), ("kv_heads", full.kv_heads), ("ffn", full.ffn),
                        ("vocab", full.vocab)):
            if n % world:
                raise N.Refused(N.FKC_ERR_ARGUMENT, f"{what} {n} does not split over {world} ranks.")
        s = dataclasses.replace(full, heads=full.heads // world, kv_heads=full.kv_heads // world,
                                ffn=full.ffn // world)
        self.ctx, self.full, self.s, self.m = ctx, full, s, batch
        # The layer's plan options: a route in a step of its own (optGated),
        # gelus stored by their own step (optStoreGelus).
        self.gated, self.store_gelus = gated, store_gelus
        self.rank, self.world = rank, world
        # Bytes of a weight and of a cache element.
        self.wb = {"f32": 4, "bf16": 2, "f16": 2}.get(s.weights)
        self.cb = {"f32": 4, "bf16": 2, "f16": 2}.get(s.cache)
        if self.wb is None or self.cb is None:
            raise N.Refused(N.FKC_ERR_ARGUMENT, f"no kernels for {s.weights} weights and {s.cache} caches.")
        if s.experts > 1024:
            raise N.Refused(N.FKC_ERR_ARGUMENT, "routed experts: at most 1024 experts.")
        if s.experts and s.expert_scale and (s.experts * self.wb) % 16:
            raise N.Refused(N.FKC_ERR_ARGUMENT, "expert scales: the experts' scales must fill whole 16 bytes, so that "
                                                "the weights after them start on a 16-byte boundary.")
        if self.wb == 2 and any(n % 8 for n in (s.d_model, s.q_width, s.kv_width, s.ffn)):
            raise N.Refused(N.FKC_ERR_ARGUMENT, "16-bit weights: d_model, the q and kv widths and ffn must be "
                            "multiples of 8, so that every weight starts on a 16-byte boundary.")
        # For decode batches the streaming and batched GEMVs take (up to 64
        # rows), the arena interleaves gate and up rows (gate_i at row 2i, up_i at
        # 2i + 1), so that the [gate; up] step computes mlp_act = silu(gate) *
        # up on its own tiles and stores it, and the down step reads it: the
        # same bits as recomputing it in the down step, computed once.
        self.gate_up_interleaved = batch <= 64
        # Tensor parallelism's sums travel through peer memory (the context's
        # peer set, tp.init) for the batches the streaming GEMV takes; larger
        # batches use NCCL.
        # (Routed experts sum their ranks' shares by NCCL.)
        self.peer_exchange = world > 1 and batch <= 4 and peer_exchange and not s.experts
        self.vocab_local = full.vocab // world
        # Weights: per layer [q;k;v], o, [gate;up], down, two norms; then the
        # tied embedding/LM head and the final norm. N(0, 0.02), the norm
        # gains too (the configs give no other law for them).
        d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
        self.layer_elems = sum(self.layer_sizes())
        wb = self.wb
        self.arena = ctx.alloc(wb * (s.layers * self.layer_elems + full.vocab * d + d))
        fill = self._fill(s.weights)
        if host_weights is None:
            # A rank's layer shards from its own seed; the embedding and the
            # norms alike on every rank (16-bit: the same values, rounded).
            layers = N.DeviceBuffer(ctx, self.arena.ptr, wb * s.layers * self.layer_elems)
            fill(layers, seed + 7919 * rank, 0.0, 0.02)
            rest = N.DeviceBuffer(ctx, self.embed_ptr(), wb * (full.vocab * d + d))
            fill(rest, seed + 104729, 0.0, 0.02)
            for l in range(s.layers):
                w = self.layer_weights(l)
                fill(N.DeviceBuffer(ctx, w["attn_norm"], 2 * wb * d), seed + 3 * l + 1, 0.0, 0.02)
                if s.experts:  # the router (and the experts' scales) whole on every rank
                    fill(N.DeviceBuffer(ctx, w["router"], wb * s.experts * d), seed + 611953 + l, 0.0, 0.02)
                    if s.expert_scale:
                        fill(N.DeviceBuffer(ctx, w["expert_scale"], wb * s.experts), seed + 711957 + l, 1.0, 0.25)
        else:
            self.arena.upload(host_weights)
        self.cos, self.sin = ctx.rope_tables(s.theta, s.head_dim, s.head_dim // 2, s.positions)
        self.kbase, self.vbase = self._kv_arena()
        # A paged cache's kernels reach each block through a table of the
        # blocks' addresses (the Paged layout, src/FuryKernel/Program/
        # Graph.hs:144-152; tables, IR.hs:400-429): [layers][blocks] u64 for
        # the keys and for the values, here pointing into the pool's blocks
        # (set_block_addresses points them anywhere else).
        self.ktab = self.vtab = None
        if s.paged:
            self.ktab, self.vtab = self._block_table(self.kbase), self._block_table(self.vbase)
        if prefill_kv is not None:
            kv = s.layers * self._kv_units() * s.kv_heads * self._kv_unit_len() * s.head_dim
            cfill = self._fill(s.cache)
            cfill(N.DeviceBuffer(ctx, self.kbase, self.cb * kv), seed + 1 + 17 * rank, 0.0, prefill_kv)
            cfill(N.DeviceBuffer(ctx, self.vbase, self.cb * kv), seed + 2 + 17 * rank, 0.0, prefill_kv)
        m = batch
        # A step's row inputs in one buffer, so that one copy brings them in:
        # the tokens, the positions, the slots, each part on a 16-byte
        # boundary as every buffer a kernel binds (leastAlign,
        # src/FuryKernel/Type.hs:66-71).
        # With a paged cache the third part is the rows' block tables
        # [m, table_len] instead of their slots.
        self.row_stride = (m + 3) // 4 * 4
        seq = s.table_len if s.paged else 1
        self.rows_words = 2 * self.row_stride + (m * seq + 3) // 4 * 4
        self.rows = ctx.zeros(self.rows_words, np.uint32)
        rs = 4 * self.row_stride
        self.tokens = N.DeviceBuffer(ctx, self.rows.ptr, 4 * m, np.uint32, (m,))
        self.pos = N.DeviceBuffer(ctx, self.rows.ptr + rs, 4 * m, np.uint32, (m,))
        self.slot = N.DeviceBuffer(ctx, self.rows.ptr + 2 * rs, 4 * m * seq, np.uint32,
                                   (m, seq) if s.paged else (m,))
        self.out_ids = ctx.zeros(m, np.uint32)
        self.x = ctx.zeros((m, d))
        self.x1 = ctx.zeros((m, d))
        self.partial = ctx.zeros((m, d))
        self.qkv = ctx.zeros((m, qw + 2 * kvw))
        self.att = ctx.zeros((m, qw))
        self.gu = ctx.zeros((m, 2 * f))
        self.act = ctx.zeros((m, f))
        if s.experts:  # the routed FFN's rows: the normed row, logits, route, experts' in and out
            e, k = s.experts, s.top_k
            self.moe = {"mlp_in": ctx.zeros((m, d)), "router_logits": ctx.zeros((m, e)),
                        "route_ids": ctx.zeros((m, k), np.uint32), "route_weights": ctx.zeros((m, k)),
                        "experts_gu": ctx.zeros((m, k * 2 * f)), "experts_act": ctx.zeros((m, k * f)),
                        "experts_out": ctx.zeros((m, k * d))}
        self.logits = ctx.zeros((m, self.vocab_local))
        self.pairs = ctx.zeros(2 * m, np.uint32)
        self.pairs_all = ctx.zeros(2 * m * world, np.uint32)
        self.chunk = chunk
        self.max_splits = (s.positions + chunk - 1) // chunk
        self.part = [ctx.zeros(m * s.heads * self.max_splits), ctx.zeros(m * s.heads * self.max_splits),
                     ctx.zeros(m * s.heads * self.max_splits * s.head_dim)]
        self.pdl = pdl
        # The weight bytes each streaming GEMV brings toward L2 by bulk
        # prefetch before it waits for its predecessor (0: its first lines
        # only), and the next GEMV's weight bytes an attention launch brings
        # toward L2 while it runs. Measured on config 5 (same process,
        # repeated): 64 MiB a GEMV takes 2% off the batch-1 step and adds 2%
        # at batch 4, so it is the default at batch 1 only; the attention's
        # prefetch competes with its own KV loads and is off.
        self.prefetch_attention = prefetch_attention
        self.prefetch_gemv = (64 << 20 if batch == 1 else 0) if prefetch_gemv is None else prefetch_gemv
        # The decode step's KV store and attention as one launch
        # (attend_decode), for rows in distinct slots (set_rows checks): by
        # default for the small batches whose steps are launch-bound (one
        # launch a layer fewer); at batch 16 the separate store measured
        # faster (0.617 against 0.658 ms a layer at context 2048).
        # (No fused form reads a paged cache.)
        if fuse_attention is None:
            fuse_attention = m <= 4
        # (A paged cache's fused form needs every block-table entry
        # distinct: set_rows checks the tables it uploads.)
        self.fuse_attention = fuse_attention and m <= 64
        # A committed selection (furykernel_b200.select): each GEMV shape's
        # split-K, the same at every batch.
        self.splits = {}
        if selection is not None:
            from . import select

            self.splits = select.splits_for(self, selection)
        self.launches = self._launches()
        self.graph = None

    # -- layout
    def _kv_units(self) -> int:
        """A layer's ring slots, or its pool's blocks."""
        return self.s.blocks if self.s.paged else self.s.slots

    def _kv_unit_len(self) -> int:
        """Positions a slot or a block holds."""
        return self.s.block_size if self.s.paged else self.s.length

    def _kv_arena(self):
        import ctypes

        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        s = self.s
        N.check(N.lib().fkc_kv_arena_elem(self.ctx.handle, s.layers, self._kv_units(), s.kv_heads,
                                          self._kv_unit_len(), s.head_dim, self.cb, ctypes.byref(k),
                                          ctypes.byref(v)))
        return k.value, v.value

    LAYER_ORDER = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "attn_norm",
                   "mlp_norm")
    # With routed experts: the router and the experts' tables (each entry
    # [2 ffn, d] gate/up and [d, ffn] down) in place of the dense FFN.
    MOE_ORDER = ("q_proj", "k_proj", "v_proj", "o_proj", "router", "experts_gate_up", "experts_down", "attn_norm",
                 "mlp_norm")

    def layer_order(self) -> tuple:
        if self.s.experts and getattr(self.s, "expert_scale", False):  # the scales after the router
            return self.MOE_ORDER[:5] + ("expert_scale",) + self.MOE_ORDER[5:]
        return self.MOE_ORDER if self.s.experts else self.LAYER_ORDER

    def _fill(self, t: str):
        """The seeded normal fill of elements of type t (16-bit: the f32
        fill's values, rounded)."""
        return {"f32": self.ctx.fill_normal, "bf16": self.ctx.fill_normal_bf16,
                "f16": self.ctx.fill_normal_f16}[t]

    def layer_sizes(self) -> list:
        s = self.s
        d, qw, kvw, f = s.d_model, s.q_width, s.kv_width, s.ffn
        if s.experts:
            scale = [s.experts] if getattr(s, "expert_scale", False) else []
            return [qw * d, kvw * d, kvw * d, d * qw, s.experts * d] + scale + \
                [s.experts * 2 * f * d, s.experts * d * f, d, d]
        return [qw * d, kvw * d, kvw * d, d * qw, f * d, f * d, d * f, d, d]

    def layer_weights(self, l: int) -> dict:
        base = self.arena.ptr + self.wb * l * self.layer_elems
        off, at = {}, 0
        for name, n in zip(self.layer_order(), self.layer_sizes()):
            off[name] = base + self.wb * at
            at += n
        return off

    def embed_ptr(self) -> int:
        return self.arena.ptr + self.wb * self.s.layers * self.layer_elems

    def final_norm_ptr(self) -> int:
        return self.embed_ptr() + self.wb * self.full.vocab * self.full.d_model

    def block_bytes(self) -> int:
        """Bytes of one block of a paged cache: kv_heads x block_size x head_dim elements."""
        s = self.s
        return self.cb * s.kv_heads * s.block_size * s.head_dim

    def _block_table(self, pool: int):
        """A [layers][blocks] u64 table of the pool's blocks' addresses."""
        s = self.s
        addr = pool + np.arange(s.layers * s.blocks, dtype=np.uint64) * np.uint64(self.block_bytes())
        return self.ctx.to_device(addr.reshape(s.layers, s.blocks))

    def set_block_addresses(self, layer: int, keys, values) -> None:
        """Points a paged cache's blocks of one layer at arrays of the
        caller's (each block_bytes() long, 16-byte aligned, wherever it was
        allocated): `keys[b]` and `values[b]` the device addresses of block
        b's keys and values. The launch list binds the tables, so a captured
        step reads the new addresses on its next replay."""
        s = self.s
        if not s.paged:
            raise N.Refused(N.FKC_ERR_ARGUMENT, "set_block_addresses: the engine's caches are Ring caches.")
        if not 0 <= layer < s.layers:
            raise N.Refused(N.FKC_ERR_ARGUMENT, f"set_block_addresses: layer {layer} of {s.layers}.")
        rows = []
        for what, a in (("key", keys), ("value", values)):
            a = np.asarray(a, np.uint64)
            if a.shape != (s.blocks,):
                raise N.Refused(N.FKC_ERR_ARGUMENT, f"set_block_addresses: {a.size} {what} blocks, not {s.blocks}.")
            if np.any(a == 0) or np.any(a % 16):
                raise N.Refused(N.FKC_ERR_ARGUMENT, f"set_block_addresses: a {what} block's address is null or "
                                                    "not 16-byte aligned.")
            rows.append(a)
        for tab, row in ((self.ktab, rows[0]), (self.vtab, rows[1])):
            N.check(N.lib().fkc_buf_upload(self.ctx.handle, tab.ptr + 8 * layer * s.blocks, row.ctypes.data,
                                           row.nbytes))

    def kv_layer(self, l: int):
        """A layer's caches as its launches bind them: a ring's slab of the
        arena, or a paged cache's row of each block-address table."""
        s = self.s
        if s.paged:
            return self.ktab.ptr + 8 * l * s.blocks, self.vtab.ptr + 8 * l * s.blocks
        per = self.cb * self._kv_units() * s.kv_heads * self._kv_unit_len() * s.head_dim
        return self.kbase + l * per, self.vbase + l * per

    # -- the step's launches
    def launch_addresses(self) -> dict:
        """The device addresses the decode step's launches bind (the C++
        host library's fkh_llama_desc)."""
        kb, vb = (self.ktab.ptr, self.vtab.ptr) if self.s.paged else (self.kbase, self.vbase)
        return {"arena": self.arena.ptr, "kbase": kb, "vbase": vb, "cos_t": self.cos.ptr,
                "sin_t": self.sin.ptr, "tokens": self.tokens.ptr, "pos": self.pos.ptr, "slot": self.slot.ptr,
                "x": self.x.ptr, "x1": self.x1.ptr, "qkv": self.qkv.ptr, "att": self.att.ptr, "gu": self.gu.ptr,
                "act": self.act.ptr, "logits": self.logits.ptr, "out_ids": self.out_ids.ptr,
                "partial": self.partial.ptr, "pairs": self.pairs.ptr, "pairs_all": self.pairs_all.ptr,
                "part": [b.ptr for b in self.part],
                **{name: buf.ptr for name, buf in getattr(self, "moe", {}).items()}}

    def _launches(self) -> list:
        """The decode step's launches, from libfurykernel_host.so
        (fkh_llama_launches): the plans of the embedding, a layer and the
        head lowered to table launches, then the rewrites below."""
        from . import _host

        return [Launch(k, p, b) for k, p, b in _host.llama_launches(*self.launch_args())]

    def launch_args(self) -> tuple:
        """fkh_llama_desc's fields: the shape, the batch, the rank, the
        choices and the addresses."""
        return (self.full, self.m, self.rank, self.world, self.ctx.sms, self.chunk, self.gate_up_interleaved,
                self.peer_exchange, self.fuse_attention, self.launch_addresses(), getattr(self, "splits", None),
                getattr(self, "gated", False), getattr(self, "store_gelus", False))

    def _run(self, L: Launch) -> None:
        if L.kernel == "__allreduce__":
            N.check(N.lib().fkc_allreduce_sum_f32(self.ctx.handle, L.bufs[0], L.params["count"]))
        elif L.kernel == "__allgather__":
            N.check(N.lib().fkc_allgather_u32(self.ctx.handle, L.bufs[0], L.bufs[1], L.params["count"]))
        else:
            L.run(self.ctx)

    ATTEND = ("attend_decode", "attend_split")

    def _next_gemv_weights(self, i: int):
        """(address, bytes) of the weights of the first GEMV after launch i."""
        for L in self.launches[i + 1:]:
            if L.kernel.startswith("gemv"):
                nbytes = self.wb * L.params["n"] * L.params["k"]
                return L.bufs[0], nbytes - nbytes % 16
        return 0, 0

    def _run_all(self) -> None:
        """The step's launches in order. Every streaming GEMV gets its own
        L2 prefetch budget (prefetch_gemv, fkc_set_prefetch); an attention
        launch brings the next GEMV's weights toward L2 while it runs (up to
        prefetch_attention bytes, fkc_set_l2_prefetch)."""
        if self.prefetch_gemv:
            self.ctx.set_prefetch(self.prefetch_gemv)
        try:
            for i, L in enumerate(self.launches):
                att = self.prefetch_attention > 0 and L.kernel.startswith(self.ATTEND)
                if att:
                    ptr, nbytes = self._next_gemv_weights(i)
                    self.ctx.set_l2_prefetch(ptr, min(nbytes, self.prefetch_attention))
                try:
                    self._run(L)
                finally:
                    if att:
                        self.ctx.set_l2_prefetch(0, 0)
        finally:
            if self.prefetch_gemv:
                self.ctx.set_prefetch(0)

    def run_eager(self) -> None:
        self.ctx.set_pdl(False)
        self._run_all()

    def capture(self) -> N.Graph:
        if self.graph is None:
            self.ctx.set_pdl(self.pdl)
            self.ctx.capture_begin()
            try:
                self._run_all()
            finally:
                g = self.ctx.capture_end()
                self.ctx.set_pdl(False)
            self.graph = g
        return self.graph

    def check_rows(self, tokens, positions, slots) -> None:
        """Refuses row inputs the kernels would index past their buffers
        with: ids past the vocabulary, positions past the RoPE tables, slots
        past the KV arena (or, paged, block-table entries past the pool)."""
        s = self.s
        seq = ("block", slots, s.blocks) if s.paged else ("slot", slots, s.slots)
        for what, v, bound in (("token", tokens, self.full.vocab), ("position", positions, s.positions), seq):
            v = np.asarray(v)
            if v.size and int(v.max()) >= bound:
                raise N.Refused(N.FKC_ERR_ARGUMENT, f"a {what} {int(v.max())} is past the engine's {bound}.")

    def set_rows(self, tokens, positions, slots=None) -> None:
        """A step's rows: tokens, positions, and each row's ring slot or,
        with a paged cache, its block table [m, table_len]."""
        if self.s.paged:
            if slots is None:
                raise N.Refused(N.FKC_ERR_ARGUMENT, "a paged cache's rows need their block tables.")
            slots = np.asarray(slots, np.uint32)
            if slots.shape != (self.m, self.s.table_len):
                raise N.Refused(N.FKC_ERR_ARGUMENT, f"block tables of shape {slots.shape}, not "
                                                    f"({self.m}, {self.s.table_len}).")
        slots = np.asarray(slots if slots is not None else np.arange(self.m), np.uint32)
        self.check_rows(tokens, positions, slots)
        if self.fuse_attention and np.unique(slots).size != slots.size:
            what = "every block-table entry distinct" if self.s.paged else "its rows in distinct slots"
            raise N.Refused(N.FKC_ERR_ARGUMENT, f"a decode step needs {what} (the fused attention stores a row's "
                                                "key while the others read).")
        self.tokens.upload(np.asarray(tokens, np.uint32))
        self.pos.upload(np.asarray(positions, np.uint32))
        self.slot.upload(slots)

    def step(self) -> np.ndarray:
        self.capture().launch()
        self.ctx.sync()
        return self.out_ids.download()

    def launch_count(self) -> int:
        """Kernels of this library a step launches (collectives excluded)."""
        return sum(1 for L in self.launches if not L.kernel.startswith("__"))

    def weight_bytes(self) -> int:
        """The weights a step streams on this rank: the layers' shards, the
        LM head's vocabulary rows and the final norm."""
        s = self.s
        return self.wb * (s.layers * self.layer_elems + self.vocab_local * s.d_model + s.d_model)

    def algorithmic_bytes(self, contexts) -> int:
        """Bytes a decode step must move on this rank: every weight once, each
        row's keys and values over its context, per layer."""
        s = self.s
        kv = sum(2 * s.kv_heads * s.head_dim * self.cb * (int(c) + 1) for c in contexts) * s.layers
        return self.weight_bytes() + kv


def shard_weights(full: LlamaShape, layers: list, embed: np.ndarray, final_norm: np.ndarray, rank: int,
                  world: int, interleave: bool = False) -> np.ndarray:
    """One rank's weight arena from the whole model's host weights, in the
    engine's layout: per layer q/k/v rows of its heads, o's columns of its
    heads, gate/up rows of its ffn slice, down's columns of that slice,
    the norms; then the whole embedding and the final norm.

    `layers` holds per layer the f32 arrays q [H*hd, d], k and v
    [KV*hd, d], o [d, H*hd], gate and up [F, d], down [d, F], attn_norm and
    mlp_norm [d]; with routed experts, router [E, d], expert_scale [E] (with
    the shape's expert_scale), egu [E, 2F, d] (each expert's gate rows, then
    its up rows) and edn [E, d, F] in place of gate, up and down. A rank
    holds the whole router and scales and, of every expert, the gate and up
    rows and the down columns of its ffn slice."""
    hd, d = full.head_dim, full.d_model
    hq, hk, fl = full.heads // world, full.kv_heads // world, full.ffn // world
    qs = slice(rank * hq * hd, (rank + 1) * hq * hd)
    ks = slice(rank * hk * hd, (rank + 1) * hk * hd)
    fs = slice(rank * fl, (rank + 1) * fl)
    parts = []
    for w in layers:
        parts += [w["q"][qs], w["k"][ks], w["v"][ks], np.ascontiguousarray(w["o"][:, qs])]
        if full.experts:
            f = full.ffn
            egu = np.concatenate([w["egu"][:, fs], w["egu"][:, f + rank * fl:f + (rank + 1) * fl]], axis=1)
            parts += [w["router"]] + ([w["expert_scale"]] if full.expert_scale else [])
            parts += [egu, np.ascontiguousarray(w["edn"][:, :, fs]), w["attn_norm"], w["mlp_norm"]]
            continue
        gate, up = w["gate"][fs], w["up"][fs]
        gu = np.stack([gate, up], axis=1).reshape(2 * fl, d) if interleave else [gate, up]
        parts += [gu] if interleave else gu
        parts += [np.ascontiguousarray(w["down"][:, fs]), w["attn_norm"], w["mlp_norm"]]
    parts += [embed, final_norm]
    return np.concatenate([np.ascontiguousarray(a, np.float32).ravel() for a in parts])
