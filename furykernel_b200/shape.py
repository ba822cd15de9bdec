"""The shape of a Llama-shaped decoder: dimensions, element types, the KV
cache's layout (a ring, or a paged pool) and routed experts. The engine,
the prefill, the tensor-parallel sharding and the host library's launch
lists (libfurykernel_host.so, fkh_llama_shape) all take it."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class LlamaShape:
    d_model: int = 4096
    heads: int = 32
    kv_heads: int = 32
    head_dim: int = 128
    ffn: int = 11008
    vocab: int = 32000
    layers: int = 32
    theta: float = 10000.0
    eps: float = 1e-5
    slots: int = 1  # sequences the ring holds
    length: int = 4096  # ring length
    positions: int = 4096  # bound of the positions a row may have
    # Every weight's element type: "f32", "bf16" (the reference's,
    # Build.hs:171-175) or "f16" (Check.hs:105-111).
    weights: str = "f32"
    # The KV caches' element type: "f32", "bf16" (CacheBF16) or "f16"
    # (CacheF16, Graph.hs:165-180).
    cache: str = "f32"
    # A paged cache (Graph.hs:144-152) instead of the ring: a pool of `blocks`
    # blocks of `block_size` positions a layer, which each row lists in its
    # block table of table_len entries. 0: the ring of `slots` and `length`.
    blocks: int = 0
    block_size: int = 0
    # Routed experts in place of the dense FFN: `experts` of ffn each, every
    # row taking its top_k (experts 0: the dense SiLU-gated FFN).
    experts: int = 0
    top_k: int = 2
    # Each chosen expert's weight times its own scale (the route's expert
    # scale, RouteSpec, Graph.hs:249-257): a weight [experts] after the router.
    expert_scale: bool = False

    @property
    def q_width(self):
        return self.heads * self.head_dim

    @property
    def kv_width(self):
        return self.kv_heads * self.head_dim

    @property
    def paged(self):
        return self.block_size > 0

    @property
    def table_len(self):
        """Block-table entries a row has: enough blocks for every position."""
        return (self.positions + self.block_size - 1) // self.block_size if self.paged else 0
