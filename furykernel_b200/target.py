"""The CUDA target as the reference's backend interface sees it.

`Target Cuda` (src/FuryKernel/Target.hs:39-70) gives a B200's limits;
`cuda` is a `Backend` (src/FuryKernel/Backend.hs:156-162) whose
`backend_lower` resolves each checked kernel to the prebuilt sm_100a entry of
the same name and ABI hash, and returns a `Lowered` with one
`LoweredKernel` a kernel (Backend.hs:164-228). Kernels that no entry
implements, or whose ABI differs from the entry's, are refused as findings,
as checkOverrides words an ABI difference (src/FuryKernel/Abi.hs:172-190).

SPEC_KERNELS declares this path's spec kernels' interfaces: what the eDSL
kernels of each planned step bind. The library's table must agree with
them hash for hash (tests/test_boundary.py).
"""

from __future__ import annotations

from dataclasses import dataclass, field

from . import abi as A
from .abi import Buffer, DimRange, KernelSig, Param, Table


@dataclass(frozen=True)
class TargetCaps:
    """TargetCaps (Target.hs:73-82)."""

    name: str
    simd_width: int
    max_threads: int
    tg_mem_bytes: int
    max_buffers: int
    lane_load_max: int
    fragments: tuple = ()


# A B200 (sm_100a): 32-lane warps, 1024 threads a block, 227 KiB of shared
# memory a block, 16-byte lane loads; fragments are not this target's (its
# tensor-core tiles are tcgen05's, inside hand-written kernels).
CUDA = TargetCaps("Cuda", 32, 1024, 232448, 31, 16, ())


@dataclass
class Finding:
    """A refusal (src/FuryKernel/Finding.hs:11-17)."""

    rule: str
    message: str


@dataclass
class LoweredKernel:
    """One kernel's launch table (Backend.hs:203-228)."""

    name: str
    entry: str
    abi: A.Abi
    ir_hash: int
    threads: int
    groups: str
    bindings: list
    params_binding: int | None
    tg_memory: int


@dataclass
class Lowered:
    language: str
    options: dict
    source: str
    kernels: list = field(default_factory=list)


def _f32(name, access="read"):
    return Buffer(name, access, "f32")


def _u32(name, access="read"):
    return Buffer(name, access, "u32")


def _bf16(name, access="read"):
    return Buffer(name, access, "bf16")


def _dim(name, lo, hi, mult=1):
    return Param(name, "u32", DimRange(lo, hi, mult))


def _u(name):
    return Param(name, "u32")


def _f(name):
    return Param(name, "f32")


_GEMV = [_dim("n", 1, 1048576), _dim("k", 4, 65536, 4), _dim("m", 1, 65535), _dim("split", 1, 8), _u("ldx"),
         _u("ldy")]
_MAX = 4294967295

SPEC_KERNELS = {
    k.name: k
    for k in [
        KernelSig("reduce_groups", [_f32("x"), _f32("partials", "write")], [_dim("n", 1, 2147483648)], threads=256),
        KernelSig("reduce_final", [_f32("partials"), _f32("y", "write")], [_dim("count", 1, 16777216)], threads=256),
        KernelSig("rmsnorm_rows", [_f32("x"), _f32("gamma"), _f32("y", "write")],
                  [_dim("rows", 1, 1048576), _dim("h", 4, 16384, 4), _f("eps"), _f("factor")]),
        KernelSig("softmax_rows", [_f32("x"), _f32("y", "write")], [_dim("rows", 1, 1048576), _dim("h", 4, 16384, 4)]),
        KernelSig("gemv", [_f32("w"), _f32("x"), _f32("y", "write")], _GEMV),
        KernelSig("gemv_add", [_f32("w"), _f32("x"), _f32("r"), _f32("y", "write")], _GEMV + [_u("ldr")]),
        KernelSig("gemv_rmsnorm", [_f32("w"), _f32("x"), _f32("gamma"), _f32("y", "write")],
                  _GEMV + [_f("eps"), _f("factor")]),
        KernelSig("gemv_rmsnorm_silu", [_f32("w"), _f32("x"), _f32("gamma"), _f32("y", "write")],
                  _GEMV + [_f("eps"), _f("factor")], threads=512),
        KernelSig("gemv_silu", [_f32("w"), _f32("x"), _f32("y", "write")], _GEMV + [_u("up_off")]),
        KernelSig("gemv_silu_add", [_f32("w"), _f32("x"), _f32("r"), _f32("y", "write")],
                  _GEMV + [_u("ldr"), _u("up_off")]),
        KernelSig("kv_store_ring",
                  [_f32("qkv"), _f32("cos"), _f32("sin"), _u32("pos"), _u32("slot"), _f32("k_cache", "read_write"),
                   _f32("v_cache", "read_write")],
                  [_dim("m", 1, 65535), _dim("kv_heads", 1, 1024), _dim("d", 2, 2048, 2), _dim("length", 1, _MAX),
                   _u("rotated"), _u("ldq"), _u("k_off"), _u("v_off")], threads=64),
        KernelSig("attend_split",
                  [_f32("qkv"), _f32("cos"), _f32("sin"), _u32("pos"), _u32("slot"), _f32("k_cache"),
                   _f32("v_cache"), _f32("part_m", "write"), _f32("part_l", "write"), _f32("part_acc", "write")],
                  [_dim("m", 1, 16384), _dim("heads", 1, 1024), _dim("kv_heads", 1, 1024), _dim("d", 128, 128),
                   _dim("length", 1, _MAX), _u("rotated"), _dim("chunk", 1, 256), _dim("max_splits", 1, 65535),
                   _u("ldq"), _u("q_off"), _f("scale")], threads=128),
        KernelSig("attend_decode",
                  [_f32("qkv"), _f32("cos"), _f32("sin"), _u32("pos"), _u32("slot"), _f32("k_cache", "read_write"),
                   _f32("v_cache", "read_write"), _f32("part_m", "write"), _f32("part_l", "write"),
                   _f32("part_acc", "write")],
                  [_dim("m", 1, 64), _dim("heads", 1, 1024), _dim("kv_heads", 1, 1024), _dim("d", 128, 128),
                   _dim("length", 1, _MAX), _u("rotated"), _dim("chunk", 1, 256), _dim("max_splits", 1, 65535),
                   _u("ldq"), _u("q_off"), _u("k_off"), _u("v_off"), _f("scale")], threads=128),
        KernelSig("attend_prompt",
                  [_f32("qkv"), _f32("cos"), _f32("sin"), _u32("pos"), _u32("slot"), _f32("k_cache"),
                   _f32("v_cache"), _f32("out", "write")],
                  [_dim("m", 1, 65535), _dim("heads", 1, 1024), _dim("kv_heads", 1, 1024), _dim("d", 128, 128),
                   _dim("length", 1, _MAX), _u("rotated"), _u("ldq"), _u("q_off"), _u("ldo"),
                   _dim("max_pos", 0, _MAX - 1), _f("scale")], threads=256),
        KernelSig("attend_combine",
                  [_f32("part_m"), _f32("part_l"), _f32("part_acc"), _u32("pos"), _f32("out", "write")],
                  [_dim("m", 1, 65535), _dim("heads", 1, 1024), _dim("d", 1, 1024), _dim("chunk", 1, 256),
                   _dim("max_splits", 1, 65535), _u("ldo")], threads=128),
        KernelSig("gather", [_f32("table"), _u32("tokens"), _f32("y", "write")],
                  [_dim("width", 4, 1048576, 4), _dim("m", 1, 65535), _f("factor")]),
        KernelSig("argmax", [_f32("x"), _u32("ids", "write")], [_dim("m", 1, 65535), _dim("n", 1, _MAX), _u("ldx")],
                  threads=1024),
        KernelSig("rope", [_f32("x"), _u32("pos"), _f32("cos"), _f32("sin"), _f32("y", "write")],
                  [_dim("m", 1, 65535), _dim("heads", 1, 65535), _dim("d", 2, 2048, 2), _u("rotated"), _u("ldx"),
                   _u("ldy")], threads=64),
        KernelSig("split_tf32", [_f32("x"), _f32("hi", "write"), _f32("lo", "write")], [_dim("n", 1, _MAX)]),
        KernelSig("gemm_tf32x3",
                  [_f32("a"), _f32("a_hi", "read_write"), _f32("a_lo", "read_write"), _f32("w_hi"), _f32("w_lo"),
                   _f32("c", "write")],
                  [_dim("M", 1, 1048576), _dim("N", 1, 1048576), _dim("K", 32, 1048576, 32), _u("ldc")],
                  threads=192),
        KernelSig("gemm_tf32x3w",
                  [_f32("a"), _f32("a_hi", "read_write"), _f32("a_lo", "read_write"), _f32("w"), _f32("c", "write")],
                  [_dim("M", 1, 1048576), _dim("N", 1, 1048576), _dim("K", 16, 1048576, 16), _u("ldc")],
                  threads=192),
        KernelSig("argmax_pairs", [_f32("x"), _u32("pairs", "write")],
                  [_dim("m", 1, 65535), _dim("n", 1, _MAX), _u("ldx"), _u("offset")], threads=1024),
        KernelSig("argmax_pick", [_u32("pairs"), _u32("ids", "write")], [_dim("shards", 1, 64), _dim("m", 1, 65535)]),
        KernelSig("argmax_scatter", [_f32("x")], [_dim("m", 1, 4), _dim("n", 1, _MAX), _u("ldx"), _u("offset")],
                  threads=1024),
        KernelSig("argmax_gather_pick", [_u32("ids", "write")], [_dim("m", 1, 4)]),
        KernelSig("gemv_scatter", [_f32("w"), _f32("x")],
                  [_dim("n", 1, 65536), _dim("k", 4, 65536, 4), _dim("m", 1, 4), _dim("split", 1, 8), _u("ldx"),
                   _dim("xbuf", 0, 1)], threads=512),
        *[KernelSig(name, [_f32("w"), _f32("r"), _f32("gamma"), _f32("xout", "write"), _f32("y", "write")],
                    [_dim("n", 1, 1048576), _dim("k", 4, 16384, 4), _dim("m", 1, 4), _dim("split", 1, 8), _u("ldr"),
                     _u("ldy"), _f("eps"), _f("factor"), _dim("xbuf", 0, 1)], threads=512)
          for name in ("gemv_reduce_rmsnorm", "gemv_reduce_rmsnorm_silu")],
        KernelSig("advance", [_u32("ids"), _u32("tokens", "write"), _u32("pos", "read_write")], [_dim("m", 1, 65535)]),
        KernelSig("add", [_f32("a"), _f32("b"), _f32("y", "write")], [_dim("n", 1, _MAX)]),
        KernelSig("silu_mul", [_f32("a"), _f32("b"), _f32("y", "write")], [_dim("n", 1, _MAX)]),
        KernelSig("silu_pairs", [_f32("x"), _f32("y", "write")], [_dim("n", 1, _MAX)]),
        KernelSig("gemv_bf16", [_bf16("w"), _bf16("x"), _bf16("y", "write")],
                  [_dim("n", 1, 1048576), _dim("k", 4, 65536, 4), _dim("m", 1, 16), _dim("pack", 4, 16, 4),
                   _dim("split", 1, 16), _u("ldx"), _u("ldy")], threads=512),
        # Routed experts (Graph.hs:306-340).
        KernelSig("route_topk", [_f32("x"), _u32("ids", "write"), _f32("ws", "write")],
                  [_dim("m", 1, 65535), _dim("n", 1, 1024), _dim("k", 1, 8), _u("ldx")], threads=32),
        KernelSig("route_topk_scaled", [_f32("x"), _f32("scale"), _u32("ids", "write"), _f32("ws", "write")],
                  [_dim("m", 1, 65535), _dim("n", 1, 1024), _dim("k", 1, 8), _u("ldx")], threads=32),
        KernelSig("gemv_routed", [_f32("table"), _u32("ids"), _f32("x"), _f32("y", "write")],
                  [_dim("entries", 1, 4096), _dim("n", 1, 1048576), _dim("kk", 4, 65536, 4), _dim("m", 1, 65535),
                   _dim("k", 1, 8), _dim("split", 1, 8), _u("ldx"), _u("ldy"), _u("per_rank")]),
        KernelSig("gated_gelu", [_f32("x"), _f32("y", "write")], [_dim("segments", 1, _MAX), _dim("f", 1, _MAX)]),
        KernelSig("combine_ranks_add", [_f32("r"), _f32("ws"), _f32("segs"), _f32("y", "write")],
                  [_dim("m", 1, 65535), _dim("k", 1, 8), _dim("d", 1, _MAX)]),
        # Paged caches (Graph.hs:144-152): a row's block table (indices)
        # instead of its slot; each cache's blocks through a table of their
        # addresses (IR.hs:400-429), bound after the buffers.
        KernelSig("kv_store_paged",
                  [_f32("qkv"), _f32("cos"), _f32("sin"), _u32("pos"), _u32("table")],
                  [_dim("m", 1, 65535), _dim("kv_heads", 1, 1024), _dim("d", 2, 2048, 2), _dim("block_size", 1, 65536),
                   _dim("table_len", 1, _MAX), _dim("blocks", 1, _MAX), _u("rotated"), _u("ldq"), _u("k_off"),
                   _u("v_off")], tables=[Table("k_cache", "read_write", "f32"), Table("v_cache", "read_write", "f32")],
                  threads=64),
        KernelSig("attend_split_paged",
                  [_f32("qkv"), _f32("cos"), _f32("sin"), _u32("pos"), _u32("table"), _f32("part_m", "write"),
                   _f32("part_l", "write"), _f32("part_acc", "write")],
                  [_dim("m", 1, 16384), _dim("heads", 1, 1024), _dim("kv_heads", 1, 1024), _dim("d", 128, 128),
                   _dim("block_size", 1, 65536), _dim("table_len", 1, _MAX), _dim("blocks", 1, _MAX), _u("rotated"),
                   _dim("chunk", 1, 256), _dim("max_splits", 1, 65535), _u("ldq"), _u("q_off"), _f("scale")],
                  tables=[Table("k_cache", "read", "f32"), Table("v_cache", "read", "f32")], threads=128),
        KernelSig("attend_decode_paged",
                  [_f32("qkv"), _f32("cos"), _f32("sin"), _u32("pos"), _u32("table"), _f32("part_m", "write"),
                   _f32("part_l", "write"), _f32("part_acc", "write")],
                  [_dim("m", 1, 64), _dim("heads", 1, 1024), _dim("kv_heads", 1, 1024), _dim("d", 128, 128),
                   _dim("block_size", 1, 65536), _dim("table_len", 1, _MAX), _dim("blocks", 1, _MAX), _u("rotated"),
                   _dim("chunk", 1, 256), _dim("max_splits", 1, 65535), _u("ldq"), _u("q_off"), _u("k_off"),
                   _u("v_off"), _f("scale")],
                  tables=[Table("k_cache", "read_write", "f32"), Table("v_cache", "read_write", "f32")], threads=128),
        KernelSig("attend_prompt_paged",
                  [_f32("qkv"), _f32("cos"), _f32("sin"), _u32("pos"), _u32("table"), _f32("out", "write")],
                  [_dim("m", 1, 65535), _dim("heads", 1, 1024), _dim("kv_heads", 1, 1024), _dim("d", 128, 128),
                   _dim("block_size", 1, 65536), _dim("table_len", 1, _MAX), _dim("blocks", 1, _MAX),
                   _u("rotated"), _u("ldq"), _u("q_off"), _u("ldo"), _dim("max_pos", 0, _MAX - 1), _f("scale")],
                  tables=[Table("k_cache", "read", "f32"), Table("v_cache", "read", "f32")], threads=256),
    ]
}


# The 16-bit forms (the model's weights, or its KV caches, in bf16 or f16:
# the reference's element types, Build.hs:171-194, Check.hs:105-111,
# Graph.hs:169-180): an f32 entry's parameters with the named buffers of
# that type, named by the suffix of the type.
WEIGHT_SUFFIX = {"f32": "", "bf16": "_wbf16", "f16": "_wf16"}
CACHE_SUFFIX = {"f32": "", "bf16": "_kvbf16", "f16": "_kvf16"}
_VARIANTS = [
    *[(base, base + WEIGHT_SUFFIX[t], {"w", "gamma"}, t)
      for t in ("bf16", "f16")
      for base in ("gemv", "gemv_add", "gemv_rmsnorm", "gemv_rmsnorm_silu", "gemv_silu", "gemv_silu_add",
                   "gemv_scatter", "gemv_reduce_rmsnorm", "gemv_reduce_rmsnorm_silu")],
    *[(base, base + WEIGHT_SUFFIX[t], {buf}, t)
      for t in ("bf16", "f16")
      for base, buf in (("gather", "table"), ("rmsnorm_rows", "gamma"), ("split_tf32", "x"),
                        ("gemv_routed", "table"), ("route_topk_scaled", "scale"))],
    *[(base, base + CACHE_SUFFIX[t], {"k_cache", "v_cache"}, t)
      for t in ("bf16", "f16")
      for base in ("kv_store_ring", "attend_split", "attend_decode", "attend_prompt", "kv_store_paged",
                   "attend_split_paged", "attend_decode_paged", "attend_prompt_paged")],
]
for _base, _name, _retyped, _t in _VARIANTS:
    _k = SPEC_KERNELS[_base]
    SPEC_KERNELS[_name] = KernelSig(_name, [Buffer(b.name, b.access, _t if b.name in _retyped else b.type)
                                            for b in _k.buffers], _k.params,
                                    [Table(b.name, b.access, _t if b.name in _retyped else b.type)
                                     for b in _k.tables], threads=_k.threads)


class CudaBackend:
    """`cuda :: Backend Cuda`: the name and the lowering."""

    name = "cuda"

    def backend_lower(self, kernels: list) -> tuple[list, Lowered | None]:
        """(findings, lowered): findings empty iff every kernel resolves.

        Like the CPU target's `clashes` (src/FuryKernel/Cpu.hs:97-106), a
        name lowered twice is refused."""
        from . import _native as N

        findings: list = []
        counts: dict = {}
        for k in kernels:
            counts[k.name] = counts.get(k.name, 0) + 1
        for name, c in sorted(counts.items()):
            if c > 1:
                findings.append(Finding("Names", f"The kernel {name} is lowered {c} times into one module."))
        table = N.table()
        out = []
        for k in kernels:
            a = A.abi_of(k)
            e = table.get(k.name)
            if e is None:
                findings.append(Finding("Overrides", f"No kernel of the target replaces {k.name}."))
                continue
            if e.abi_hash != a.hash:
                mine, theirs = a.description.splitlines(), e.abi_description.splitlines()
                diff = next(((x, y) for x, y in zip(mine, theirs) if x != y), None)
                if diff is None:
                    diff = (mine[len(theirs)] if len(mine) > len(theirs) else "",
                            theirs[len(mine)] if len(theirs) > len(mine) else "")
                findings.append(Finding("Overrides", f"The target's {k.name} has another ABI than {k.name}: "
                                                     f"{diff[1]} where {k.name} has {diff[0]}."))
                continue
            out.append(LoweredKernel(k.name, k.name, a, 0, e.threads, "", [(b.name, i) for i, b in enumerate(k.buffers)],
                                     None, 0))
        if findings:
            return findings, None
        return [], Lowered("cuda", {"language_version": None, "math": "Strict"}, "", out)


cuda = CudaBackend()
