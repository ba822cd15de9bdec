"""A kernel's binary interface, restating src/FuryKernel/Abi.hs.

The ABI is the buffers in declaration order, the tables after them and the
one parameter struct laid out as C lays out a struct of its fields
(Abi.hs:113-133); its hash is 64-bit FNV-1a over a canonical text
(abiDescription, Abi.hs:136-159; fnv1a64, Abi.hs:259-262). The target's
table (include/furykernel_cuda.h) is keyed by name and this hash, as tuned
overrides are (Abi.hs:160-246).
"""

from __future__ import annotations

from dataclasses import dataclass, field

SIZES = {"f32": 4, "f16": 2, "bf16": 2, "i32": 4, "u32": 4, "i8": 1, "u8": 1, "bool": 1}


@dataclass(frozen=True)
class DimRange:
    """The values a dimension may take (IR.hs:363-368)."""

    lo: int
    hi: int
    mult: int = 1

    def text(self) -> str:
        """dimRangeText (Emit/Rust.hs:106-108)."""
        return f"{self.lo}..{self.hi}" + (f" multiple of {self.mult}" if self.mult > 1 else "")

    def holds(self, v: int) -> bool:
        return self.lo <= v <= self.hi and (self.mult <= 1 or v % self.mult == 0)


@dataclass(frozen=True)
class Param:
    name: str
    type: str
    dim: DimRange | None = None  # a dimension, or a scalar


@dataclass(frozen=True)
class Buffer:
    name: str
    access: str  # "read", "write", "read_write"
    type: str
    align: int = 16


@dataclass(frozen=True)
class Table:
    name: str
    access: str
    type: str
    align: int = 16


@dataclass
class Field:
    name: str
    type: str
    offset: int
    dim: DimRange | None


@dataclass
class Abi:
    buffers: list
    tables: list
    params: list  # Field
    params_size: int
    hash: int = 0
    description: str = ""


@dataclass
class KernelSig:
    """What the ABI sees of a kernel: its name, buffers, tables, parameters."""

    name: str
    buffers: list
    params: list
    tables: list = field(default_factory=list)
    threads: int = 256


def fnv1a64(data: str | bytes) -> int:
    if isinstance(data, str):
        data = data.encode()
    h = 0xCBF29CE484222325
    for b in data:
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def hex64(w: int) -> str:
    return "0x" + format(w, "016x")


def layout(params: list) -> tuple[list, int]:
    """Fields at offsets aligned to their sizes; the size rounded up to the
    largest alignment, 0 without fields (Abi.hs:121-133)."""
    fields, off = [], 0
    for p in params:
        size = SIZES[p.type]
        at = (off + size - 1) // size * size
        fields.append(Field(p.name, p.type, at, p.dim))
        off = at + size
    align = max([1] + [SIZES[p.type] for p in params])
    return fields, (off + align - 1) // align * align if params else 0


def description(buffers: list, tables: list, fields: list, size: int) -> str:
    lines = ["abi 1"]
    lines += [f"buffer {b.name} {b.access} {b.type} align {b.align}" for b in buffers]
    lines += [f"table {t.name}{'' if t.access == 'read' else ' ' + t.access} {t.type} align {t.align}" for t in tables]
    lines += [f"param {f.name} {f.type} at {f.offset}" for f in fields]
    lines += [f"params size {size}"]
    return "".join(line + "\n" for line in lines)


def abi_of(k: KernelSig) -> Abi:
    fields, size = layout(k.params)
    text = description(k.buffers, k.tables, fields, size)
    return Abi(list(k.buffers), list(k.tables), fields, size, fnv1a64(text), text)
