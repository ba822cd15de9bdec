"""ctypes binding of libfurykernel_cuda.so (include/furykernel_cuda.h).

The library is loaded from the package's _build directory, where build()
puts it. There is no fallback: without the library, or without a B200,
every entry point here raises.
"""

from __future__ import annotations

import ctypes
import os
import struct
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libfurykernel_cuda.so")

FKC_OK = 0
FKC_ERR_ARGUMENT = 1
FKC_ERR_CUDA = 2
FKC_ERR_NCCL = 3
FKC_ERR_STATE = 4

_lib = None


class FkcError(RuntimeError):
    """A failed entry point: its code and the library's message."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class Refused(FkcError):
    """A launch or lookup the target refuses (FKC_ERR_ARGUMENT)."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FkcError(FKC_ERR_STATE, f"furykernel-cuda is not built: {LIB_PATH} is missing (run build()).")
        L = ctypes.CDLL(LIB_PATH)
        vp, sz, u32, u64, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
        pvp = ctypes.POINTER(ctypes.c_void_p)
        sig = {
            "fkc_last_error": (ctypes.c_char_p, []),
            "fkc_version": (i32, []),
            "fkc_open": (i32, [i32, pvp]),
            "fkc_close": (i32, [vp]),
            "fkc_stream": (i32, [vp, pvp]),
            "fkc_sm_count": (i32, [vp, ctypes.POINTER(i32)]),
            "fkc_set_pdl": (i32, [vp, i32]),
            "fkc_set_wait_limit": (i32, [vp, u32]),
            "fkc_set_prefetch": (i32, [vp, u64]),
            "fkc_set_l2_prefetch": (i32, [vp, vp, u64]),
            "fkc_set_wait_stats": (i32, [vp, i32]),
            "fkc_set_gemm_tile": (i32, [vp, ctypes.c_uint, ctypes.c_uint]),
            "fkc_read_wait_stats": (i32, [vp, ctypes.POINTER(u64), ctypes.POINTER(u64)]),
            "fkc_sync": (i32, [vp]),
            "fkc_status": (i32, [vp, ctypes.POINTER(i32)]),
            "fkc_buf_alloc": (i32, [vp, sz, pvp]),
            "fkc_buf_free": (i32, [vp, vp]),
            "fkc_buf_zero": (i32, [vp, vp, sz]),
            "fkc_buf_upload": (i32, [vp, vp, vp, sz]),
            "fkc_buf_download": (i32, [vp, vp, vp, sz]),
            "fkc_host_alloc": (i32, [sz, pvp]),
            "fkc_host_free": (i32, [vp]),
            "fkc_kv_arena": (i32, [vp, u32, u32, u32, u32, u32, pvp, pvp]),
            "fkc_kv_arena_elem": (i32, [vp, u32, u32, u32, u32, u32, u32, pvp, pvp]),
            "fkc_rope_tables": (i32, [vp, ctypes.c_double, u32, u32, u32, pvp, pvp]),
            "fkc_fill_normal": (i32, [vp, vp, u64, u64, ctypes.c_double, ctypes.c_double]),
            "fkc_fill_uniform": (i32, [vp, vp, u64, u64, ctypes.c_double, ctypes.c_double]),
            "fkc_fill_normal_bf16": (i32, [vp, vp, u64, u64, ctypes.c_double, ctypes.c_double]),
            "fkc_fill_normal_f16": (i32, [vp, vp, u64, u64, ctypes.c_double, ctypes.c_double]),
            "fkc_kernel_count": (i32, []),
            "fkc_kernel_describe": (i32, [i32, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p),
                                          ctypes.POINTER(u64), ctypes.POINTER(u32), ctypes.POINTER(u32),
                                          ctypes.POINTER(u32)]),
            "fkc_kernel_find": (i32, [ctypes.c_char_p, u64, ctypes.POINTER(i32)]),
            "fkc_fnv1a64": (u64, [vp, sz]),
            "fkc_launch": (i32, [vp, i32, vp, sz, pvp, i32]),
            "fkc_capture_begin": (i32, [vp]),
            "fkc_capture_end": (i32, [vp, pvp]),
            "fkc_graph_launch": (i32, [vp, vp]),
            "fkc_graph_destroy": (i32, [vp]),
            "fkc_step": (i32, [vp, vp, vp, vp, sz, vp, vp, sz]),
            "fkc_time_graph": (i32, [vp, vp, i32, i32, ctypes.POINTER(ctypes.c_float)]),
            "fkc_comm_unique_id": (i32, [vp]),
            "fkc_comm_init": (i32, [vp, i32, i32, vp]),
            "fkc_allreduce_sum_f32": (i32, [vp, vp, sz]),
            "fkc_allgather_u32": (i32, [vp, vp, vp, sz]),
            "fkc_comm_rank": (i32, [vp, ctypes.POINTER(i32), ctypes.POINTER(i32)]),
            "fkc_reduce_sum_f32_noalloc": (i32, [vp, u64, vp, vp]),
            "fkc_peer_region_bytes": (sz, []),
            "fkc_peer_alloc": (i32, [vp, sz, pvp, vp]),
            "fkc_peer_open": (i32, [vp, vp, pvp]),
            "fkc_peer_set": (i32, [vp, i32, i32, pvp]),
            "fkc_comm_destroy": (i32, [vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != FKC_OK:
        msg = lib().fkc_last_error().decode()
        raise (Refused if rc == FKC_ERR_ARGUMENT else FkcError)(rc, msg)


# ---------------------------------------------------------------------------
# The kernel table, as the library describes it


@dataclass
class ParamField:
    name: str
    type: str
    offset: int


@dataclass
class BufferBinding:
    name: str
    access: str
    type: str
    align: int


@dataclass
class TableEntry:
    """One LoweredKernel of the target (src/FuryKernel/Backend.hs:203-228)."""

    id: int
    name: str
    abi_description: str
    abi_hash: int
    threads: int
    params_size: int
    buffers: list = field(default_factory=list)
    params: list = field(default_factory=list)

    def pack(self, values: dict) -> bytes:
        """The parameter struct's bytes in C layout (Abi.hs:113-133)."""
        buf = bytearray(self.params_size)
        names = {p.name for p in self.params}
        extra = set(values) - names
        if extra:
            raise Refused(FKC_ERR_ARGUMENT, f"{self.name} has no parameter {sorted(extra)[0]}.")
        for p in self.params:
            if p.name not in values:
                raise Refused(FKC_ERR_ARGUMENT, f"{self.name}: no value for the parameter {p.name}.")
            v = values[p.name]
            fmt = {"u32": "<I", "f32": "<f", "i32": "<i"}[p.type]
            struct.pack_into(fmt, buf, p.offset, v)
        return bytes(buf)


def parse_abi(text: str):
    bufs, params = [], []
    for line in text.splitlines():
        w = line.split()
        if not w:
            continue
        if w[0] == "buffer":
            bufs.append(BufferBinding(w[1], w[2], w[3], int(w[5])))
        elif w[0] == "table":  # bound after the buffers; a read-only table's line names no access
            access = "read" if len(w) == 5 else w[2]
            bufs.append(BufferBinding(w[1], access, w[-3], int(w[-1])))
        elif w[0] == "param":
            params.append(ParamField(w[1], w[2], int(w[4])))
    return bufs, params


_table = None


def table() -> dict:
    global _table
    if _table is None:
        L = lib()
        out = {}
        for i in range(L.fkc_kernel_count()):
            name, abi = ctypes.c_char_p(), ctypes.c_char_p()
            h, th, ps, nb = ctypes.c_uint64(), ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
            check(L.fkc_kernel_describe(i, ctypes.byref(name), ctypes.byref(abi), ctypes.byref(h), ctypes.byref(th),
                                        ctypes.byref(ps), ctypes.byref(nb)))
            text = abi.value.decode()
            bufs, params = parse_abi(text)
            out[name.value.decode()] = TableEntry(i, name.value.decode(), text, h.value, th.value, ps.value, bufs,
                                                  params)
        _table = out
    return _table


# ---------------------------------------------------------------------------
# Device memory and contexts


class DeviceBuffer:
    """A buffer the context owns: its address, size and element type."""

    def __init__(self, ctx: "Context", ptr: int, nbytes: int, dtype=np.float32, shape=None):
        self.ctx, self.ptr, self.nbytes = ctx, ptr, nbytes
        self.dtype = np.dtype(dtype)
        self.shape = shape if shape is not None else (nbytes // self.dtype.itemsize,)

    def download(self) -> np.ndarray:
        out = np.empty(self.shape, self.dtype)
        check(lib().fkc_buf_download(self.ctx.handle, out.ctypes.data, self.ptr, out.nbytes))
        return out

    def upload(self, a: np.ndarray) -> None:
        a = np.ascontiguousarray(a, self.dtype)
        assert a.nbytes <= self.nbytes
        check(lib().fkc_buf_upload(self.ctx.handle, self.ptr, a.ctypes.data, a.nbytes))

    def at(self, elements: int) -> int:
        """The address `elements` elements in."""
        return self.ptr + elements * self.dtype.itemsize

    def free(self) -> None:
        if self.ptr:
            check(lib().fkc_buf_free(self.ctx.handle, self.ptr))
            self.ptr = 0


class Graph:
    def __init__(self, ctx: "Context", handle: int):
        self.ctx, self.handle = ctx, handle

    def launch(self) -> None:
        check(lib().fkc_graph_launch(self.ctx.handle, self.handle))

    def time(self, warmup: int, iters: int) -> float:
        ms = ctypes.c_float()
        check(lib().fkc_time_graph(self.ctx.handle, self.handle, warmup, iters, ctypes.byref(ms)))
        return ms.value

    def destroy(self) -> None:
        if self.handle:
            check(lib().fkc_graph_destroy(self.handle))
            self.handle = 0


class Context:
    """A device context (fkc_open): memory, launches, graphs, NCCL."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().fkc_open(device, ctypes.byref(h)))
        self.handle = h.value
        self.device = device
        sms = ctypes.c_int()
        check(lib().fkc_sm_count(self.handle, ctypes.byref(sms)))
        self.sms = sms.value

    def close(self) -> None:
        if self.handle:
            check(lib().fkc_close(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def stream(self) -> int:
        s = ctypes.c_void_p()
        check(lib().fkc_stream(self.handle, ctypes.byref(s)))
        return s.value or 0

    def set_pdl(self, on: bool) -> None:
        check(lib().fkc_set_pdl(self.handle, 1 if on else 0))

    def set_prefetch(self, nbytes: int) -> None:
        """The L2 bulk-prefetch budget of later streaming GEMV launches (0:
        the first lines of each warp's first row only)."""
        check(lib().fkc_set_prefetch(self.handle, nbytes))

    def set_l2_prefetch(self, ptr: int, nbytes: int) -> None:
        """A range later attention launches bring toward L2 while they run
        (0, 0: none)."""
        check(lib().fkc_set_l2_prefetch(self.handle, ptr or None, nbytes))

    def set_wait_limit(self, microseconds: int) -> None:
        """The bound of each wait on another rank, in microseconds (0: the
        default, about 2 s)."""
        check(lib().fkc_set_wait_limit(self.handle, microseconds))

    def set_gemm_tile(self, tm: int, parts: int = 1) -> None:
        """gemm_tf32x3w's tile for later launches: tm A rows against 128 W
        rows; parts 1, a tile a CTA; 2, two K halves a tile; 0, an equal
        share of the slabs to each of min(tiles, SMs) CTAs. tm 0, the
        shape's own pick."""
        check(lib().fkc_set_gemm_tile(self.handle, tm, parts))

    def set_wait_stats(self, on: bool) -> None:
        """Whether blocks that wait on their peers add their waits to the
        context's totals (launches and captures after the call)."""
        check(lib().fkc_set_wait_stats(self.handle, 1 if on else 0))

    def read_wait_stats(self) -> tuple:
        """(nanoseconds waited, waits) since the last read; then cleared."""
        ns, n = ctypes.c_uint64(), ctypes.c_uint64()
        check(lib().fkc_read_wait_stats(self.handle, ctypes.byref(ns), ctypes.byref(n)))
        return ns.value, n.value

    def sync(self) -> None:
        check(lib().fkc_sync(self.handle))

    def status(self) -> int:
        """The device status word (0, or a bounded wait's code), then cleared."""
        code = ctypes.c_int()
        check(lib().fkc_status(self.handle, ctypes.byref(code)))
        return code.value

    def alloc(self, nbytes: int, dtype=np.float32, shape=None) -> DeviceBuffer:
        p = ctypes.c_void_p()
        check(lib().fkc_buf_alloc(self.handle, nbytes, ctypes.byref(p)))
        return DeviceBuffer(self, p.value, nbytes, dtype, shape)

    def empty(self, shape, dtype=np.float32) -> DeviceBuffer:
        shape = tuple(shape) if isinstance(shape, (tuple, list)) else (shape,)
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        return self.alloc(n, dtype, shape)

    def zeros(self, shape, dtype=np.float32) -> DeviceBuffer:
        b = self.empty(shape, dtype)
        check(lib().fkc_buf_zero(self.handle, b.ptr, b.nbytes))
        return b

    def to_device(self, a: np.ndarray) -> DeviceBuffer:
        a = np.ascontiguousarray(a)
        b = self.alloc(a.nbytes, a.dtype, a.shape)
        b.upload(a)
        return b

    def fill_normal(self, buf: DeviceBuffer, seed: int, mu: float = 0.0, sigma: float = 1.0) -> None:
        check(lib().fkc_fill_normal(self.handle, buf.ptr, buf.nbytes // 4, seed, mu, sigma))

    def fill_normal_bf16(self, buf: DeviceBuffer, seed: int, mu: float = 0.0, sigma: float = 1.0) -> None:
        """fill_normal's values rounded to bf16, nbytes / 2 of them."""
        check(lib().fkc_fill_normal_bf16(self.handle, buf.ptr, buf.nbytes // 2, seed, mu, sigma))

    def fill_normal_f16(self, buf: DeviceBuffer, seed: int, mu: float = 0.0, sigma: float = 1.0) -> None:
        """fill_normal's values rounded to f16, nbytes / 2 of them."""
        check(lib().fkc_fill_normal_f16(self.handle, buf.ptr, buf.nbytes // 2, seed, mu, sigma))

    def fill_uniform(self, buf: DeviceBuffer, seed: int, a: float = -1.0, b: float = 1.0) -> None:
        check(lib().fkc_fill_uniform(self.handle, buf.ptr, buf.nbytes // 4, seed, a, b))

    def rope_tables(self, theta: float, d: int, rotated: int, positions: int):
        c, s = ctypes.c_void_p(), ctypes.c_void_p()
        check(lib().fkc_rope_tables(self.handle, theta, d, rotated, positions, ctypes.byref(c), ctypes.byref(s)))
        n = positions * rotated * 4
        return (DeviceBuffer(self, c.value, n, np.float32, (positions, rotated)),
                DeviceBuffer(self, s.value, n, np.float32, (positions, rotated)))

    def launch(self, kernel: str, params: dict, bufs: list) -> None:
        """Launches a table entry: params by name, buffers in declaration
        order, then its tables (device addresses of arrays of addresses)."""
        e = table().get(kernel)
        if e is None:
            raise Refused(FKC_ERR_ARGUMENT, f"The target has no kernel {kernel}.")
        raw = e.pack(params)
        ptrs = (ctypes.c_void_p * len(bufs))(*[b.ptr if isinstance(b, DeviceBuffer) else int(b) for b in bufs])
        pbuf = ctypes.create_string_buffer(raw, len(raw)) if raw else None
        check(lib().fkc_launch(self.handle, e.id, pbuf, len(raw), ptrs, len(bufs)))

    def capture_begin(self) -> None:
        check(lib().fkc_capture_begin(self.handle))

    def capture_end(self) -> Graph:
        g = ctypes.c_void_p()
        check(lib().fkc_capture_end(self.handle, ctypes.byref(g)))
        return Graph(self, g.value)

    def step(self, graph: Graph, host_in: np.ndarray, dev_in: DeviceBuffer, host_out: np.ndarray,
             dev_out: DeviceBuffer) -> None:
        check(lib().fkc_step(self.handle, graph.handle, host_in.ctypes.data, dev_in.ptr, host_in.nbytes,
                             host_out.ctypes.data, dev_out.ptr, host_out.nbytes))

    # NCCL
    @staticmethod
    def comm_unique_id() -> bytes:
        b = ctypes.create_string_buffer(128)
        check(lib().fkc_comm_unique_id(b))
        return b.raw

    def comm_init(self, nranks: int, rank: int, uid: bytes) -> None:
        b = ctypes.create_string_buffer(uid, 128)
        check(lib().fkc_comm_init(self.handle, nranks, rank, b))

    def allreduce_sum(self, buf: DeviceBuffer, count: int | None = None) -> None:
        check(lib().fkc_allreduce_sum_f32(self.handle, buf.ptr, count if count is not None else buf.nbytes // 4))

    def comm_destroy(self) -> None:
        check(lib().fkc_comm_destroy(self.handle))


def pinned(shape, dtype) -> np.ndarray:
    """A numpy array over pinned host memory (freed with the process)."""
    n = int(np.prod(shape)) * np.dtype(dtype).itemsize
    p = ctypes.c_void_p()
    check(lib().fkc_host_alloc(n, ctypes.byref(p)))
    buf = (ctypes.c_char * n).from_address(p.value)
    return np.frombuffer(buf, dtype=dtype, count=int(np.prod(shape))).reshape(shape)
