"""The drop-in boundary on the CPU: the C-ABI library loads and exports every
entry point include/furykernel_cuda.h declares, its kernel table's ABI texts
are the reference's canonical form, and the backend resolves this path's
spec kernels by name and hash. No GPU compute runs here."""

import ctypes
import os
import re

import pytest

from furykernel_b200 import _native as N
from furykernel_b200 import abi as A
from furykernel_b200 import target as T

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "furykernel_cuda.h")).read()
    return sorted(set(re.findall(r"\b(fkc_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(N.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 30
    for n in names:
        assert hasattr(lib, n), n


def test_fnv1a_reference_vectors():
    # test/Test/FuryKernel/AbiTest.hs:33-36.
    for s, h in [("", 0xCBF29CE484222325), ("a", 0xAF63DC4C8601EC8C), ("foobar", 0x85944171F73967E8)]:
        assert A.fnv1a64(s) == h
        assert N.lib().fkc_fnv1a64(s.encode(), len(s)) == h


def test_c_layout_of_parameters():
    # AbiTest.hs:37-42.
    P = A.Param
    fields, size = A.layout([P("a", "u8"), P("b", "f32"), P("c", "f16"), P("d", "u32")])
    assert [(f.name, f.offset) for f in fields] == [("a", 0), ("b", 4), ("c", 8), ("d", 12)]
    assert size == 16
    assert A.layout([])[1] == 0
    assert A.layout([P("a", "f32"), P("b", "u8")])[1] == 8


def test_description_and_pinned_hash_of_the_scale_kernel():
    # AbiTest.hs:43-53 (the rmsnorm test kernel's text) and :68-71 (scale's
    # ABI hash pinned at 0xe99ad54061a304ff).
    rms = A.KernelSig("rmsnorm", [A.Buffer("x", "read", "bf16"), A.Buffer("w", "read", "bf16"),
                                  A.Buffer("y", "write", "bf16")],
                      [A.Param("rows", "u32", A.DimRange(1, 4096)), A.Param("eps", "f32")])
    assert A.abi_of(rms).description == (
        "abi 1\nbuffer x read bf16 align 16\nbuffer w read bf16 align 16\nbuffer y write bf16 align 16\n"
        "param rows u32 at 0\nparam eps f32 at 4\nparams size 8\n")
    scale = A.KernelSig("scale", [A.Buffer("x", "read", "bf16"), A.Buffer("y", "write", "bf16")],
                        [A.Param("n", "u32", A.DimRange(1, 65536)), A.Param("s", "f32")])
    assert A.abi_of(scale).hash == 0xE99AD54061A304FF


def test_table_agrees_with_spec_kernels():
    table = N.table()
    assert set(table) == set(T.SPEC_KERNELS)
    for name, k in T.SPEC_KERNELS.items():
        a = A.abi_of(k)
        assert table[name].abi_description == a.description, name
        assert table[name].abi_hash == a.hash, name
        assert table[name].threads == k.threads, name


def test_backend_lowers_spec_kernels():
    findings, lowered = T.cuda.backend_lower(list(T.SPEC_KERNELS.values()))
    assert findings == []
    assert lowered.language == "cuda" and lowered.options["math"] == "Strict"
    assert [k.name for k in lowered.kernels] == list(T.SPEC_KERNELS)


def test_backend_refuses_another_abi_and_duplicates():
    k = T.SPEC_KERNELS["add"]
    other = A.KernelSig("add", [A.Buffer("a", "read", "f32"), A.Buffer("b", "read", "f32"),
                                A.Buffer("y", "write", "f32", 32)], k.params)
    findings, lowered = T.cuda.backend_lower([other])
    assert lowered is None
    assert findings[0].message == ("The target's add has another ABI than add: buffer y write f32 align 16 "
                                   "where add has buffer y write f32 align 32.")
    findings, _ = T.cuda.backend_lower([k, k])
    assert findings[0].message == "The kernel add is lowered 2 times into one module."
    findings, _ = T.cuda.backend_lower([A.KernelSig("nope", [], [])])
    assert findings[0].message == "No kernel of the target replaces nope."


def test_kernel_find_refuses_by_hash():
    lib = N.lib()
    i = ctypes.c_int()
    assert lib.fkc_kernel_find(b"add", N.table()["add"].abi_hash, ctypes.byref(i)) == 0
    assert lib.fkc_kernel_find(b"add", 1, ctypes.byref(i)) == N.FKC_ERR_ARGUMENT
    assert "another ABI" in lib.fkc_last_error().decode()
    assert lib.fkc_kernel_find(b"nope", 1, ctypes.byref(i)) == N.FKC_ERR_ARGUMENT


def test_no_device_is_an_error_not_a_fallback():
    # Here there is no GPU: opening a context must fail loudly.
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(N.FkcError):
        N.Context(0)
