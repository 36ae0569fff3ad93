"""The C ABI library loads on a machine without a GPU and exports every declared symbol.

Only host-side argument validation is exercised here (those paths return before any CUDA
call); compute calls are in the gpu-marked tests.
"""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for header in os.listdir(os.path.join(ROOT, "include")):
        if header.endswith(".h"):
            text = open(os.path.join(ROOT, "include", header)).read()
            names.update(re.findall(r"\b(pcu_b200_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_the_node_executors():
    names = _declared()
    for required in ("pcu_b200_strict_matmul", "pcu_b200_strict_sgd", "pcu_b200_strict_mse",
                     "pcu_b200_checked_binary", "pcu_b200_checked_relu", "pcu_b200_checked_relu_backward",
                     "pcu_b200_status_reset"):
        assert required in names


def test_library_exports_every_declared_symbol(provider):
    lib = provider.library()
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_library_links_no_driver_at_load_time():
    out = os.popen(f"ldd {os.path.join(ROOT, 'fusion-pcu_b200', 'libpcu_b200.so')}").read()
    assert "libcuda.so" not in out and "not found" not in out, out


def test_host_validation_rejects_bad_arguments(provider):
    lib = provider.library()
    status = ctypes.c_uint64(0)
    sp = ctypes.byref(status)
    # bad dtype / policy / op, missing status: all rejected before any device work
    assert lib.pcu_b200_checked_binary(7, 0, 0, None, None, None, 0, 0, 0, sp, None) == 1
    assert lib.pcu_b200_checked_binary(0, 9, 0, None, None, None, 0, 0, 0, sp, None) == 1
    assert lib.pcu_b200_checked_binary(0, 0, 9, None, None, None, 0, 0, 0, sp, None) == 1
    assert lib.pcu_b200_strict_sgd(0, 0, None, None, None, 4, 0x3F000000, None, None) == 1
    # a non-finite learning rate is rejected (the capture-time rule of Graph::sgd_update)
    assert lib.pcu_b200_strict_sgd(0, 0, ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 4,
                                   0x7FC00000, sp, None) == 1
    # MSE of zero elements has no fault domain (fault_domain.rs:99-104)
    assert lib.pcu_b200_strict_mse(0, 0, ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 0, None,
                                   0, sp, None) == 1
    # the packed event bound rows*columns*inner*2 <= 2^60 (strict_matmul.rs:121-127)
    big = 1 << 21
    assert lib.pcu_b200_strict_matmul(0, 2, ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), big,
                                      big, big, big, big, 0, 0, None, 0, sp, None) == 2
    # empty outputs are a successful no-op
    assert lib.pcu_b200_strict_matmul(0, 0, None, None, None, 0, 5, 5, 5, 5, 0, 0, None, 0, sp, None) == 0
    assert lib.pcu_b200_abi_version() == 2
    # row-sharded all-gather: the rank must index the peer list, and a call with peers needs a
    # call number (the write-side order of the peer stores)
    peers = (ctypes.c_void_p * 1)(16)
    dev = ctypes.c_void_p(256)
    for rank, epoch in ((2, 1), (-1, 1), (0, 0)):
        assert lib.pcu_b200_strict_matmul_rows_allgather(0, 0, dev, dev, dev, 0, 4, 8, 4, 4, 4, 4, 0, peers, 1, rank,
                                                         epoch, None, 0, sp, None) == 1
    # a buffer of the all-gather is C rounded up to 256 bytes plus a 256-byte flag block
    assert lib.pcu_b200_peer_rows_bytes(0, 3, 5) == 256 + 256
    assert lib.pcu_b200_peer_rows_bytes(1, 64, 64) == 64 * 64 * 8 + 256
    assert lib.pcu_b200_peer_rows_bytes(5, 64, 64) == 0
    assert lib.pcu_b200_error_string(3).decode().startswith("workspace")


@pytest.mark.parametrize("rows,inner,columns", [(1, 1, 1), (8192, 8192, 8192), (3, 0, 5)])
def test_workspace_sizes(provider, rows, inner, columns):
    lib = provider.library()
    need = lib.pcu_b200_strict_matmul_workspace_size(rows, inner, columns)
    assert need >= 4 * (rows + columns) and need % 256 == 0
    # strict MSE keeps one ordered-sum map per chunk (F32: 1024 elements -> a 16-byte head and
    # 2 x 23 u32 increments; F64: 512 elements -> a head and 2 x 52 u64 increments), plus one per
    # block of 64 chunks and one per superblock of 64 blocks
    for dtype, chunk, per_chunk in ((0, 1024, 16 + 2 * 23 * 4), (1, 512, 16 + 2 * 52 * 8)):
        got = lib.pcu_b200_strict_mse_workspace_size(dtype, 1 << 28)
        assert got >= ((1 << 28) // chunk) * per_chunk and got % 256 == 0
        assert got < ((1 << 28) // chunk) * per_chunk * 1.1


def _c_signatures():
    """(name, return type, parameter count) of every function declared in include/*.h."""
    sigs = []
    for header in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not header.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", header)).read()
        text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
        text = re.sub(r"//[^\n]*", " ", text)
        for ret, name, params in re.findall(r"([\w\s\*]+?)\b(pcu_b200_\w+)\s*\(([^;{}]*?)\)\s*;", text, flags=re.S):
            tokens = ret.replace("*", " * ").split()
            kind = "pointer" if tokens and tokens[-1] == "*" else (tokens[-1] if tokens else "")
            plist = [] if params.strip() in ("", "void") else [q.strip() for q in params.split(",")]
            sigs.append((name, kind, plist))
    return sigs


def _param_fits(param, ctype):
    """A C parameter and its ctypes type agree: a pointer for a pointer, the same width for an
    integer."""
    if "*" in param or "[" in param:
        return ctype in (ctypes.c_void_p, ctypes.c_char_p) or issubclass(ctype, (ctypes._Pointer, ctypes.Array))
    base = param.replace("const", " ").split()[0]
    width = {"int": 4, "int32_t": 4, "uint32_t": 4, "uint64_t": 8, "size_t": 8}.get(base)
    return width is not None and ctypes.sizeof(ctype) == width and issubclass(ctype, ctypes._SimpleCData)


def test_ctypes_declarations_match_the_headers(provider):
    """The Python binding (and the graph layer's, declared on the same library object) gives every
    entry point with parameters argtypes of the header's length, each a pointer where the header
    has a pointer and an integer of the header's width otherwise, and a restype wide enough for
    size_t, uint64_t and pointer results (ctypes would otherwise truncate them to an int)."""
    import importlib

    L = importlib.import_module("fusion-pcu_b200.graph")._lib()
    wrong = []
    for name, kind, params in _c_signatures():
        fn = getattr(L, name)
        if params and (fn.argtypes is None or len(fn.argtypes) != len(params)):
            wrong.append((name, "argtypes", None if fn.argtypes is None else len(fn.argtypes), len(params)))
        elif params:
            wrong += [(name, "parameter", i, q, t) for i, (q, t) in enumerate(zip(params, fn.argtypes))
                      if not _param_fits(q, t)]
        want = {"size_t": (ctypes.c_size_t,), "uint64_t": (ctypes.c_uint64,),
                "pointer": (ctypes.c_void_p, ctypes.c_char_p)}.get(kind)
        if want and fn.restype not in want:
            wrong.append((name, "restype", fn.restype, kind))
    assert not wrong, wrong
