"""libmolten_rt.so: loads without a GPU, exports exactly the functions
include/molten_rt.h declares, and rejects bad arguments on the host."""
import ctypes
import os
import re
import subprocess

import pytest

from molten_b200 import _capi

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "molten_rt.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(molten_\w+)\s*\(", text, re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _capi.load_library()
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_capi.SIGNATURES)
    out = subprocess.run(["nm", "-D", "--defined-only", str(_capi.LIB_PATH)],
                         capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (molten_\w+)", out))
    assert exported == set(names)


def test_version_and_last_error():
    lib = _capi.load_library()
    assert lib.molten_version() == 101
    assert isinstance(lib.molten_last_error(), bytes)


def test_struct_layouts_match_the_header():
    # sizes of the by-value kernel parameter blocks
    assert ctypes.sizeof(_capi.RowArgs) == 160
    assert ctypes.sizeof(_capi.GemmArgs) == 448
    assert _capi.GemmArgs.inp.offset == 256 and _capi.GemmArgs.m.offset == 384
    assert _capi.GemmArgs.status.offset == 416


def test_null_and_bad_arguments_are_rejected():
    lib = _capi.load_library()
    assert lib.molten_device_count(None) == 1
    assert b"null" in lib.molten_last_error()
    assert lib.molten_module_load(None, 0, None) == 1
    h = ctypes.c_void_p()
    assert lib.molten_module_load(b"/nonexistent.cubin", 0, ctypes.byref(h)) == 4
    assert b"cannot open" in lib.molten_last_error()
    assert lib.molten_launch(None, b"k", None, None, 0, None) == 1
    assert lib.molten_module_unload(None) == 1
    # TMA descriptor checks happen before any driver call
    buf = ctypes.create_string_buffer(256)
    aligned = (ctypes.addressof(buf) + 63) & ~63
    assert lib.molten_encode_tma_2d(ctypes.c_void_p(aligned + 8), 0, ctypes.c_void_p(4096),
                                    64, 64, 128, 64, 64, 1) == 1          # map misaligned
    assert lib.molten_encode_tma_2d(ctypes.c_void_p(aligned), 0, ctypes.c_void_p(4100),
                                    64, 64, 128, 64, 64, 1) == 1          # base misaligned
    assert b"16-byte" in lib.molten_last_error()
    assert lib.molten_encode_tma_2d(ctypes.c_void_p(aligned), 0, ctypes.c_void_p(4096),
                                    64, 64, 120, 64, 64, 1) == 1          # stride
    assert lib.molten_encode_tma_2d(ctypes.c_void_p(aligned), 2, ctypes.c_void_p(4096),
                                    64, 64, 256, 64, 64, 1) == 1          # 256 B box row
    assert lib.molten_encode_tma_2d(ctypes.c_void_p(aligned), 0, ctypes.c_void_p(4096),
                                    64, 64, 128, 64, 64, 64) == 1         # row over a 64 B span
    assert lib.molten_encode_tma_2d(ctypes.c_void_p(aligned), 0, ctypes.c_void_p(4096),
                                    64, 64, 128, 32, 32, 48) == 1         # no such swizzle
    assert b"swizzle" in lib.molten_last_error()
    assert lib.molten_read_status(0, None, 0) == 1


def test_device_count_without_gpu_is_zero_or_error():
    lib = _capi.load_library()
    n = ctypes.c_int(-1)
    rc = lib.molten_device_count(ctypes.byref(n))
    assert rc in (0, 2) and n.value >= 0
