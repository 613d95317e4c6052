"""ctypes binding of libmolten_rt.so (declarations in include/molten_rt.h)."""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "lib"
LIB_PATH = LIB_DIR / "libmolten_rt.so"

MOLTEN_OK = 0
MAX_IO = 8
DT_BF16, DT_F16, DT_F32 = 0, 1, 2

# every function of the C ABI: name -> (restype, argtypes)
_c = ctypes
SIGNATURES = {
    "molten_version": (_c.c_int, []),
    "molten_last_error": (_c.c_char_p, []),
    "molten_device_count": (_c.c_int, [_c.POINTER(_c.c_int)]),
    "molten_sync": (_c.c_int, [_c.c_int]),
    "molten_module_load": (_c.c_int, [_c.c_char_p, _c.c_int, _c.POINTER(_c.c_void_p)]),
    "molten_module_load_data": (_c.c_int, [_c.c_void_p, _c.c_size_t, _c.c_int,
                                           _c.POINTER(_c.c_void_p)]),
    "molten_module_unload": (_c.c_int, [_c.c_void_p]),
    "molten_kernel_info": (_c.c_int, [_c.c_void_p, _c.c_char_p, _c.POINTER(_c.c_int),
                                      _c.POINTER(_c.c_int), _c.POINTER(_c.c_int)]),
    "molten_max_resident": (_c.c_int, [_c.c_void_p, _c.c_char_p, _c.c_void_p,
                                       _c.POINTER(_c.c_int), _c.POINTER(_c.c_int)]),
    "molten_launch": (_c.c_int, [_c.c_void_p, _c.c_char_p, _c.c_void_p, _c.c_void_p,
                                 _c.c_size_t, _c.c_void_p]),
    "molten_encode_tma_2d": (_c.c_int, [_c.c_void_p, _c.c_int, _c.c_void_p, _c.c_uint64,
                                        _c.c_uint64, _c.c_uint64, _c.c_uint32, _c.c_uint32,
                                        _c.c_int]),
    "molten_status_word": (_c.c_int, [_c.c_int, _c.POINTER(_c.c_void_p)]),
    "molten_read_status": (_c.c_int, [_c.c_int, _c.POINTER(_c.c_int), _c.c_int]),
    "molten_scores_softmax_bf16_noalloc": (_c.c_int, [_c.c_void_p, _c.c_void_p, _c.c_void_p,
                                                      _c.c_longlong, _c.c_longlong,
                                                      _c.c_longlong, _c.c_void_p]),
}


LAUNCH_PDL = 1          # MOLTEN_LAUNCH_PDL


class LaunchCfg(ctypes.Structure):
    _fields_ = [("grid", ctypes.c_uint32 * 3), ("block", ctypes.c_uint32 * 3),
                ("cluster", ctypes.c_uint32 * 3), ("smem_bytes", ctypes.c_uint32),
                ("flags", ctypes.c_uint32)]


class RowArgs(ctypes.Structure):
    """molten_row_args / molten::RowArgs (160 bytes)."""
    _fields_ = [("inp", ctypes.c_void_p * MAX_IO), ("out", ctypes.c_void_p * MAX_IO),
                ("rows", ctypes.c_longlong), ("row_offset", ctypes.c_longlong),
                ("cols", ctypes.c_longlong), ("status", ctypes.c_void_p)]


class GemmArgs(ctypes.Structure):
    """molten_gemm_args / molten::GemmArgs (448 bytes, 64-byte aligned on
    the device side; the explicit tail keeps the host copy the same size)."""
    _fields_ = [("tmap_a", ctypes.c_ubyte * 128), ("tmap_b", ctypes.c_ubyte * 128),
                ("inp", ctypes.c_void_p * MAX_IO), ("out", ctypes.c_void_p * MAX_IO),
                ("m", ctypes.c_longlong), ("n", ctypes.c_longlong), ("k", ctypes.c_longlong),
                ("row_offset", ctypes.c_longlong), ("status", ctypes.c_void_p),
                ("batch", ctypes.c_int), ("pad_", ctypes.c_int), ("work", ctypes.c_void_p),
                ("tile_count", ctypes.c_void_p)]


class AttnArgs(ctypes.Structure):
    """molten_attn_args / molten::AttnArgs (448 bytes, 64-byte aligned on the
    device side)."""
    _fields_ = [("tmap_q", ctypes.c_ubyte * 128), ("tmap_k", ctypes.c_ubyte * 128),
                ("tmap_p", ctypes.c_ubyte * 128), ("out", ctypes.c_void_p),
                ("m", ctypes.c_longlong), ("n", ctypes.c_longlong), ("d", ctypes.c_longlong),
                ("row_offset", ctypes.c_longlong), ("status", ctypes.c_void_p),
                ("batch", ctypes.c_int), ("tail_", ctypes.c_ubyte * 12)]


assert ctypes.sizeof(RowArgs) == 160
assert ctypes.sizeof(AttnArgs) == 448
assert ctypes.sizeof(GemmArgs) == 448


class MoltenError(RuntimeError):
    """A call into libmolten_rt.so failed."""


_lib = None


def load_library(path: os.PathLike = None):
    """Load (once) and return the runtime library; raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise MoltenError(
            f"{p} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(molten_b200.build.build_runtime)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def last_error() -> str:
    return load_library().molten_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != MOLTEN_OK:
        raise MoltenError(f"{what} failed (code {rc}): {last_error()}")


def device_count() -> int:
    n = ctypes.c_int(0)
    check(load_library().molten_device_count(ctypes.byref(n)), "molten_device_count")
    return n.value


class Module:
    """A cubin loaded on one device."""

    def __init__(self, cubin_path: str, device: int):
        self.lib = load_library()
        self.handle = ctypes.c_void_p()
        self.device = device
        self.path = cubin_path
        check(self.lib.molten_module_load(str(cubin_path).encode(), device,
                                          ctypes.byref(self.handle)),
              f"loading {cubin_path}")

    def kernel_info(self, name: str) -> dict:
        regs, thr, smem = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        check(self.lib.molten_kernel_info(self.handle, name.encode(), ctypes.byref(regs),
                                          ctypes.byref(thr), ctypes.byref(smem)),
              f"kernel info of {name}")
        return {"registers": regs.value, "max_threads": thr.value, "static_smem": smem.value}

    def max_resident(self, name: bytes, cfg: LaunchCfg) -> tuple:
        """(CTAs per SM, clusters on the device) that fit at once with cfg."""
        per_sm, clusters = ctypes.c_int(), ctypes.c_int()
        check(self.lib.molten_max_resident(self.handle, name, ctypes.byref(cfg),
                                           ctypes.byref(per_sm), ctypes.byref(clusters)),
              f"occupancy of {name.decode()}")
        return per_sm.value, clusters.value

    def launch(self, name: bytes, cfg: LaunchCfg, params, stream: int) -> None:
        rc = self.lib.molten_launch(self.handle, name, ctypes.byref(cfg), ctypes.byref(params),
                                    ctypes.sizeof(params), ctypes.c_void_p(stream))
        if rc != MOLTEN_OK:
            raise MoltenError(f"launching {name.decode()} failed (code {rc}): {last_error()}")

    def unload(self) -> None:
        if self.handle:
            check(self.lib.molten_module_unload(self.handle), "unloading module")
            self.handle = ctypes.c_void_p()


def encode_tma_2d(dtype_code: int, base: int, inner: int, outer: int, row_stride_bytes: int,
                  box_inner: int, box_outer: int, swizzle: int = 128) -> bytes:
    """128-byte TMA descriptor for a row-major 2-D matrix; ``swizzle`` is the
    span in bytes (0 none, 32, 64, 128)."""
    lib = load_library()
    buf = ctypes.create_string_buffer(128 + 64)
    addr = ctypes.addressof(buf)
    aligned = (addr + 63) & ~63
    check(lib.molten_encode_tma_2d(ctypes.c_void_p(aligned), dtype_code, ctypes.c_void_p(base),
                                   inner, outer, row_stride_bytes, box_inner, box_outer,
                                   int(swizzle)),
          "encoding a TMA descriptor")
    return ctypes.string_at(aligned, 128)


def status_word(device: int) -> int:
    p = ctypes.c_void_p()
    check(load_library().molten_status_word(device, ctypes.byref(p)), "status word")
    return p.value


def read_status(device: int, reset: bool = True) -> int:
    v = ctypes.c_int(0)
    check(load_library().molten_read_status(device, ctypes.byref(v), 1 if reset else 0),
          "reading the status word")
    return v.value
