"""nvcc driver: builds libmolten_rt.so and the generated kernels' cubins.

Every device build targets sm_100a only:
``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3``.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import threading
import tempfile
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC_DIR = PKG_DIR / "csrc"
ENGINE_INCLUDE = CSRC_DIR / "include"
ABI_INCLUDE = REPO_DIR / "include"
LIB_DIR = PKG_DIR / "lib"
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUBIN_FLAGS = GENCODE + ["-cubin", "-O3", "-std=c++17", "-lineinfo",
                         "-diag-suppress", "177,550"]


class BuildError(RuntimeError):
    """nvcc failed."""


def nvcc_path() -> str:
    for cand in (os.environ.get("MOLTEN_NVCC"),
                 shutil.which("nvcc"),
                 os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"),
                 "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise BuildError("nvcc not found (set MOLTEN_NVCC or CUDA_HOME)")


def _engine_digest() -> str:
    h = hashlib.sha256()
    for f in sorted((ENGINE_INCLUDE / "molten").glob("*.cuh")):
        h.update(f.name.encode())
        h.update(f.read_bytes())
    return h.hexdigest()


def default_cache_dir() -> Path:
    env = os.environ.get("MOLTEN_CACHE_DIR")
    if env:
        return Path(env)
    d = PKG_DIR / "_kcache"
    try:
        d.mkdir(exist_ok=True)
        # a probe per process and thread: concurrent builders must not
        # remove each other's probe
        probe = d / f".w.{os.getpid()}.{threading.get_ident()}"
        probe.write_text("")
        probe.unlink()
        return d
    except OSError:
        return Path(tempfile.gettempdir()) / "molten_cache"


def cubin_key(source: str, extra_flags=()) -> str:
    h = hashlib.sha256()
    h.update(source.encode())
    h.update(" ".join(CUBIN_FLAGS + list(extra_flags)).encode())
    h.update(_engine_digest().encode())
    return h.hexdigest()[:20]


def build_cubin(source: str, name: str, cache_dir: os.PathLike = None, verbose: bool = False,
                extra_flags=()) -> Path:
    """Compile a generated module to a cubin (cached by content hash)."""
    cache = Path(cache_dir) if cache_dir else default_cache_dir()
    cache.mkdir(parents=True, exist_ok=True)
    key = cubin_key(source, extra_flags)
    cubin = cache / f"{name}_{key}.cubin"
    if cubin.exists() and cubin.stat().st_size > 0:
        return cubin
    cu = cache / f"{name}_{key}.cu"
    cu.write_text(source)
    # private temporary per build (process and thread): two builders of the
    # same source each publish a complete file with an atomic rename
    tmp = cache / f".{name}_{key}.{os.getpid()}.{threading.get_ident()}.cubin"
    cmd = [nvcc_path(), *CUBIN_FLAGS, *extra_flags, f"-I{ENGINE_INCLUDE}", "-o", str(tmp), str(cu)]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise BuildError(f"nvcc failed for {name} ({cu}):\n{res.stderr[-4000:]}")
    os.replace(tmp, cubin)      # atomic: concurrent builders never see a partial file
    return cubin


def build_runtime(verbose: bool = False, force: bool = False) -> Path:
    """Build molten_b200/lib/libmolten_rt.so (the C-ABI runtime)."""
    LIB_DIR.mkdir(exist_ok=True)
    out = LIB_DIR / "libmolten_rt.so"
    srcs = [CSRC_DIR / "runtime.cu", CSRC_DIR / "noalloc_scores.cu"]
    deps = srcs + [ABI_INCLUDE / "molten_rt.h"] + list((ENGINE_INCLUDE / "molten").glob("*.cuh"))
    if out.exists() and not force and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return out
    tmp = LIB_DIR / f".libmolten_rt.{os.getpid()}.so"
    cmd = [nvcc_path(), *GENCODE, "-lineinfo", "-O2", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-cudart", "static", f"-I{ABI_INCLUDE}", f"-I{ENGINE_INCLUDE}",
           "-o", str(tmp), *map(str, srcs)]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise BuildError(f"building libmolten_rt.so failed:\n{res.stderr[-4000:]}")
    os.replace(tmp, out)
    return out
