"""Recipe: build the reference's hand-written CUDA kernels for sm_100a.

TEST INFRASTRUCTURE ONLY.  The reference ships its GPU comparison points as
one torch extension source, ``benchmarks/reference_kernels.cu`` (fused
RMSNorm :12-50, RMSNorm*SiLU*gate :104-144, GELU+bias :169-185, pybind
bindings :205-210).  This compiles that file, where it lies in the
reference checkout, with nvcc for sm_100a through torch's extension builder,
into ``oracle/_ref/molten_reference_kernels*.so``; nothing of the reference
is copied into the repository.  Only tests load the result, to check the
reference's kernels against the oracle and to time them beside this
library's kernels on the same GPU.

    python oracle/build_ref.py [REFERENCE_CHECKOUT]

The checkout is the argument, else $MOLTEN_REFERENCE, else the build
container's /root/reference.  Without a checkout (the GPU machines) nothing
is built and the prebuilt library, if any, is used.
"""

from __future__ import annotations

import glob
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "molten_reference_kernels"
SOURCE = Path("benchmarks") / "reference_kernels.cu"


def reference_dir(arg: str | None = None) -> Path | None:
    for cand in (arg, os.environ.get("MOLTEN_REFERENCE"), "/root/reference"):
        if cand and (Path(cand) / SOURCE).is_file():
            return Path(cand)
    return None


def built_library() -> Path | None:
    hits = sorted(glob.glob(str(OUT / f"{NAME}*.so")))
    return Path(hits[0]) if hits else None


def build(arg: str | None = None, verbose: bool = False) -> Path | None:
    """Compile the reference's kernels if a checkout is present and the
    library is missing or older than the source; returns the library."""
    ref = reference_dir(arg)
    lib = built_library()
    if ref is None:
        return lib
    src = ref / SOURCE
    if lib is not None and lib.stat().st_mtime >= src.stat().st_mtime:
        return lib
    OUT.mkdir(exist_ok=True)
    # sm_100a only (torch's own architecture list would add every arch it
    # was built for)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from torch.utils.cpp_extension import load
    load(name=NAME, sources=[str(src)], build_directory=str(OUT),
         extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
         verbose=verbose)
    return built_library()


def load_library():
    """The built extension module (torch must be importable), or None."""
    lib = built_library()
    if lib is None:
        return None
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the extension links against torch's libraries)
    loader = importlib.machinery.ExtensionFileLoader(NAME, str(lib))
    spec = importlib.util.spec_from_file_location(NAME, str(lib), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    out = build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True)
    print(out if out else "no reference checkout found: nothing built")
