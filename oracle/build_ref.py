"""Build recipe for the reference's own ``_C`` extension into ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY. The product never imports, links or runs anything
built here.  The reference kernels serve one purpose: a second, independent
pin for the oracle and for the CUDA path, run side by side on the GPU box in
the ``-m gpu`` parity tests (``tests/test_ref_cuda_parity.py``).

The recipe compiles the seven reference sources in place (they are read, never
copied) with ``torch.utils.cpp_extension.load``: it is this repository's own
recipe, not the reference's ``setup.py``.  The module is named
``metagross_ref_C`` so that it can never be mistaken for the product's ``_C``.
It targets sm_100 (the arch the reference's own build would pick for
``TORCH_CUDA_ARCH_LIST=10.0``).

Run where the reference sources are mounted (the path argument, else
``$METAGROSS_REFERENCE_ROOT``, else the default mount point below):
    python oracle/build_ref.py [/path/to/reference]
The output ``oracle/_ref/metagross_ref_C*.so`` is git-ignored but travels to
the GPU box with the working tree.
"""
from __future__ import annotations

import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
BUILD_DIR = os.path.join(OUT_DIR, "build")
REF_SOURCES = [
    "csrc/bindings.cpp",
    "csrc/sanity_add.cu",
    "csrc/quantize.cu",
    "csrc/dequantize.cu",
    "csrc/paged_attention.cu",
    "csrc/quantize_int4.cu",
    "csrc/dequantize_int4.cu",
]


# Where the reference's sources are read from: the environment variable
# METAGROSS_REFERENCE_ROOT, else the recipe's default mount point.
DEFAULT_REFERENCE_ROOT = "/root/reference"


def reference_root() -> str:
    return os.environ.get("METAGROSS_REFERENCE_ROOT", DEFAULT_REFERENCE_ROOT)


def sources_present(root: str | None = None) -> bool:
    root = root or reference_root()
    return all(os.path.exists(os.path.join(root, s)) for s in REF_SOURCES)


def built_module_path() -> str | None:
    hits = sorted(glob.glob(os.path.join(OUT_DIR, "metagross_ref_C*.so")))
    return hits[0] if hits else None


def build(root: str | None = None, verbose: bool = False) -> str | None:
    """Compile the reference ``_C`` if its sources are present; return the .so path."""
    root = root or reference_root()
    srcs = [os.path.join(root, s) for s in REF_SOURCES]
    if not all(os.path.exists(s) for s in srcs):
        return built_module_path()
    newest_src = max(os.path.getmtime(s) for s in srcs)
    existing = built_module_path()
    if existing and os.path.getmtime(existing) >= newest_src:
        return existing
    from torch.utils.cpp_extension import load

    os.makedirs(BUILD_DIR, exist_ok=True)
    load(
        name="metagross_ref_C",
        sources=srcs,
        extra_include_paths=[os.path.join(root, "csrc")],
        extra_cuda_cflags=["-O3", "-gencode=arch=compute_100,code=sm_100"],
        extra_cflags=["-O3"],
        build_directory=BUILD_DIR,
        verbose=verbose,
        is_python_module=True,
    )
    so = sorted(glob.glob(os.path.join(BUILD_DIR, "metagross_ref_C*.so")))
    if not so:
        return None
    dst = os.path.join(OUT_DIR, os.path.basename(so[0]))
    shutil.copy2(so[0], dst)
    return dst


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
