"""The reference's own tests for this path, run unchanged against this
repository through the ``metagross`` import path (the alias package at the
repository root).

Where the reference's sources are mounted (``$METAGROSS_REFERENCE_ROOT``, else
the recipe default of oracle/build_ref.py), its test files for the paged cache,
allocator, quantize/dequantize ops and attention (tests/test_quantize.py,
test_int4.py, test_attention.py, test_cuda_stress.py, test_edge_cases.py,
test_block_allocator.py, test_sanity.py and their helper tests/reference.py)
are copied to a temporary directory -- they are read, never stored in this
repository -- and run by pytest in a child process with this repository first
on ``sys.path``.  Without a GPU most of them skip themselves; on a B200 with
the reference mounted every one runs.  Not marked gpu: it needs the reference
sources, which GPU boxes do not carry.
"""
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FILES = ["__init__.py", "reference.py", "test_quantize.py", "test_int4.py", "test_attention.py",
         "test_cuda_stress.py", "test_edge_cases.py", "test_block_allocator.py", "test_sanity.py"]


def _reference_tests_dir():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import build_ref

    d = os.path.join(build_ref.reference_root(), "tests")
    return d if all(os.path.exists(os.path.join(d, f)) for f in FILES) else None


def test_reference_suite_passes_against_this_package(tmp_path):
    src = _reference_tests_dir()
    if src is None:
        pytest.skip("reference sources not mounted")
    dst = tmp_path / "tests"
    dst.mkdir()
    for f in FILES:
        shutil.copy(os.path.join(src, f), dst / f)
    (tmp_path / "conftest.py").write_text(f"import sys\nsys.path.insert(0, {ROOT!r})\n")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "tests"], cwd=tmp_path,
                       capture_output=True, text=True, timeout=900)
    tail = "\n".join(r.stdout.splitlines()[-15:])
    assert r.returncode == 0, tail
    assert " failed" not in tail and " error" not in tail, tail
    assert " passed" in tail, tail
