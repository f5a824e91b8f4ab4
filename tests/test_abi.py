"""The C-ABI library: it loads, exports every symbol include/*.h declares, and
its host-only entry points behave without a GPU (no compute calls here)."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def _declared_symbols() -> list[str]:
    text = "\n".join(p.read_text() for p in sorted((REPO / "include").glob("*.h")))
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lt_[a-z0-9_]+)\s*\(", text)))


def test_library_built(pkg):
    assert pkg.LIB_PATH.exists(), "run llmtoy-zig_b200/build.py"


def test_exports_every_declared_symbol(pkg):
    lib = pkg.load_library()
    declared = _declared_symbols()
    assert declared, "no declarations parsed"
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, f"declared but not exported: {missing}"
    assert sorted(pkg.EXPORTS) == declared


def test_exports_are_c_linkage(pkg):
    out = subprocess.run(["nm", "-D", "--defined-only", str(pkg.LIB_PATH)], capture_output=True, text=True).stdout
    names = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for s in _declared_symbols():
        assert s in names, f"{s} is not an unmangled dynamic symbol"


def test_row_bytes_host_only(pkg):
    lib = pkg.load_library()
    assert lib.lt_row_bytes(pkg.Q4_K, 2048) == 8 * 144
    assert lib.lt_row_bytes(pkg.Q6_K, 2816) == 11 * 210
    assert lib.lt_row_bytes(pkg.Q8_0, 896) == 28 * 34
    assert lib.lt_row_bytes(pkg.F16, 10) == 20
    assert lib.lt_row_bytes(3, 256) == 0  # Q4_1 is not supported
    for t in (pkg.F32, pkg.F16, pkg.Q8_0, pkg.Q4_K, pkg.Q6_K):
        assert lib.lt_row_bytes(t, 2048) == pkg.row_bytes(t, 2048)


def test_api_version_and_status_strings(pkg):
    lib = pkg.load_library()
    assert lib.lt_api_version() == 1
    assert lib.lt_status_string(0) == b"ok"
    assert lib.lt_status_string(5) == b"device wait timed out"


def test_null_arguments_rejected_without_device(pkg):
    lib = pkg.load_library()
    assert lib.lt_init(0, None) == 1  # LT_EINVAL before touching CUDA
    assert lib.lt_tensor_describe(None, None) == 1
    assert lib.lt_sync(None) == 1


def test_no_cpu_fallback_without_gpu(pkg):
    """On a host without a usable sm_100 device the context refuses to exist."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(pkg.LtError) as ei:
        pkg.Context(0)
    assert ei.value.status == 6  # LT_ENODEV


def test_cpp_host_header_compiles():
    """The C++ mirror of the reference operator names builds against the ABI."""
    hdr = REPO / "llmtoy-zig_b200" / "host" / "llmtoy_ops.hpp"
    res = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Wextra", f"-I{REPO / 'include'}",
                          "-x", "c++", str(hdr)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
