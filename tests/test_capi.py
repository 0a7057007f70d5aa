"""The C-ABI library loads and exports every entry point include/svdq_b200.h declares
(no compute calls: runs without a GPU)."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "svdq_b200.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(svdq_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from krea2_svdquant_b200 import build
    build.build()
    return ctypes.CDLL(build.LIB_PATH)


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("svdq_act_quant", "svdq_w4a16_prep", "svdq_linear_gemm", "svdq_repack_weight",
                 "svdq_build_up_hl", "svdq_last_error", "svdq_device_error"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_binding_covers_header():
    from krea2_svdquant_b200 import _lib
    assert set(declared_functions()) <= set(_lib.SIGNATURES)


def test_version_and_error_string(lib):
    from krea2_svdquant_b200 import _lib
    L = _lib.lib()
    assert L.svdq_version().decode().startswith("svdq_b200")
    assert isinstance(L.svdq_last_error(), bytes)


def test_invalid_arguments_rejected_without_gpu():
    """Host-side validation runs before any CUDA call: a bad group size is an error status."""
    from krea2_svdquant_b200 import _lib
    L = _lib.lib()
    st = L.svdq_act_quant(ctypes.c_void_p(16), 8, ctypes.c_void_p(16), None, 0, None, None, 0,
                          4, 8, 64, 96, None, None, None, None, 0, None, 0, None)
    assert st == 1
    assert "a_group" in L.svdq_last_error().decode()
    st = L.svdq_linear_gemm(None, None, None, None, 0, None, None, 0, 8, 4, 8, 64, None)
    assert st == 1
    st = L.svdq_linear_gemm(ctypes.c_void_p(256), ctypes.c_void_p(256), None, None, 0, None, ctypes.c_void_p(256),
                            0, 8, 4, 8, 96, None)
    assert st == 1 and "K_pad" in L.svdq_last_error().decode()


C_PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "svdq_b200.h"
int main(void) {
  const char* v = svdq_version();
  if (!v || strncmp(v, "svdq_b200", 9) != 0) return 2;
  /* argument validation runs before any CUDA call: a bad group size is an error status */
  int st = svdq_act_quant((const void*)16, 8, (const void*)16, NULL, 0, NULL, NULL, 0, 4, 8, 64, 96,
                          NULL, NULL, NULL, NULL, 0, NULL, 0, (cudaStream_t)0);
  if (st != SVDQ_ERR_INVALID_ARGUMENT) return 3;
  if (strstr(svdq_last_error(), "a_group") == NULL) return 4;
  if (svdq_act_quant_workspace_bytes(0, 64, 32, 0) != 0) return 5;
  if (svdq_act_quant_noalloc_scratch_bytes() != (size_t)8 << 20) return 6;
  if (svdq_prefetcher_create(0, 0, NULL) != SVDQ_ERR_INVALID_ARGUMENT) return 7;
  printf("ok %s\n", v);
  return 0;
}
"""


def test_header_is_c_and_links(tmp_path):
    """The header compiles as C99 and a C program links against the library and calls it."""
    import shutil
    import subprocess
    from krea2_svdquant_b200 import build
    build.build()
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    src = tmp_path / "abi.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "abi"
    lib_dir = os.path.dirname(build.LIB_PATH)
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), "-I", cuda_inc,
                    str(src), "-L", lib_dir, "-lsvdq_b200", "-Wl,-rpath," + lib_dir, "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, (out.returncode, out.stdout, out.stderr)
    assert out.stdout.startswith("ok svdq_b200")
