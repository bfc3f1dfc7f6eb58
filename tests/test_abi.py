"""CPU checks of the C ABI library: it loads without a GPU, exports every entry point that
include/ggo.h declares, and validates arguments before touching the device."""
import ctypes
import os
import re

import pytest

from build_ext import lib_path

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "ggo.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ggo_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    assert lib_path().exists(), "libggo_b200.so not built"
    return ctypes.CDLL(str(lib_path()))


def test_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_metadata_calls(lib):
    assert lib.ggo_version() == 100
    lib.ggo_status_string.restype = ctypes.c_char_p
    for code in range(0, 12):
        assert lib.ggo_status_string(code)
    lib.ggo_workspace_size.restype = ctypes.c_size_t
    assert lib.ggo_workspace_size() == 256
    lib.ggo_kernel_launches.restype = ctypes.c_uint64
    assert lib.ggo_kernel_launches() >= 0
    lib.ggo_moe_route_scratch_bytes.restype = ctypes.c_size_t
    lib.ggo_moe_route_scratch_bytes.argtypes = [ctypes.c_int64, ctypes.c_int]
    assert lib.ggo_moe_route_scratch_bytes(16384, 8) == (16384 // 32 + 1) * 8 * 4


def _gemm(lib, a=1 << 20, b=1 << 20, c=1 << 20, cnt=1 << 20, e=8, t=256, n=1024, k=512, dt=0,
          tc=4, ws=1 << 20):
    f = lib.ggo_grouped_gemm
    f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                          ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_void_p, ctypes.c_void_p]
    # pointers are never dereferenced on these error paths (validated before any device work)
    return f(a, b, c, cnt, e, t, n, k, dt, tc, 1, ws, None)


def test_argument_validation_before_device_work(lib):
    assert _gemm(lib, a=None) == 1            # GGO_ERR_INVALID_ARG
    assert _gemm(lib, e=0) == 1
    assert _gemm(lib, tc=9) == 1
    assert _gemm(lib, dt=7) == 3              # GGO_ERR_DTYPE
    assert _gemm(lib, k=500) == 4             # GGO_ERR_ALIGNMENT (K % 8)
    assert _gemm(lib, n=1001) == 4
    assert _gemm(lib, a=(1 << 20) + 8) == 4   # 16-byte alignment
    assert _gemm(lib, e=2000) == 5            # GGO_ERR_TOO_MANY_SEGMENTS
    assert _gemm(lib, t=0) == 0               # empty problem: nothing to launch


def test_moe_validation(lib):
    f = lib.ggo_moe_route
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int] + \
        [ctypes.c_void_p] * 5
    p = 1 << 20
    assert f(p, 16, 8, 9, p, p, p, p, None) == 1     # top_k > E
    assert f(p, 16, 2048, 2, p, p, p, p, None) == 1  # E > 1024
    assert f(None, 16, 8, 2, p, p, p, p, None) == 1


def test_mxfp8_metadata_and_validation(lib):
    lib.ggo_mxfp8_scale_bytes.restype = ctypes.c_size_t
    lib.ggo_mxfp8_scale_bytes.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int64]
    assert lib.ggo_mxfp8_scale_bytes(256, 2, 512) == (2 + 2) * 4 * 512
    assert lib.ggo_mxfp8_scale_bytes(256, 2, 100) == 0   # K must be a multiple of 128
    lib.ggo_mxfp8_glu_rows.restype = ctypes.c_int64
    lib.ggo_mxfp8_glu_rows.argtypes = [ctypes.c_int64]
    assert lib.ggo_mxfp8_glu_rows(200) == 512 and lib.ggo_mxfp8_glu_rows(256) == 512
    q = lib.ggo_quantize_mxfp8
    q.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                  ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    p = 1 << 20
    assert q(None, 0, p, 1, 16, 128, p, p, None) == 1
    assert q(p, 0, p, 1, 16, 100, p, p, None) == 4      # K % 128
    assert q(p, 7, p, 1, 16, 128, p, p, None) == 3      # dtype
    assert q(p, 0, p, 2000, 16, 128, p, p, None) == 5   # too many segments
    assert q(p, 0, p, 1, 0, 128, p, p, None) == 0       # nothing to do
    g = lib.ggo_grouped_gemm_mxfp8
    g.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_int] + \
        [ctypes.c_int64] * 3 + [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    assert g(p, p, p, p, p, p, 8, 8, 256, 1024, 64, 1, p, None) == 4   # K % 128
    assert g(p, None, p, p, p, p, 8, 8, 256, 1024, 128, 1, p, None) == 1
    assert g(p, p + 8, p, p, p, p, 8, 8, 256, 1024, 128, 1, p, None) == 4  # scale alignment


C_PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "ggo.h"
int main(void) {
  /* metadata and host-side validation only: no GPU is needed for these paths */
  if (ggo_version() != 100) return 1;
  if (ggo_workspace_size() != GGO_WORKSPACE_BYTES) return 2;
  if (strlen(ggo_status_string(GGO_ERR_ALIGNMENT)) == 0) return 3;
  char dummy[64];
  int st = ggo_grouped_gemm(NULL, dummy, dummy, (const int64_t*)dummy, 8, 256, 1024, 512,
                            GGO_DTYPE_BF16, GGO_TILE_AUTO, 1, dummy, (cudaStream_t)0);
  if (st != GGO_ERR_INVALID_ARG) return 4;
  st = ggo_grouped_gemm_noalloc(dummy, dummy, dummy, (const int64_t*)dummy,
                                GGO_NOALLOC_MAX_EXPERTS + 1, 16, 64, 64, GGO_DTYPE_BF16,
                                GGO_TILE_AUTO, 1, (cudaStream_t)0);
  if (st != GGO_ERR_TOO_MANY_SEGMENTS) return 5;
  printf("ok\n");
  return 0;
}
"""


def test_header_is_plain_c(tmp_path):
    """include/ggo.h compiles as C99 and a C program links and runs against libggo_b200.so."""
    import subprocess
    src = tmp_path / "abi.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "abi"
    inc = os.path.dirname(HEADER)
    libdir = os.path.dirname(str(lib_path()))
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", inc, "-I",
                        "/usr/local/cuda/include", str(src), "-o", str(exe), f"-L{libdir}",
                        "-lggo_b200", f"-Wl,-rpath,{libdir}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.returncode, r.stderr)
