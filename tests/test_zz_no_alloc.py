"""The allocation-free grouped GEMM entry point (ggo_grouped_gemm_noalloc).

Some callers cannot allocate device memory: code that runs inside a custom allocator's own
callbacks, plugin hosts that give a kernel library no allocator, or code that owns no device
memory. For them the library keeps its scratch in a fixed device array of its own. This test calls
that entry point through the C ABI (ctypes, raw device pointers) twice in a row and checks each
result against the regular entry point, ggo_grouped_gemm, within the parity tolerance of the other
GPU tests. The file name makes pytest collect it last.
"""
import ctypes

import pytest
import torch

from gpu_util import assert_parity
from inputs import EDGE_CASES, edge_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _lib():
    from build_ext import lib_path
    lib = ctypes.CDLL(str(lib_path()))
    common = [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.ggo_grouped_gemm.argtypes = common + [ctypes.c_void_p, ctypes.c_void_p]
    lib.ggo_grouped_gemm_noalloc.argtypes = common + [ctypes.c_void_p]
    lib.ggo_workspace_size.restype = ctypes.c_size_t
    return lib


def test_noalloc_matches_regular_entry_point_twice():
    torch.cuda.init()
    lib = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    for case in ("ragged", "span_gt4"):  # two calls in a row with different problems
        x, w, tpe = edge_inputs(EDGE_CASES[case])
        xd, wd, td = x.to(DEV), w.to(DEV), tpe.to(DEV)
        E, T, N, K = w.size(0), x.size(0), w.size(1), w.size(2)
        ref = torch.empty(T, N, device=DEV, dtype=torch.bfloat16)
        ws = torch.zeros(lib.ggo_workspace_size(), dtype=torch.uint8, device=DEV)
        assert lib.ggo_grouped_gemm(xd.data_ptr(), wd.data_ptr(), ref.data_ptr(), td.data_ptr(),
                                    E, T, N, K, 0, 4, 1, ws.data_ptr(), stream) == 0
        for _ in range(2):
            out = torch.full((T, N), float("nan"), device=DEV, dtype=torch.bfloat16)
            st = lib.ggo_grouped_gemm_noalloc(xd.data_ptr(), wd.data_ptr(), out.data_ptr(),
                                              td.data_ptr(), E, T, N, K, 0, 4, 1, stream)
            assert st == 0
            torch.cuda.synchronize()
            assert_parity(out, ref, f"noalloc {case}")


def test_noalloc_rejects_too_many_experts():
    lib = _lib()
    p = 1 << 20  # never dereferenced: the size check comes first
    assert lib.ggo_grouped_gemm_noalloc(p, p, p, p, 1025, 16, 64, 64, 0, 4, 1, None) == 5
