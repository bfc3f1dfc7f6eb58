"""CPU-side behaviour of the Python API: names, enum values and host-side checks identical to the
reference (grouped_gemm_opt/__init__.py:1-5, ops.py:8-64)."""
import pytest
import torch


def test_public_names():
    import grouped_gemm_opt as g
    for name in ["grouped_gemm_opt", "TileConfig", "triton_fused_moe", "triton_grouped_gemm"]:
        assert name in g.__all__ and hasattr(g, name)
    assert hasattr(g, "fused_moe")


def test_tile_config_values_match_reference():
    from grouped_gemm_opt import TileConfig
    assert {t.name: int(t) for t in TileConfig} == {
        "Co_128x128x64": 0, "Co_128x256x64": 1, "PP_128x128x128": 2, "PP_128x256x64": 3,
        "AUTO": 4, "CuBLAS_Seq": 5}


def test_cpu_tensors_rejected_like_reference():
    from grouped_gemm_opt import grouped_gemm_opt
    x = torch.randn(4, 8, dtype=torch.bfloat16)
    w = torch.randn(2, 8, 8, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        grouped_gemm_opt(x, w, torch.tensor([2, 2]))


def test_native_binding_loaded():
    from grouped_gemm_opt._native import _C
    assert _C.abi_version() == 100
    for fn in ["grouped_gemm_opt_forward", "grouped_gemm_segments", "grouped_gemm_swiglu",
               "moe_route", "moe_permute", "moe_combine", "workspace_error"]:
        assert hasattr(_C, fn)


def test_fused_moe_shape_checks():
    from grouped_gemm_opt import fused_moe
    x = torch.randn(4, 16)
    with pytest.raises(AssertionError):
        fused_moe(x, torch.randn(4, 8), torch.randn(8, 32, 16), torch.randn(8, 16, 8), 9)
    with pytest.raises(AssertionError):  # wrong local expert count
        fused_moe(x, torch.randn(4, 8), torch.randn(4, 32, 16), torch.randn(4, 16, 8), 2)


def test_bench_reference_arm_prints_the_same_config(capsys):
    """The reference arm of bench.py (the reference's CPU algorithm for the layer) prints the same
    metric, unit and config dict as the GPU arm, so the two lines compare like for like."""
    import importlib.util
    import json
    import os
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    argv = sys.argv
    sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3",
                "--ref-tokens", "16", "--gpus", "2"]
    try:
        bench.main()
    finally:
        sys.argv = argv
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == bench.UNIT and line["config"] == bench.layer_config(2)
    assert line["value"] > 0 and line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["scaling"] == "strong" and line["higher_is_better"] is True
