"""Loads the native extension. There is no fallback: if ``_C`` (and the ``libggo_b200.so`` it links)
is missing, importing the package raises, naming the build command."""
try:
    from grouped_gemm_opt import _C  # noqa: F401
except ImportError as exc:  # pragma: no cover - exercised only on a broken install
    raise ImportError(
        "grouped_gemm_opt native extension is not built; run "
        "`python groupedgemm-opt_b200/build_ext.py` (needs nvcc for sm_100a)") from exc

__all__ = ["_C"]
