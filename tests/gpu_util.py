"""Helpers for the GPU parity tests: the north_star tolerance, written out once."""
import torch

# bf16 inputs, fp32 accumulation: max |diff| / max |ref| <= 1e-2 and cosine >= 0.9999.
MAX_REL = 1e-2
MIN_COS = 0.9999


def parity(out: torch.Tensor, ref: torch.Tensor):
    o = out.detach().float().cpu().reshape(-1)
    r = ref.detach().float().cpu().reshape(-1)
    assert o.shape == r.shape, (o.shape, r.shape)
    if r.numel() == 0:
        return 0.0, 1.0
    assert torch.isfinite(o).all(), "non-finite output"
    d = (o - r).abs().max().item()
    rel = d / max(r.abs().max().item(), 1e-12)
    cos = torch.nn.functional.cosine_similarity(o.double(), r.double(), dim=0).item()
    return rel, cos


def assert_parity(out, ref, what=""):
    rel, cos = parity(out, ref)
    assert rel <= MAX_REL and cos >= MIN_COS, f"{what}: max_rel={rel:.3e} cos={cos:.6f}"


def reference_allclose(out, ref, dtype=torch.bfloat16):
    """The reference's own acceptance check (benchmarks/benchmark.py:256-259)."""
    atol = 1e-2 if dtype == torch.bfloat16 else 5e-3
    return torch.allclose(out.float().cpu(), ref.float().cpu(), atol=atol, rtol=1e-2)
