"""Failure detection on the GPU without a fault: a test hook (GGO_TEST_INJECT_STALL) makes the
CTA that claims the first tile leave that tile's first pipeline stage unarmed and lowers the
bounded-wait limit to ~10 ms. The kernel
must return on its own, record a timeout in the workspace (read back as RuntimeError by
check_device_errors) and leave the context usable: the next normal call is correct."""
import time

import pytest
import torch

import grouped_gemm_oracle as oracle
from gpu_util import assert_parity
from inputs import gemm_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("tc", [1, 3])  # single-CTA 128x256 kernel, CTA-pair kernel
def test_bounded_wait_times_out_and_recovers(tc, monkeypatch):
    import grouped_gemm_opt as ggo
    x, w, tpe = gemm_inputs([700, 300, 1100, 20], 512, 1024, seed=tc)
    xd, wd, td = x.to(DEV), w.to(DEV), tpe.to(DEV)
    ggo.check_device_errors(0)
    monkeypatch.setenv("GGO_TEST_INJECT_STALL", "1")
    t0 = time.time()
    ggo.grouped_gemm_opt(xd, wd, td, tc)
    torch.cuda.synchronize()
    assert time.time() - t0 < 30.0
    with pytest.raises(RuntimeError, match="error code 8$"):  # GGO_ERR_DEVICE_TIMEOUT
        ggo.check_device_errors(0)
    monkeypatch.delenv("GGO_TEST_INJECT_STALL")
    out = ggo.grouped_gemm_opt(xd, wd, td, tc)
    torch.cuda.synchronize()
    ggo.check_device_errors(0)
    assert_parity(out, oracle.sequential_gemm(x, w, tpe), f"after timeout tc={tc}")


def test_ep_peer_wait_times_out_then_succeeds():
    """The expert-parallel peer wait on one GPU: an epoch nobody posted makes the bounded wait
    expire (recorded as GGO_ERR_DEVICE_TIMEOUT), a posted one passes."""
    import grouped_gemm_opt as ggo
    from grouped_gemm_opt import _C
    E = 8
    board = torch.zeros(_C.ep_board_bytes(E) // 8, dtype=torch.int64, device=DEV)
    ggo.check_device_errors(0)
    _C.ep_wait(board.data_ptr(), 1, E, 3, 1, 1 << 24, 0)  # nothing posted epoch 1 for slot 3
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="error code 8$"):
        ggo.check_device_errors(0)
    _C.ep_signal([board.data_ptr()], 0, E, 3, 1, 0)
    _C.ep_wait(board.data_ptr(), 1, E, 3, 1, 1 << 24, 0)
    torch.cuda.synchronize()
    ggo.check_device_errors(0)
    assert int(board[8 * E + 3 * 8 + 0]) == 1  # flags[slot 3][rank 0]


def test_checked_combine_poisons_after_expired_wait():
    """After an expired peer wait the checked combine (the last stage of the fused
    expert-parallel layer) returns NaN rows instead of numbers built from stale buffers; once the
    error is read and cleared it combines normally again."""
    import grouped_gemm_opt as ggo
    from grouped_gemm_opt import _C
    E, T, H, k = 8, 16, 64, 2
    g = torch.Generator().manual_seed(0)
    y = torch.randn(T * k, H, generator=g).to(torch.bfloat16).to(DEV)
    w = torch.rand(T, k, generator=g).to(DEV)
    pos = torch.randperm(T * k, generator=g).to(torch.int32).to(DEV)
    ggo.check_device_errors(0)
    good = _C.moe_combine(y, w, pos, True)
    assert torch.isfinite(good.float()).all()
    board = torch.zeros(_C.ep_board_bytes(E) // 8, dtype=torch.int64, device=DEV)
    _C.ep_wait(board.data_ptr(), 1, E, 2, 1, 1 << 24, 0)  # nobody posts: the wait expires
    bad = _C.moe_combine(y, w, pos, True)
    torch.cuda.synchronize()
    assert torch.isnan(bad.float()).all()
    assert torch.isfinite(_C.moe_combine(y, w, pos).float()).all()  # unchecked form unaffected
    with pytest.raises(RuntimeError, match="error code"):
        ggo.check_device_errors(0)
    again = _C.moe_combine(y, w, pos, True)
    assert torch.equal(again, good)
