"""Expert-parallel orchestration of fused_moe on CPU gloo ranks (world size 2 and 4).

The compute stages are replaced by the CPU oracle (MoEOps), so this exercises exactly the host
logic of grouped_gemm_opt/moe.py: count exchange, split sizes, row all-to-all into the
[source rank][local expert] segment layout, reverse all-to-all and combine. Dispatch indexing
must be bit-exact (checked on the rows each rank's gate/up stage receives); the layer output must
match the single-process oracle. A second test makes one rank fail before the exchange and checks
that the other rank gets an error from the process-group timeout instead of hanging.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import grouped_gemm_oracle as oracle

T_PER_RANK, H, F, E, K = 24, 32, 16, 8, 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(rank):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(T_PER_RANK, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T_PER_RANK, E, generator=g)
    return x, logits


def _weights():
    g = torch.Generator().manual_seed(7)
    wgu = (torch.randn(E, 2 * F, H, generator=g) * 0.1).to(torch.bfloat16)
    wd = (torch.randn(E, H, F, generator=g) * 0.1).to(torch.bfloat16)
    return wgu, wd


def cpu_ops(record):
    from grouped_gemm_opt.moe import MoEOps

    def route(logits, k):
        ids, w, tpe = oracle.route(logits.float().numpy(), k)
        return torch.from_numpy(ids), torch.from_numpy(w), torch.from_numpy(tpe), None

    def permute(x, ids, scratch, e):
        st, pos = oracle.permute_indices(ids.numpy(), e)
        return x[torch.from_numpy(st).long()], torch.from_numpy(st), torch.from_numpy(pos)

    def gate_up(xr, w, counts, ne, sort):
        record["x_recv"] = xr.clone()
        record["counts"] = counts.clone()
        return oracle.swiglu_gemm(xr, w, counts, ne).to(torch.bfloat16)

    def down(h, w, counts, ne, sort):
        return oracle.segments_gemm(h, w, counts, ne).to(torch.bfloat16)

    def combine(y, w, pos):
        return oracle.combine(y, w.numpy(), pos.numpy())

    return MoEOps(route, permute, gate_up, down, combine)


def _worker(rank, world, port, q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=8))
    try:
        from grouped_gemm_opt import fused_moe
        x, logits = _inputs(rank)
        wgu, wd = _weights()
        el = E // world
        mine = slice(rank * el, (rank + 1) * el)
        if rank == fail_rank:
            q.put((rank, "failed-on-purpose", None))
            raise SystemExit(0)  # leaves before the exchange: the host-side failure
        record = {}
        out = fused_moe(x, logits, wgu[mine].contiguous(), wd[mine].contiguous(), K,
                        ep_group=dist.group.WORLD, ops=cpu_ops(record))
        q.put((rank, "ok", (out.float().numpy(), record["x_recv"].float().numpy(),
                            record["counts"].numpy())))
    except SystemExit:
        pass
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, "error", repr(exc)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, status, payload = q.get(timeout=120)
        res[r] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def _expected_recv(rank, world):
    """Rows rank `rank` must receive: from every source, its rows for rank's experts, in the
    source's sorted order (expert-major, token order)."""
    el = E // world
    rows, counts = [], []
    for src in range(world):
        x, logits = _inputs(src)
        ids, _, tpe = oracle.route(logits.numpy(), K)
        st, _ = oracle.permute_indices(ids, E)
        start = int(tpe[:rank * el].sum())
        n = int(tpe[rank * el:(rank + 1) * el].sum())
        rows.append(x[torch.from_numpy(st[start:start + n]).long()].float().numpy())
        counts.extend(tpe[rank * el:(rank + 1) * el].tolist())
    return np.concatenate(rows), np.array(counts)


@pytest.mark.parametrize("world", [2, 4])
def test_ep_matches_single_process(world):
    res = _run(world)
    wgu, wd = _weights()
    for r in range(world):
        status, payload = res[r]
        assert status == "ok", payload
        out, x_recv, counts = payload
        exp_rows, exp_counts = _expected_recv(r, world)
        assert np.array_equal(counts, exp_counts)
        assert np.array_equal(x_recv, exp_rows)  # dispatch is bit-exact
        x, logits = _inputs(r)
        ref = oracle.moe_layer(x, logits, wgu, wd, K, round_to=torch.bfloat16).numpy()
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5)


def test_ep_rank_failure_is_reported_not_hung():
    res = _run(2, fail_rank=1)
    assert res[1][0] == "failed-on-purpose"
    assert res[0][0] == "error", res[0]
