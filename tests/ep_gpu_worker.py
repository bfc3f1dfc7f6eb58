"""Worker for tests/test_ep_gpu.py, launched by torchrun with one rank per GPU (NCCL).

Every rank builds the same global problem from seeds that do not depend on the number of ranks
(tokens and logits from one seed, expert e's weights from seed base + e), runs the
expert-parallel fused_moe on its token slice with its slice of experts -- the NCCL all-to-all
path, and the fused peer-memory path twice (its buffers are reused across layers) -- and sends
a seeded sample of output tokens to rank 0, which checks them against the CPU oracle (all
experts, global routing) at the parity bar of tests/gpu_util.py. Rank 0 prints
"EP_OK <path> <max_rel> <cos>" per path, or raises.

argv: T H F E top_k [n_sample]
"""
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "groupedgemm-opt_b200"))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
sys.path.insert(0, HERE)


def expert_weights(e, H, F, device="cuda"):
    g = torch.Generator(device=device).manual_seed(1000 + e)
    wgu = (torch.randn(2 * F, H, device=device, generator=g) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(H, F, device=device, generator=g) * 0.02).to(torch.bfloat16)
    return wgu, wd


def main():
    T, H, F, E, k = (int(a) for a in sys.argv[1:6])
    n_sample = int(sys.argv[6]) if len(sys.argv) > 6 else 48
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dist.barrier()
    from grouped_gemm_opt import EPBuffers, fused_moe
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, device="cuda", generator=g)
    tl, el = T // world, E // world
    wgl = torch.empty(el, 2 * F, H, dtype=torch.bfloat16, device="cuda")
    wdl = torch.empty(el, H, F, dtype=torch.bfloat16, device="cuda")
    for i in range(el):
        a, b = expert_weights(rank * el + i, H, F)
        wgl[i].copy_(a)
        wdl[i].copy_(b)
    xs, ls = x[rank * tl:(rank + 1) * tl].contiguous(), logits[rank * tl:(rank + 1) * tl].contiguous()
    grp = dist.group.WORLD
    outs = {"nccl": fused_moe(xs, ls, wgl, wdl, k, ep_group=grp)}
    bufs = EPBuffers(grp, tl, H, k, E, torch.bfloat16)
    for i in range(2):  # twice: buffers and epochs carry over between layers
        outs[f"p2p{i}"] = fused_moe(xs, ls, wgl, wdl, k, ep_group=grp, ep_buffers=bufs)
    torch.cuda.synchronize()
    bufs.check()

    gs = torch.Generator().manual_seed(21)
    idx = torch.randperm(T, generator=gs)[:n_sample].sort().values
    mine = (idx >= rank * tl) & (idx < (rank + 1) * tl)
    loc = (idx[mine] - rank * tl).cuda()
    got = {}
    for name, o in outs.items():
        assert o.shape == (tl, H), (name, o.shape)
        buf = torch.zeros(n_sample, H, dtype=torch.float32, device="cuda")
        buf[mine.cuda()] = o[loc].float()
        dist.all_reduce(buf)
        got[name] = buf.cpu()
    bufs.close()
    if rank == 0:
        import grouped_gemm_oracle as oracle
        from gpu_util import MAX_REL, MIN_COS, parity
        ref = oracle.moe_tokens(
            x[idx.cuda()].cpu(), logits[idx.cuda()].cpu(),
            lambda e: tuple(t.cpu() for t in expert_weights(e, H, F)), k,
            round_to=torch.bfloat16)
        for name, o in got.items():
            rel, cos = parity(o, ref)
            assert rel <= MAX_REL and cos >= MIN_COS, f"{name}: max_rel={rel:.3e} cos={cos:.6f}"
            print(f"EP_OK {name} {rel:.3e} {cos:.7f}", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
