"""Worker for tests/test_ep_gpu.py, launched by torchrun with one rank per GPU (NCCL).

Every rank builds the same global problem from seeds, runs the expert-parallel fused_moe on its
token slice with its slice of experts, and compares with the single-GPU fused_moe of the same
tokens (all experts local). Prints one line per rank: "EP_OK rank max_rel" or raises.
"""
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "groupedgemm-opt_b200"))


def main():
    T, H, F, E, k = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4]), \
        int(sys.argv[5])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from grouped_gemm_opt import EPBuffers, fused_moe
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, device="cuda", generator=g)
    wgu = (torch.randn(E, 2 * F, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(E, H, F, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    tl, el = T // world, E // world
    xs, ls = x[rank * tl:(rank + 1) * tl], logits[rank * tl:(rank + 1) * tl]
    out = fused_moe(xs, ls, wgu[rank * el:(rank + 1) * el].contiguous(),
                    wd[rank * el:(rank + 1) * el].contiguous(), k, ep_group=dist.group.WORLD)
    ref = fused_moe(xs, ls, wgu, wd, k)
    bufs = EPBuffers(dist.group.WORLD, tl, H, k, E, torch.bfloat16)
    wgl = wgu[rank * el:(rank + 1) * el].contiguous()
    wdl = wd[rank * el:(rank + 1) * el].contiguous()
    outs_p2p = [fused_moe(xs, ls, wgl, wdl, k, ep_group=dist.group.WORLD, ep_buffers=bufs)
                for _ in range(2)]  # twice: buffers are reused across layers
    torch.cuda.synchronize()
    rels = []
    for o in [out] + outs_p2p:
        d = (o.float() - ref.float()).abs().max().item()
        rels.append(d / max(ref.float().abs().max().item(), 1e-12))
        assert o.shape == ref.shape and rels[-1] <= 1e-2, rels
    bufs.close()
    print(f"EP_OK {rank} " + " ".join(f"{r:.3e}" for r in rels), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
