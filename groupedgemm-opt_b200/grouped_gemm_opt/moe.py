"""Fused MoE layer: router -> permute -> gate/up GEMM with SwiGLU -> down GEMM -> combine,
single-GPU or expert-parallel over a torch.distributed group.

The reference's fused-MoE entry point (grouped_gemm_opt/triton_fused_moe.py:104-150) is only the
grouped GEMM over pre-sorted rows; this module is the complete layer that its name promises.

Conventions (fixed here, relied on by the kernels and the tests):
  * router: top-k of the fp32 logits, ties to the lower expert index, softmax over the k selected
    logits (Mixtral style), weights kept in fp32.
  * sorted order: expert-major, then token index (a stable counting sort).
  * w_gate_up [E, 2F, H]: rows 0..F-1 are the gate projection, rows F..2F-1 the up projection.
  * w_down [E, H, F].
  * combine: fp32 sum over the k slots in slot order, rounded once to the activation dtype.

Expert parallelism (``ep_group`` of P ranks): each rank holds E/P consecutive experts
(rank r owns [r*E/P, (r+1)*E/P)) and its own tokens. After the local route + permute, rows bound
for rank r are one contiguous run (experts are sorted globally). Per layer:
  1. all_to_all of the per-(destination, local expert) counts (int64, P*E/P entries);
  2. one device->host read of the split sizes (the only host sync of the layer);
  3. all_to_all_single of the rows;
  4. the received rows are [source rank][local expert] segments -- fed directly to the grouped
     GEMMs as segments (segment s uses local expert s % (E/P)), no re-sort;
  5. reverse all_to_all_single of the down-projection rows, back into the sender's sorted order;
  6. local combine.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

from grouped_gemm_opt.ops import TileConfig


@dataclass
class MoEOps:
    """The five compute stages of the layer. The product uses :func:`cuda_ops`; host-logic tests
    substitute CPU implementations to exercise the expert-parallel orchestration on gloo ranks."""
    route: Callable      # (logits, top_k) -> (ids int32 [T,k], w fp32 [T,k], tpe int64 [E], scratch)
    permute: Callable    # (x, ids, scratch, E) -> (x_sorted [T*k,H], sorted_token, slot_pos)
    gate_up: Callable    # (x_rows, w_gu, seg_counts, n_experts, sort_by_m) -> h [rows, F]
    down: Callable       # (h, w_d, seg_counts, n_experts, sort_by_m) -> y [rows, H]
    combine: Callable    # (y_sorted, w, slot_pos) -> out [T, H]


def cuda_ops() -> MoEOps:
    from grouped_gemm_opt._native import _C

    return MoEOps(
        route=lambda logits, k: _C.moe_route(logits, k),
        permute=lambda x, ids, scratch, e: _C.moe_permute(x, ids, scratch, e),
        gate_up=lambda x, w, c, e, s: _C.grouped_gemm_swiglu(x, w, c, e, s),
        down=lambda h, w, c, e, s: _C.grouped_gemm_segments(h, w, c, e, int(TileConfig.AUTO), s),
        combine=lambda y, w, pos: _C.moe_combine(y, w, pos),
    )


def _check(hidden, router_logits, w_gate_up, w_down, top_k, world):
    assert hidden.dim() == 2 and router_logits.dim() == 2
    assert w_gate_up.dim() == 3 and w_down.dim() == 3
    T, H = hidden.shape
    E = router_logits.size(1)
    assert router_logits.size(0) == T, "router_logits must have one row per token"
    assert E % world == 0, f"num_experts={E} not divisible by the expert-parallel size {world}"
    el = E // world
    assert w_gate_up.size(0) == el and w_down.size(0) == el, (
        f"each rank must hold {el} experts, got w_gate_up {w_gate_up.size(0)}, "
        f"w_down {w_down.size(0)}")
    assert w_gate_up.size(2) == H and w_down.size(1) == H, "hidden size mismatch"
    assert w_gate_up.size(1) == 2 * w_down.size(2), "w_gate_up must have 2F rows, w_down F columns"
    assert 0 < top_k <= E
    return T, H, E, el


def fused_moe(
    hidden: torch.Tensor,
    router_logits: torch.Tensor,
    w_gate_up: torch.Tensor,
    w_down: torch.Tensor,
    top_k: int,
    ep_group: Optional[dist.ProcessGroup] = None,
    sort_by_m: bool = True,
    ops: Optional[MoEOps] = None,
) -> torch.Tensor:
    """MoE layer forward.

    Args:
        hidden: [T, H] bf16/fp16 tokens of this rank.
        router_logits: [T, E] router scores over ALL experts (any float dtype; routed in fp32).
        w_gate_up: [E_local, 2F, H] gate rows then up rows, for the experts this rank owns.
        w_down: [E_local, H, F].
        top_k: experts per token.
        ep_group: expert-parallel process group (None: single GPU, E_local = E).
        sort_by_m: heaviest-expert-first tile order inside the grouped GEMMs.
        ops: compute stages (defaults to the CUDA kernels).

    Returns: [T, H] = sum_j w[t,j] * down(silu(gate(x_t)) * up(x_t)) for the top-k experts.
    """
    world = dist.get_world_size(ep_group) if ep_group is not None else 1
    T, H, E, el = _check(hidden, router_logits, w_gate_up, w_down, top_k, world)
    if ops is None:
        ops = cuda_ops()
    hidden = hidden.contiguous()
    ids, w, tpe, scratch = ops.route(router_logits, top_k)
    xs, _sorted_token, slot_pos = ops.permute(hidden, ids, scratch, E)
    if world == 1:
        h = ops.gate_up(xs, w_gate_up, tpe, E, sort_by_m)
        y = ops.down(h, w_down, tpe, E, sort_by_m)
        return ops.combine(y, w, slot_pos)

    send_counts = tpe.view(world, el)
    recv_counts = torch.empty_like(tpe)
    dist.all_to_all_single(recv_counts, tpe, group=ep_group)
    # one host read of both split vectors
    splits = torch.stack([send_counts.sum(1), recv_counts.view(world, el).sum(1)]).cpu()
    send_splits = splits[0].tolist()
    recv_splits = splits[1].tolist()
    x_recv = xs.new_empty((int(sum(recv_splits)), H))
    dist.all_to_all_single(x_recv, xs, recv_splits, send_splits, group=ep_group)
    h = ops.gate_up(x_recv, w_gate_up, recv_counts, el, sort_by_m)
    y = ops.down(h, w_down, recv_counts, el, sort_by_m)
    y_back = y.new_empty((xs.size(0), H))
    dist.all_to_all_single(y_back, y, send_splits, recv_splits, group=ep_group)
    return ops.combine(y_back, w, slot_pos)
