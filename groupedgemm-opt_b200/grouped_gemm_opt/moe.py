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
     GEMMs as segments (segment s uses local expert s % (E/P)), no re-sort (NCCL path; the fused
     peer-memory path lays the receive buffer out expert-major, one segment per local expert);
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


class StageEvents:
    """Per-stage device timing of the layer: pass as ``fused_moe(..., timer=StageEvents())``.
    Every stage boundary records a CUDA event on the current stream (no synchronisation), so the
    layer runs exactly as it does without a timer. ``ms()`` (after a synchronize) returns the
    summed milliseconds of every stage over all layers timed with this object."""

    def __init__(self):
        self._marks = []  # [(layer index, stage name, event)]
        self._layer = -1

    def start(self):
        self._layer += 1
        self.mark("start")

    def mark(self, name: str):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self._marks.append((self._layer, name, ev))

    def layers(self) -> int:
        return self._layer + 1

    def ms(self) -> dict:
        tot = {}
        for (l0, _, e0), (l1, name, e1) in zip(self._marks, self._marks[1:]):
            if l0 == l1:
                tot[name] = tot.get(name, 0.0) + e0.elapsed_time(e1)
        return tot


def _mark(timer, name):
    if timer is not None:
        timer.mark(name)


def cuda_ops() -> MoEOps:
    from grouped_gemm_opt._native import _C

    return MoEOps(
        route=lambda logits, k: _C.moe_route(logits, k),
        permute=lambda x, ids, scratch, e: _C.moe_permute(x, ids, scratch, e),
        gate_up=lambda x, w, c, e, s: _C.grouped_gemm_swiglu(x, w, c, e, s),
        down=lambda h, w, c, e, s: _C.grouped_gemm_segments(h, w, c, e, int(TileConfig.AUTO), s),
        combine=lambda y, w, pos: _C.moe_combine(y, w, pos),
    )


class EPBuffers:
    """Receive buffers of the fused expert-parallel path, shared between the ranks of one node
    through CUDA IPC. Create once per (group, sizes) on every rank (a collective call):

        bufs = EPBuffers(group, max_tokens_per_rank, hidden, top_k, num_experts, torch.bfloat16)
        out = fused_moe(x, logits, w_gu_local, w_d_local, top_k, ep_group=group, ep_buffers=bufs)

    Per rank: recv rows [capacity, H] and their origins [capacity] int32, where capacity =
    world * max_tokens * top_k (every routed row of every rank fits even if all go to one rank),
    and the return buffer [max_tokens * top_k, H] that owners scatter results into.
    """

    def __init__(self, group, max_tokens: int, hidden: int, top_k: int, num_experts: int,
                 dtype=torch.bfloat16, device=None):
        from grouped_gemm_opt._native import _C
        self._C = _C
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert self.world <= 8, "the fused path addresses at most 8 ranks (one NVLink domain)"
        assert num_experts % self.world == 0
        self.max_tokens, self.hidden, self.top_k = max_tokens, hidden, top_k
        self.num_experts, self.dtype = num_experts, dtype
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.capacity = self.world * max_tokens * top_k
        esz = torch.empty(0, dtype=dtype).element_size()
        sizes = {"recv": self.capacity * hidden * esz, "origin": self.capacity * 4,
                 "back": max_tokens * top_k * hidden * esz,
                 "board": int(_C.ep_board_bytes(num_experts))}
        self._own = {}
        handles = {}
        for name, nbytes in sizes.items():
            ptr, h = _C.ipc_alloc(max(nbytes, 256))
            self._own[name] = ptr
            handles[name] = h
        # the sync board must start at zero (counts and epoch flags) before any peer writes to it
        dev = self.device.index
        self._board_elems = int(_C.ep_board_bytes(num_experts)) // 8
        _C.tensor_view(self._own["board"], [self._board_elems], torch.int64, dev).zero_()
        torch.cuda.synchronize(self.device)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, handles, group=group)
        self.ptrs = {name: [] for name in sizes}
        self._opened = []
        for r in range(self.world):
            for name in sizes:
                if r == self.rank:
                    self.ptrs[name].append(self._own[name])
                else:
                    ptr = _C.ipc_open(gathered[r][name])
                    self._opened.append(ptr)
                    self.ptrs[name].append(ptr)
        dev = self.device.index
        self.recv = _C.tensor_view(self._own["recv"], [self.capacity, hidden], dtype, dev)
        self.origin = _C.tensor_view(self._own["origin"], [self.capacity], torch.int32, dev)
        self.back = _C.tensor_view(self._own["back"], [max_tokens * top_k, hidden], dtype, dev)
        self.flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        # own board: counts rows of every rank (first `world` of 8), then the epoch flags
        self.board_counts = _C.tensor_view(self._own["board"], [8, num_experts], torch.int64, dev)
        self.epoch = 0
        self.wait_limit_cycles = 1 << 34  # ~10 s at 1.9 GHz, then the wait records a timeout
        dist.barrier(group=group)

    def fence(self):
        """Stream-ordered cross-rank barrier: a one-element all-reduce. Every rank's earlier
        kernels (and their peer stores) are complete when it returns on any rank's stream."""
        dist.all_reduce(self.flag, group=self.group)

    def check(self):
        """Synchronises and raises RuntimeError if a peer wait of a layer on this stream expired
        (a rank fell behind or left). Layers after such a failure return NaN rows rather than
        stale data, so a caller that skips this check still cannot mistake them for results."""
        from grouped_gemm_opt.ops import check_device_errors
        check_device_errors(self.device.index)

    def close(self):
        if self._C is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            self._C.ipc_close(p)
        dist.barrier(group=self.group)
        for p in self._own.values():
            self._C.ipc_free(p)
        self._C = None


def _fused_moe_p2p(hidden, router_logits, w_gate_up, w_down, top_k, bufs: "EPBuffers",
                   sort_by_m, timer=None):
    """Expert-parallel layer over NVLink peer memory: the dispatch kernel writes rows into the
    owners' receive buffers, the down GEMM's epilogue writes results back into the sources'
    return buffers. The phases are ordered by device-side epoch flags in the IPC-shared sync
    boards (post with system-scope stores, bounded waits): no host synchronisation and no
    NCCL call in the layer."""
    C = bufs._C
    world, rank = bufs.world, bufs.rank
    T, H = hidden.shape
    E = router_logits.size(1)
    el = E // world
    assert T <= bufs.max_tokens and H == bufs.hidden and top_k == bufs.top_k, "EPBuffers too small"
    assert E == bufs.num_experts and hidden.dtype == bufs.dtype
    bufs.epoch += 1
    ep, dev, boards, own = bufs.epoch, hidden.device.index, bufs.ptrs["board"], bufs._own["board"]
    lim = bufs.wait_limit_cycles
    ids, w, tpe, scratch = C.moe_route(router_logits, top_k)
    _mark(timer, "route")
    # phase 0: every rank's counts land in every board
    C.ep_publish_counts(tpe, boards, rank, 0, ep)
    C.ep_wait(own, world, E, 0, ep, lim, dev)
    _mark(timer, "count_exchange")
    counts_all = bufs.board_counts[:world]
    slot_pos = C.ep_dispatch(hidden, ids, scratch, counts_all, rank, bufs.ptrs["recv"],
                             bufs.ptrs["origin"])
    _mark(timer, "dispatch")
    # phase 1: every source has delivered its rows to this rank
    C.ep_signal(boards, rank, E, 1, ep, dev)
    C.ep_wait(own, world, E, 1, ep, lim, dev)
    _mark(timer, "dispatch_wait")
    # receive buffer is expert-major: one segment per local expert, rows from every source
    seg_counts = counts_all[:, rank * el:(rank + 1) * el].sum(0)
    h = C.ep_grouped_gemm(bufs.recv, w_gate_up, seg_counts, el, True, None, [], sort_by_m)
    _mark(timer, "gate_up")
    C.ep_grouped_gemm(h, w_down, seg_counts, el, False, bufs.origin, bufs.ptrs["back"],
                      sort_by_m)
    _mark(timer, "down")
    # phase 2: every owner has scattered this rank's results back
    C.ep_signal(boards, rank, E, 2, ep, dev)
    C.ep_wait(own, world, E, 2, ep, lim, dev)
    _mark(timer, "return_wait")
    # checked combine: if any wait above expired, the result is NaN instead of stale rows
    out = C.moe_combine(bufs.back[:T * top_k], w, slot_pos, True)
    _mark(timer, "combine")
    return out


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
    ep_buffers: Optional[EPBuffers] = None,
    timer: Optional[StageEvents] = None,
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
        ep_buffers: EPBuffers of `ep_group`: selects the fused peer-memory path (dispatch and
            result scatter over NVLink inside the kernels) instead of NCCL all-to-alls.
        timer: a StageEvents that records a CUDA event after every stage (device timing).

    Returns: [T, H] = sum_j w[t,j] * down(silu(gate(x_t)) * up(x_t)) for the top-k experts.
    """
    world = dist.get_world_size(ep_group) if ep_group is not None else 1
    T, H, E, el = _check(hidden, router_logits, w_gate_up, w_down, top_k, world)
    if timer is not None:
        timer.start()
    if ep_buffers is not None and world > 1 and ops is None:
        return _fused_moe_p2p(hidden.contiguous(), router_logits, w_gate_up, w_down, top_k,
                              ep_buffers, sort_by_m, timer)
    if ops is None:
        ops = cuda_ops()
    hidden = hidden.contiguous()
    ids, w, tpe, scratch = ops.route(router_logits, top_k)
    _mark(timer, "route")
    xs, _sorted_token, slot_pos = ops.permute(hidden, ids, scratch, E)
    _mark(timer, "dispatch")
    if world == 1:
        h = ops.gate_up(xs, w_gate_up, tpe, E, sort_by_m)
        _mark(timer, "gate_up")
        y = ops.down(h, w_down, tpe, E, sort_by_m)
        _mark(timer, "down")
        out = ops.combine(y, w, slot_pos)
        _mark(timer, "combine")
        return out

    send_counts = tpe.view(world, el)
    recv_counts = torch.empty_like(tpe)
    dist.all_to_all_single(recv_counts, tpe, group=ep_group)
    # one host read of both split vectors
    splits = torch.stack([send_counts.sum(1), recv_counts.view(world, el).sum(1)]).cpu()
    _mark(timer, "count_exchange")
    send_splits = splits[0].tolist()
    recv_splits = splits[1].tolist()
    x_recv = xs.new_empty((int(sum(recv_splits)), H))
    dist.all_to_all_single(x_recv, xs, recv_splits, send_splits, group=ep_group)
    _mark(timer, "dispatch_all_to_all")
    h = ops.gate_up(x_recv, w_gate_up, recv_counts, el, sort_by_m)
    _mark(timer, "gate_up")
    y = ops.down(h, w_down, recv_counts, el, sort_by_m)
    _mark(timer, "down")
    y_back = y.new_empty((xs.size(0), H))
    dist.all_to_all_single(y_back, y, send_splits, recv_splits, group=ep_group)
    _mark(timer, "return_all_to_all")
    out = ops.combine(y_back, w, slot_pos)
    _mark(timer, "combine")
    return out


def fused_moe_host(
    hidden: torch.Tensor,
    router_logits: torch.Tensor,
    w_gate_up: torch.Tensor,
    w_down: torch.Tensor,
    top_k: int,
    out: Optional[torch.Tensor] = None,
    chunks: int = 4,
    ep_group: Optional[dist.ProcessGroup] = None,
    ep_buffers: Optional[EPBuffers] = None,
    sort_by_m: bool = True,
) -> torch.Tensor:
    """:func:`fused_moe` on HOST-resident tokens: ``hidden`` [T, H] and ``router_logits`` [T, E]
    in (pinned) host memory, weights on the GPU, result into ``out`` [T, H] in host memory
    (allocated pinned if not given).

    The tokens are split into ``chunks`` consecutive groups. Group i+1 is copied in on a copy
    stream while the layer runs on group i on the current stream, and group i-1's result is
    copied out on a third stream, so PCIe traffic hides behind the layer. Every rank of an
    expert-parallel group must call this with the same ``chunks`` (each chunk is one layer
    call, a collective over the group). Returns ``out`` once the work is enqueued; it is
    complete when the current stream is synchronised (all streams are joined back to it)."""
    assert not hidden.is_cuda and not router_logits.is_cuda, "tokens must be in host memory"
    assert w_gate_up.is_cuda and w_down.is_cuda
    T, H = hidden.shape
    dev = w_gate_up.device
    if out is None:
        out = torch.empty(T, H, dtype=hidden.dtype, pin_memory=True)
    chunks = max(1, min(chunks, T)) if T > 0 else 1
    bounds = [T * i // chunks for i in range(chunks + 1)]
    main = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    s_in.wait_stream(main)
    s_out.wait_stream(main)
    xs, ls, copied = [], [], []
    with torch.cuda.stream(s_in):
        for i in range(chunks):
            a, b = bounds[i], bounds[i + 1]
            xs.append(hidden[a:b].to(dev, non_blocking=True))
            ls.append(router_logits[a:b].to(dev, non_blocking=True))
            ev = torch.cuda.Event()
            ev.record(s_in)
            copied.append(ev)
    for i in range(chunks):
        a, b = bounds[i], bounds[i + 1]
        main.wait_event(copied[i])
        y = fused_moe(xs[i], ls[i], w_gate_up, w_down, top_k, ep_group=ep_group,
                      sort_by_m=sort_by_m, ep_buffers=ep_buffers)
        done = torch.cuda.Event()
        done.record(main)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            out[a:b].copy_(y, non_blocking=True)
            y.record_stream(s_out)
        xs[i].record_stream(main)
        ls[i].record_stream(main)
    main.wait_stream(s_out)
    main.wait_stream(s_in)
    return out


class MoEHostPipeline:
    """Streams batches of HOST-resident tokens through :func:`fused_moe`, batch after batch, the
    way a server feeds a layer: each :meth:`submit` copies its batch's tokens and logits in on a
    copy stream, runs the layer on the current stream once they have landed, and copies the
    result out to host memory on a second copy stream. Nothing joins the copy streams back to
    the current stream, so batch i+1's copy in and batch i's copy out run while the layer
    computes: in steady state the PCIe traffic of a batch costs no layer time. Each batch is one
    whole layer call (no token chunking, which would cost GEMM efficiency).

    Results are complete after :meth:`synchronize` (or a device-wide synchronize). Host buffers
    passed to :meth:`submit` must stay untouched until then. Every rank of an expert-parallel
    group submits the same number of batches in the same order (each is a collective)."""

    def __init__(self, w_gate_up: torch.Tensor, w_down: torch.Tensor, top_k: int,
                 ep_group: Optional[dist.ProcessGroup] = None,
                 ep_buffers: Optional[EPBuffers] = None, sort_by_m: bool = True):
        assert w_gate_up.is_cuda and w_down.is_cuda
        self.w_gate_up, self.w_down, self.top_k = w_gate_up, w_down, top_k
        self.ep_group, self.ep_buffers, self.sort_by_m = ep_group, ep_buffers, sort_by_m
        self.device = w_gate_up.device
        self.s_in = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)

    def submit(self, hidden: torch.Tensor, router_logits: torch.Tensor,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Enqueue one batch: ``hidden`` [T, H] and ``router_logits`` [T, E] in (pinned) host
        memory; the result goes to ``out`` [T, H] in host memory (allocated pinned if None),
        which is returned at once and is valid after :meth:`synchronize`."""
        assert not hidden.is_cuda and not router_logits.is_cuda, "tokens must be in host memory"
        if out is None:
            out = torch.empty(hidden.shape, dtype=hidden.dtype, pin_memory=True)
        main = torch.cuda.current_stream(self.device)
        with torch.cuda.stream(self.s_in):
            x = hidden.to(self.device, non_blocking=True)
            lg = router_logits.to(self.device, non_blocking=True)
            landed = torch.cuda.Event()
            landed.record(self.s_in)
        main.wait_event(landed)
        y = fused_moe(x, lg, self.w_gate_up, self.w_down, self.top_k, ep_group=self.ep_group,
                      sort_by_m=self.sort_by_m, ep_buffers=self.ep_buffers)
        x.record_stream(main)
        lg.record_stream(main)
        done = torch.cuda.Event()
        done.record(main)
        self.s_out.wait_event(done)
        with torch.cuda.stream(self.s_out):
            out.copy_(y, non_blocking=True)
            y.record_stream(self.s_out)
        return out

    def synchronize(self) -> None:
        """Wait until every submitted batch's result is in host memory; afterwards the current
        stream is ordered after all of the pipeline's work."""
        main = torch.cuda.current_stream(self.device)
        main.wait_stream(self.s_in)
        main.wait_stream(self.s_out)
        self.s_out.synchronize()


@dataclass
class MoEFP8Weights:
    """e4m3 expert weights with one fp32 scale per output channel (see quantize_moe_weights)."""
    w_gate_up_q: torch.Tensor      # [E, 2F, H] float8_e4m3fn
    w_gate_up_scale: torch.Tensor  # [E, 2F] fp32
    w_down_q: torch.Tensor         # [E, H, F] float8_e4m3fn
    w_down_scale: torch.Tensor     # [E, H] fp32


def quantize_moe_weights(w_gate_up: torch.Tensor, w_down: torch.Tensor) -> MoEFP8Weights:
    """Per-output-channel e4m3 quantisation of the layer's weights (done once, on the GPU)."""
    from grouped_gemm_opt.ops import quantize_fp8
    gq, gs = quantize_fp8(w_gate_up)
    dq, ds = quantize_fp8(w_down)
    return MoEFP8Weights(gq, gs, dq, ds)


def fused_moe_fp8(hidden: torch.Tensor, router_logits: torch.Tensor, weights: MoEFP8Weights,
                  top_k: int, sort_by_m: bool = True,
                  timer: Optional[StageEvents] = None) -> torch.Tensor:
    """Single-GPU MoE layer with FP8 (e4m3) grouped GEMMs: route -> dispatch -> per-row
    quantisation of the gathered rows -> gate/up GEMM with a scaled SwiGLU epilogue (bf16 h) ->
    per-row quantisation of h -> down GEMM with a scaled epilogue -> combine. Routing, dispatch
    and combine are the bf16 layer's; the result is bf16."""
    from grouped_gemm_opt._native import _C
    E = router_logits.size(1)
    assert weights.w_gate_up_q.size(0) == E, "all experts must be local"
    if timer is not None:
        timer.start()
    ids, w, tpe, scratch = _C.moe_route(router_logits, top_k)
    _mark(timer, "route")
    xs, _, slot_pos = _C.moe_permute(hidden.contiguous(), ids, scratch, E)
    _mark(timer, "dispatch")
    xq, xsc = _C.quantize_fp8_rows(xs)
    _mark(timer, "quantize_x")
    h = _C.grouped_gemm_swiglu_fp8(xq, xsc, weights.w_gate_up_q, weights.w_gate_up_scale, tpe, E,
                                   sort_by_m)
    _mark(timer, "gate_up")
    hq, hsc = _C.quantize_fp8_rows(h)
    _mark(timer, "quantize_h")
    y = _C.grouped_gemm_fp8(hq, hsc, weights.w_down_q, weights.w_down_scale, tpe, 4, sort_by_m)
    _mark(timer, "down")
    out = _C.moe_combine(y, w, slot_pos)
    _mark(timer, "combine")
    return out


@dataclass
class MoEMXFP8Weights:
    """MXFP8 expert weights (see quantize_moe_weights_mxfp8): e4m3 with UE8M0 block scales."""
    w_gate_up_q: torch.Tensor      # [E, 2 F_pad, H] float8_e4m3fn, blocked gate/up rows
    w_gate_up_scale: torch.Tensor  # uint8, 128x4 blocked scale layout
    w_down_q: torch.Tensor         # [E, H, F] float8_e4m3fn
    w_down_scale: torch.Tensor     # uint8
    F: int


def quantize_moe_weights_mxfp8(w_gate_up: torch.Tensor, w_down: torch.Tensor) -> MoEMXFP8Weights:
    """MX quantisation of the layer's weights (once, on the GPU); the gate/up weight is first
    reordered into the blocked layout of the MXFP8 SwiGLU GEMM."""
    from grouped_gemm_opt.ops import mxfp8_block_gate_up, quantize_mxfp8
    gq, gs = quantize_mxfp8(mxfp8_block_gate_up(w_gate_up))
    dq, ds = quantize_mxfp8(w_down)
    return MoEMXFP8Weights(gq, gs, dq, ds, w_gate_up.size(1) // 2)


def fused_moe_mxfp8(hidden: torch.Tensor, router_logits: torch.Tensor, weights: MoEMXFP8Weights,
                    top_k: int, sort_by_m: bool = True,
                    timer: Optional[StageEvents] = None) -> torch.Tensor:
    """Single-GPU MoE layer with MXFP8 grouped GEMMs: route -> dispatch -> MX quantisation of the
    gathered rows -> gate/up GEMM with the SwiGLU epilogue (bf16 h) -> MX quantisation of h ->
    down GEMM -> combine. Routing, dispatch and combine are the bf16 layer's."""
    from grouped_gemm_opt._native import _C
    E = router_logits.size(1)
    assert weights.w_gate_up_q.size(0) == E, "all experts must be local"
    if timer is not None:
        timer.start()
    ids, w, tpe, scratch = _C.moe_route(router_logits, top_k)
    _mark(timer, "route")
    xs, _, slot_pos = _C.moe_permute(hidden.contiguous(), ids, scratch, E)
    _mark(timer, "dispatch")
    xq, xsc = _C.quantize_mxfp8(xs, tpe)
    _mark(timer, "quantize_x")
    h = _C.grouped_gemm_swiglu_mxfp8(xq, xsc, weights.w_gate_up_q, weights.w_gate_up_scale, tpe,
                                     E, weights.F, sort_by_m)
    _mark(timer, "gate_up")
    hq, hsc = _C.quantize_mxfp8(h, tpe)
    _mark(timer, "quantize_h")
    y = _C.grouped_gemm_mxfp8(hq, hsc, weights.w_down_q, weights.w_down_scale, tpe, E, sort_by_m)
    _mark(timer, "down")
    out = _C.moe_combine(y, w, slot_pos)
    _mark(timer, "combine")
    return out

