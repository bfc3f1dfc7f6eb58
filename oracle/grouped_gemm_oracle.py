"""CPU oracle for the grouped-GEMM / fused-MoE hot path. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may import this module, and
only as the checker (or as the timed CPU baseline). The product path never calls it.

What it restates, with the reference file:line each function follows (paths inside
jeshxxx/GroupedGEMM-OPT):

  sequential_gemm          benchmarks/benchmark.py:91-107  -- the reference's ground truth: a
                           per-expert ``F.linear`` loop over expert-sorted row segments.
  uniform_distribution     benchmarks/benchmark.py:50-56
  skewed_distribution      benchmarks/benchmark.py:59-69
  zipf_counts / dirichlet_counts   the seeded tpe generators of the BASELINE configs (cfg3), which
                           the reference does not ship (its random_distribution,
                           benchmark.py:72-79, is unseeded).
  route / permute / combine / moe_layer / moe_tokens   the fused-MoE layer. The reference has no router,
                           permute or combine (its triton_fused_moe.py:81-101 gathers through an
                           identity map), so these restate the conventions documented in
                           grouped_gemm_opt/moe.py. Parity of these stages is UNPINNED (no
                           reference implementation exists to pin against).

  mx_quantize / mx_dequantize / mx_block_gate_up   MXFP8 (block-scaled e4m3). The reference is
                           bf16/fp16 only, so these restate the OCP Microscaling (MX) v1.0 format
                           (32-element blocks, UE8M0 scales) and the 128x4 blocked scale layout
                           of block-scaled tcgen05 MMAs, with the scale-exponent rule the library
                           documents in include/ggo.h. UNPINNED to the reference (it has no
                           counterpart); checked by known-answer vectors in tests/test_oracle.py.

Pinning: ``sequential_gemm`` and the two distribution generators are checked against golden
vectors produced by the reference's own benchmark.py (tests/golden/make_golden.py imports it and
commits small fixtures); see tests/test_oracle.py.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


# ----------------------------------------------------------------------------- grouped GEMM
def sequential_gemm(input: torch.Tensor, weights: torch.Tensor,
                    tokens_per_expert: torch.Tensor, out_dtype=None,
                    native: bool = False) -> torch.Tensor:
    """Per-expert loop (benchmark.py:91-107). Computes in fp32 from the given (bf16) values.

    Returns fp32 unless ``out_dtype`` is given (the reference returns the input dtype, i.e. a
    bf16 rounding of the same products: pass out_dtype=input.dtype for that).
    ``native=True`` runs ``F.linear`` in the operands' own dtype exactly as the reference does
    (used to time the reference algorithm as the CPU baseline)."""
    x = input if native else input.float()
    w = weights if native else weights.float()
    outs = []
    off = 0
    for g in range(w.size(0)):
        m = int(tokens_per_expert[g])
        if m > 0:
            outs.append(F.linear(x[off:off + m], w[g]))
        off += m
    out = torch.cat(outs, 0) if outs else torch.empty(0, w.size(1))
    return out if out_dtype is None else out.to(out_dtype)


def segments_gemm(input: torch.Tensor, weights: torch.Tensor, seg_counts: torch.Tensor,
                  num_experts: int, native: bool = False) -> torch.Tensor:
    """Segment form: segment s multiplies by expert s % num_experts (fp32 result). ``native``:
    F.linear in the operands' own dtype, as the reference's loop runs it (result in that dtype)."""
    x = input if native else input.float()
    w = weights if native else weights.float()
    out = torch.zeros(x.size(0), w.size(1), dtype=x.dtype)
    off = 0
    for s, m in enumerate(seg_counts.tolist()):
        if m > 0:
            out[off:off + m] = F.linear(x[off:off + m], w[s % num_experts])
        off += m
    return out


def swiglu_gemm(x: torch.Tensor, w_gate_up: torch.Tensor, seg_counts: torch.Tensor,
                num_experts: int, native: bool = False) -> torch.Tensor:
    """h = silu(x W_gate^T) * (x W_up^T) per segment; W_gu rows [0,F) gate, [F,2F) up. fp32
    (``native``: the GEMM in the operands' dtype, the activation in fp32, h in that dtype)."""
    f = w_gate_up.size(1) // 2
    gu = segments_gemm(x, w_gate_up, seg_counts, num_experts, native).float()
    h = F.silu(gu[:, :f]) * gu[:, f:]
    return h.to(x.dtype) if native else h


# ----------------------------------------------------------------------------- distributions
def uniform_distribution(total_tokens: int, num_experts: int) -> torch.Tensor:
    """benchmark.py:50-56: equal split, the remainder to the first experts."""
    base, rem = divmod(total_tokens, num_experts)
    tpe = torch.full((num_experts,), base, dtype=torch.int64)
    tpe[:rem] += 1
    return tpe


def skewed_distribution(total_tokens: int, num_experts: int, skew_factor: float = 3.0):
    """benchmark.py:59-69: power-law shares i^-skew, floored, rounding error to expert 0."""
    w = torch.pow(torch.arange(1, num_experts + 1, dtype=torch.float64), -skew_factor)
    w /= w.sum()
    tpe = (w * total_tokens).long()
    tpe[0] += total_tokens - int(tpe.sum())
    return tpe


def zipf_counts(total_tokens: int, num_experts: int, alpha: float = 1.2, seed: int = 0):
    """cfg3 routing: multinomial(total, p_i ~ 1/(i+1)^alpha), seeded."""
    g = torch.Generator().manual_seed(seed)
    p = 1.0 / torch.arange(1, num_experts + 1, dtype=torch.float64) ** alpha
    p /= p.sum()
    draws = torch.multinomial(p, total_tokens, replacement=True, generator=g)
    return torch.bincount(draws, minlength=num_experts).to(torch.int64)


def dirichlet_counts(total_tokens: int, num_experts: int, alpha: float = 0.5, seed: int = 0):
    """cfg3 'random' variant: Dirichlet(alpha) proportions, then a multinomial draw (numpy)."""
    rng = np.random.default_rng(seed)
    p = rng.dirichlet(np.full(num_experts, alpha))
    return torch.from_numpy(rng.multinomial(total_tokens, p).astype(np.int64))


# ----------------------------------------------------------------------------- fused MoE
def route(logits: np.ndarray, top_k: int):
    """Top-k (ties -> lower index) then softmax over the selected logits, fp32.
    Returns ids int32 [T,k], weights fp32 [T,k], tokens_per_expert int64 [E]."""
    lg = np.asarray(logits, dtype=np.float32)
    T, E = lg.shape
    order = np.argsort(-lg, axis=1, kind="stable")[:, :top_k]
    vals = np.take_along_axis(lg, order, axis=1)
    ex = np.exp(vals - vals[:, :1])
    w = (ex / ex.sum(axis=1, keepdims=True)).astype(np.float32)
    tpe = np.bincount(order.reshape(-1), minlength=E).astype(np.int64)
    return order.astype(np.int32), w, tpe


def permute_indices(ids: np.ndarray, num_experts: int):
    """Stable counting sort of the (token, slot) entries by expert.
    Returns sorted_token int32 [T*k] and slot_pos int32 [T*k] (index t*k+j -> sorted row)."""
    flat = ids.reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable")  # expert-major, then (t, j) order
    k = ids.shape[1]
    sorted_token = (order // k).astype(np.int32)
    slot_pos = np.empty_like(order)
    slot_pos[order] = np.arange(order.size)
    return sorted_token, slot_pos.astype(np.int32)


def combine(y_sorted: torch.Tensor, w: np.ndarray, slot_pos: np.ndarray) -> torch.Tensor:
    """out[t] = sum_j w[t,j] * y_sorted[slot_pos[t*k+j]] in fp32, slot order."""
    T, k = w.shape
    y = y_sorted.float()
    wt = torch.from_numpy(np.asarray(w, dtype=np.float32))
    pos = torch.from_numpy(np.asarray(slot_pos, dtype=np.int64)).view(T, k)
    out = torch.zeros(T, y.size(1))
    for j in range(k):
        out += wt[:, j:j + 1] * y[pos[:, j]]
    return out


def moe_layer(hidden: torch.Tensor, logits: torch.Tensor, w_gate_up: torch.Tensor,
              w_down: torch.Tensor, top_k: int, round_to=None, native: bool = False) -> torch.Tensor:
    """Whole layer in fp32. With ``round_to`` (e.g. torch.bfloat16) the intermediate activations
    (gathered rows, h, y) are rounded to that dtype as the GPU pipeline stores them. ``native``
    runs the two grouped GEMMs as the reference's per-expert F.linear loop in the weights' own
    dtype (benchmark.py:91-107), the form timed as the CPU baseline of the layer."""
    ids, w, tpe = route(logits.float().numpy(), top_k)
    E = logits.size(1)
    sorted_token, slot_pos = permute_indices(ids, E)
    xs = hidden[torch.from_numpy(sorted_token.astype(np.int64))]
    counts = torch.from_numpy(tpe)
    h = swiglu_gemm(xs, w_gate_up, counts, E, native)
    if round_to is not None:
        h = h.to(round_to)
    y = segments_gemm(h, w_down, counts, E, native)
    if round_to is not None:
        y = y.to(round_to)
    return combine(y, w, slot_pos)


def moe_tokens(hidden: torch.Tensor, logits: torch.Tensor, expert_weights, top_k: int,
               round_to=None) -> torch.Tensor:
    """moe_layer for a SAMPLE of tokens whose experts' weights are fetched one at a time:
    ``expert_weights(e)`` returns (w_gate_up[e] [2F, H], w_down[e] [H, F]) on the CPU. Tokens
    are independent in the layer (routing, the GEMM rows and the combine are all per token), so
    the rows for a sample equal the same rows of the whole layer. fp32, rounding as moe_layer."""
    ids, w, _ = route(logits.float().numpy(), top_k)
    T, k = ids.shape
    x = hidden.float()
    ys = {}
    for e in np.unique(ids):
        wgu, wd = expert_weights(int(e))
        f = wgu.size(0) // 2
        rows = np.argwhere(ids == e)  # (t, j) pairs in token order
        xe = x[torch.from_numpy(rows[:, 0].astype(np.int64))]
        gu = F.linear(xe, wgu.float())
        h = F.silu(gu[:, :f]) * gu[:, f:]
        if round_to is not None:
            h = h.to(round_to).float()
        y = F.linear(h, wd.float())
        if round_to is not None:
            y = y.to(round_to).float()
        for i, (t, j) in enumerate(rows):
            ys[(int(t), int(j))] = y[i]
    out = torch.zeros(T, x.size(1))
    wt = torch.from_numpy(np.asarray(w, dtype=np.float32))
    for t in range(T):
        for j in range(k):
            out[t] += wt[t, j] * ys[(t, j)]
    return out


# ----------------------------------------------------------------------------- MXFP8
def mx_scale_exponent(amax: np.ndarray) -> np.ndarray:
    """Shared exponent X of 32-element groups from their fp32 amax: floor(log2 amax) - 8, plus 1
    when amax / 2^floor(log2 amax) > 1.75 (so amax / 2^X <= 448 = max e4m3), clamped to
    [-127, 127]; -127 for amax == 0 (and for fp32 subnormals). Pure bit arithmetic."""
    bits = np.asarray(amax, dtype=np.float32).view(np.uint32).astype(np.int64)
    eb = (bits >> 23) & 0xFF
    mant = bits & 0x7FFFFF
    x = np.where(eb == 0, -127, eb - 127 - 8 + (mant > 0x600000).astype(np.int64))
    return np.clip(x, -127, 127)


def mx_atom_offset(block: np.ndarray, r: np.ndarray, group: np.ndarray, k: int) -> np.ndarray:
    """Byte offset of the scale of row r (0..127) of 128-row block `block`, 32-element group
    `group` in the 128x4 blocked layout: atom (block * K/128 + group // 4), byte
    (r % 32) * 16 + (r // 32) * 4 + group % 4."""
    return ((block * (k // 128) + group // 4) * 512 + (r % 32) * 16 + (r // 32) * 4 + group % 4)


def mx_quantize(x: torch.Tensor, counts) -> tuple:
    """MX e4m3 quantisation of x [rows, K] (rows in consecutive segments of `counts` rows).
    Returns (q uint8 [rows, K] e4m3 bit patterns, scales uint8 [(ceil(rows/128) + nseg) * K/128
    * 512], padding bytes 0). e4m3 rounding is torch's round-to-nearest-even float8 cast of the
    exactly scaled fp32 values (none exceeds 448, so no saturation is involved)."""
    xf = x.float().contiguous()
    rows, k = xf.shape
    assert k % 128 == 0
    g = xf.view(rows, k // 32, 32)
    amax = g.abs().amax(dim=-1).numpy()
    xe = mx_scale_exponent(amax)                                      # [rows, K/32]
    inv = torch.from_numpy(np.ldexp(np.float32(1.0), -xe).astype(np.float32))
    q = (g * inv.unsqueeze(-1)).view(rows, k).to(torch.float8_e4m3fn).view(torch.uint8)
    counts = np.minimum(np.maximum(np.asarray(counts, dtype=np.int64), 0), rows)
    nseg = counts.size
    sf = np.zeros(((rows + 127) // 128 + nseg) * (k // 128) * 512, dtype=np.uint8)
    rowoff = np.concatenate([[0], np.cumsum(counts)])
    blkoff = np.concatenate([[0], np.cumsum((counts + 127) // 128)])
    groups = np.arange(k // 32)
    for s_ in range(nseg):
        for rl in range(int(counts[s_])):
            r = rowoff[s_] + rl
            if r >= rows:
                break
            off = mx_atom_offset(blkoff[s_] + rl // 128, rl % 128, groups, k)
            sf[off] = (xe[r] + 127).astype(np.uint8)
    return q, sf


def mx_dequantize(q: torch.Tensor, sf: np.ndarray, counts, k: int) -> torch.Tensor:
    """fp32 values q * 2^(scale - 127) of MX data laid out as mx_quantize writes it."""
    qf = q.view(torch.float8_e4m3fn).float().view(-1, k)
    rows = qf.size(0)
    counts = np.minimum(np.maximum(np.asarray(counts, dtype=np.int64), 0), rows)
    rowoff = np.concatenate([[0], np.cumsum(counts)])
    blkoff = np.concatenate([[0], np.cumsum((counts + 127) // 128)])
    scale = np.ones((rows, k // 32), dtype=np.float32)
    groups = np.arange(k // 32)
    for s_ in range(counts.size):
        for rl in range(int(counts[s_])):
            r = rowoff[s_] + rl
            off = mx_atom_offset(blkoff[s_] + rl // 128, rl % 128, groups, k)
            scale[r] = np.ldexp(np.float32(1.0), sf[off].astype(np.int64) - 127)
    return (qf.view(rows, k // 32, 32) * torch.from_numpy(scale).unsqueeze(-1)).view(rows, k)


def mx_block_gate_up(w_gate_up: torch.Tensor, block: int = 128) -> torch.Tensor:
    """[E, 2F, K] gate-then-up rows -> [E, 2 F_pad, K] blocked: block j = gate rows
    block*j.. then the matching up rows, zero rows past F (F_pad = F rounded up to `block`)."""
    E, two_f, K = w_gate_up.shape
    f = two_f // 2
    fp = -(-f // block) * block
    gate = torch.zeros(E, fp, K, dtype=w_gate_up.dtype)
    up = torch.zeros(E, fp, K, dtype=w_gate_up.dtype)
    gate[:, :f] = w_gate_up[:, :f]
    up[:, :f] = w_gate_up[:, f:]
    out = torch.stack([gate.view(E, fp // block, block, K), up.view(E, fp // block, block, K)], 2)
    return out.reshape(E, 2 * fp, K)


def mx_unblock_gate_up(w_blocked: torch.Tensor, f: int, block: int = 128) -> torch.Tensor:
    """Inverse of mx_block_gate_up: [E, 2 F_pad, K] blocked -> [E, 2F, K] gate-then-up."""
    E, rows, K = w_blocked.shape
    v = w_blocked.reshape(E, rows // (2 * block), 2, block, K)
    gate = v[:, :, 0].reshape(E, -1, K)[:, :f]
    up = v[:, :, 1].reshape(E, -1, K)[:, :f]
    return torch.cat([gate, up], 1)

