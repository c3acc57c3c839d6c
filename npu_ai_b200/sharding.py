"""Fused attention over (batch, head) pairs split across the ranks of a process group.

The reference runs every (batch, head) pair of an attention block in one NPU dispatch
(npu/xdna1_gemm.py:499-600, `NpuGemm.attention`); the pairs are independent, so on several B200s they split: rank r
of W owns the contiguous pair range [r * width, min((r + 1) * width, B*H)) with width = ceil(B*H / W), runs the
fused kernel over it into a head-major buffer [width, Sq, D], and one NCCL all_gather_into_tensor assembles the
(B, H, Sq, D) result on every rank. The inputs must already be resident on every rank (each rank reads only its
pairs' rows). The model's (B, Sq, H*D) output layout costs one more pass: the gathered head-major block is
transposed into it on the device (`relayout` in the timings). No pair's data crosses NVLink more than once.

A pair range maps onto at most three strided views of the caller's tensors (the tail of one batch's heads, whole
batches, the head of the last batch's heads), so the kernel reads the operands in place: one launch per view.
"""
from __future__ import annotations

import math

import torch


def pair_range(pairs: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of the (batch, head) pairs rank `rank` of `world` computes (empty for trailing ranks when
    pairs < world). Every rank's chunk in the gather is `pair_width(pairs, world)` rows of pairs."""
    width = pair_width(pairs, world)
    lo = min(pairs, rank * width)
    return lo, min(pairs, lo + width)


def pair_width(pairs: int, world: int) -> int:
    return max(1, math.ceil(pairs / world))


def pair_segments(lo: int, hi: int, heads: int) -> list[tuple[int, int, int, int]]:
    """Split the pair range [lo, hi) (pair p = b * heads + h) into (b0, b1, h0, h1) blocks, each the heads
    [h0, h1) of batches [b0, b1): a partial leading batch, a run of whole batches, a partial trailing batch."""
    segs = []
    p = lo
    while p < hi:
        b, h = divmod(p, heads)
        if h == 0 and hi - p >= heads:
            nb = (hi - p) // heads
            segs.append((b, b + nb, 0, heads))
            p += nb * heads
        else:
            h1 = min(heads, h + (hi - p))
            segs.append((b, b + 1, h, h1))
            p += h1 - h
    return segs


def _kernel_compute(q, k, v, heads, out, head_major_in, scale, variant):
    from . import kernels
    kernels.attention(q, k, v, heads, scale=scale, head_major_in=head_major_in, head_major_out=True,
                      out_dtype=out.dtype, out=out, variant=variant)


def attention_shard(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, rank: int, world: int,
                    scale: float | None = None, head_major_in: bool = False, out_dtype: torch.dtype = torch.bfloat16,
                    variant: int = 0, compute=None) -> torch.Tensor:
    """This rank's part of the block: a head-major [width, Sq, D] buffer whose first hi - lo rows of pairs are the
    outputs of pairs [lo, hi) (the rest is padding for the equal-sized gather).

    q/k/v: the full block on this device, (B, S, H*D) or (B, H, S, D) when head_major_in. `compute` replaces the
    kernel launch (tests of the host logic on the CPU pass a CPU stand-in); by default it is the fused kernel."""
    if head_major_in:
        B, H, Sq, D = q.shape
    else:
        B, Sq, inner = q.shape
        H = int(heads)
        if H <= 0 or inner % H:
            raise ValueError(f"q's last dimension {inner} is not a multiple of heads={heads}")
        D = inner // H
    pairs = B * H
    lo, hi = pair_range(pairs, world, rank)
    width = pair_width(pairs, world)
    local = torch.empty((width, Sq, D), dtype=out_dtype, device=q.device)
    run = compute or _kernel_compute
    done = 0
    for b0, b1, h0, h1 in pair_segments(lo, hi, H):
        n = (b1 - b0) * (h1 - h0)
        if head_major_in:
            qv, kv, vv = (t[b0:b1, h0:h1] for t in (q, k, v))
        else:
            qv, kv, vv = (t[b0:b1, :, h0 * D:h1 * D] for t in (q, k, v))
        ov = local[done:done + n].view(b1 - b0, h1 - h0, Sq, D)
        run(qv, kv, vv, h1 - h0, ov, head_major_in, scale, variant)
        done += n
    return local


def attention_sharded(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, group=None,
                      scale: float | None = None, head_major_in: bool = False, head_major_out: bool = False,
                      out_dtype: torch.dtype = torch.bfloat16, variant: int = 0, compute=None,
                      timings: dict | None = None) -> torch.Tensor:
    """softmax(q k^T * scale) v over every (batch, head) pair of the block, the pairs split across the ranks of
    `group` (torch.distributed; the default group when None) and the result all-gathered on every rank.

    Returns (B, H, Sq, D) when head_major_out, else (B, Sq, H*D). With `timings` (a dict, CUDA tensors only) CUDA
    events bracket the kernel launches, the all-gather and the relayout; `resolve_timings` turns them into ms."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if head_major_in:
        B, H, Sq, D = q.shape
    else:
        B, Sq, inner = q.shape
        H = int(heads)
        D = inner // H
    pairs = B * H
    width = pair_width(pairs, world)
    ev = None
    if timings is not None and q.is_cuda:
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
    local = attention_shard(q, k, v, H, rank, world, scale=scale, head_major_in=head_major_in, out_dtype=out_dtype,
                            variant=variant, compute=compute)
    if ev is not None:
        ev[1].record()
    gathered = torch.empty((world * width, Sq, D), dtype=out_dtype, device=q.device)
    dist.all_gather_into_tensor(gathered, local, group=group)
    if ev is not None:
        ev[2].record()
    hm = gathered[:pairs].view(B, H, Sq, D)
    out = hm if head_major_out else hm.permute(0, 2, 1, 3).reshape(B, Sq, H * D)
    if ev is not None:
        ev[3].record()
        timings["events"] = ev
        timings["pairs_per_rank"] = width
        timings["gather_bytes_per_rank"] = (world - 1) * width * Sq * D * gathered.element_size()
    return out


def resolve_timings(timings: dict) -> dict:
    """ms of the kernel launches, the all-gather and the relayout recorded by attention_sharded (synchronises)."""
    ev = timings["events"]
    ev[3].synchronize()
    return {"kernel_ms": ev[0].elapsed_time(ev[1]), "gather_ms": ev[1].elapsed_time(ev[2]),
            "relayout_ms": ev[2].elapsed_time(ev[3]), "pairs_per_rank": timings["pairs_per_rank"],
            "gather_bytes_per_rank": timings["gather_bytes_per_rank"]}
