"""Vocabulary-parallel tied cross-entropy across the GPUs of one node.

The reference has no distributed code; this is the vocab split the B200
design adds. Rank r of P owns rows ``[r*Vp, min((r+1)*Vp, V))`` of the tied
matrix E (Vp = ceil(V / P)). ``hidden`` and the labels are replicated.

* forward: each rank reduces its vocab columns to per-token (max, sum-exp,
  target) — 12 bytes per token — and one ``all_gather`` exchanges them; every
  rank then merges the P triples in the same fixed order, so all ranks hold
  bit-identical lse and loss.
* backward: each rank recomputes its logits with the global lse, writes the
  complete grad of its own E rows (no communication) and a partial
  grad_hidden = G_r . E_r, summed by one fp32 ``all_reduce`` over NCCL.

Collectives go through ``torch.distributed`` (NCCL on GPUs, gloo on CPU for
the host-logic tests).
"""
from __future__ import annotations

from typing import Optional, Tuple

import os

import torch
import torch.distributed as dist

# SMs left free for the grad_hidden all_reduce while the last grad_weights
# GEMM runs (NIMBLEML_TIED_CE_COMM_SMS, default 32; with 8 at 8 ranks NCCL is
# starved and the reduction waits for the GEMM).
COMM_SMS = int(os.environ.get("NIMBLEML_TIED_CE_COMM_SMS", "32"))
# Share of the last grad_weights GEMM's rows that run beside the reduction on
# the capped SM count; the rest run on all SMs (NIMBLEML_TIED_CE_CAPPED_FRACTION,
# 1 = the whole GEMM capped).
CAPPED_FRACTION = float(os.environ.get("NIMBLEML_TIED_CE_CAPPED_FRACTION", "1.0"))
# Element type of the grad_hidden partials and of their all_reduce
# (NIMBLEML_TIED_CE_DH_REDUCE_DTYPE: auto, float32, float16 or bfloat16).
# "auto" reduces bfloat16 partials for 16-bit inputs (half the NVLink bytes of
# fp32, fp32's exponent range so no loss scale is needed; ~3e-3 relative
# error against the 1e-2 grad tolerance) and float32 partials for fp32 inputs.
_DH_REDUCE = os.environ.get("NIMBLEML_TIED_CE_DH_REDUCE_DTYPE", "auto")


def dh_reduce_dtype(compute_dtype: torch.dtype) -> torch.dtype:
    if _DH_REDUCE != "auto":
        return getattr(torch, _DH_REDUCE)
    return torch.float32 if compute_dtype == torch.float32 else torch.bfloat16
_comm_streams: dict = {}


def world_size(group=None) -> int:
    if group is None or not dist.is_available() or not dist.is_initialized():
        return 1
    return dist.get_world_size(group)


def rank_in(group=None) -> int:
    if group is None or not dist.is_available() or not dist.is_initialized():
        return 0
    return dist.get_rank(group)


def shard_range(vocab_size: int, rank: int, world: int) -> Tuple[int, int]:
    """(vocab_offset, rows) of rank's shard; the last shard may be short."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    per = -(-vocab_size // world)
    start = min(rank * per, vocab_size)
    stop = min(start + per, vocab_size)
    return start, stop - start


def gather_shard_stats(part: torch.Tensor, group=None) -> torch.Tensor:
    """(3, N) local shard statistics -> (3, P, N) statistics of every shard, rank order."""
    p = world_size(group)
    if p == 1:
        return part.unsqueeze(1)
    part = part.contiguous()
    out = torch.empty((p * part.shape[0], part.shape[1]), dtype=part.dtype, device=part.device)
    dist.all_gather_into_tensor(out, part, group=group)
    return out.view(p, part.shape[0], part.shape[1]).permute(1, 0, 2).contiguous()


def reduce_grad_hidden(grad_h: torch.Tensor, group=None) -> torch.Tensor:
    """Sums the per-shard partial grad_hidden over the group (in place, fp32)."""
    if world_size(group) > 1:
        dist.all_reduce(grad_h, op=dist.ReduceOp.SUM, group=group)
    return grad_h


def _comm_stream(device: torch.device) -> torch.cuda.Stream:
    key = device.index
    st = _comm_streams.get(key)
    if st is None:
        st = torch.cuda.Stream(device=device)
        _comm_streams[key] = st
    return st


def sharded_backward(grad_scale, h, w, labels, stats, group=None, *, grad_weights=None, accumulate=False,
                     phase_events=None):
    """Backward of one vocab shard with the grad_hidden all_reduce overlapped.

    The library computes the last slab's grad_hidden first and records an
    event; the fp32 all_reduce then runs on a side stream while the last
    grad_weights GEMM runs on all but COMM_SMS SMs (its first
    CAPPED_FRACTION of rows; the rest on all SMs). Returns (grad_hidden
    summed over ranks, in dh_reduce_dtype(h.dtype); grad_weights of this
    shard).

    ``phase_events``: optional dict of four timing-enabled CUDA events,
    recorded at the end of the backward kernels ("compute_end", current
    stream), around the all_reduce ("comm_start", "comm_end", side stream)
    and once the current stream has caught up with it ("end").
    """
    from nimbleml_b200.kernels.fused_tied_crossentropy import shard_backward

    if world_size(group) == 1:
        return shard_backward(grad_scale, h, w, labels, stats, grad_weights=grad_weights, accumulate=accumulate)
    dev = h.device
    ready = torch.cuda.Event()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    grad_h, grad_w = shard_backward(grad_scale, h, w, labels, stats, grad_hidden_dtype=dh_reduce_dtype(h.dtype),
                                    grad_weights=grad_weights, accumulate=accumulate, ready_event=ready,
                                    last_de_max_ctas=max(1, sms - COMM_SMS), capped_fraction=CAPPED_FRACTION)
    if phase_events:
        phase_events["compute_end"].record()
    comm = _comm_stream(dev)
    comm.wait_event(ready)
    with torch.cuda.stream(comm):
        if phase_events:
            phase_events["comm_start"].record()
        dist.all_reduce(grad_h, op=dist.ReduceOp.SUM, group=group)
        if phase_events:
            phase_events["comm_end"].record()
    grad_h.record_stream(comm)
    torch.cuda.current_stream(dev).wait_stream(comm)
    if phase_events:
        phase_events["end"].record()
    return grad_h, grad_w


class VocabParallelTiedHead:
    """Holds this rank's shard of the tied matrix and applies the sharded loss."""

    def __init__(self, full_weights: Optional[torch.Tensor], vocab_size: int, group=None,
                 shard: Optional[torch.Tensor] = None):
        self.group = group
        self.vocab_size = int(vocab_size)
        self.world = world_size(group)
        self.rank = rank_in(group)
        self.vocab_offset, self.rows = shard_range(self.vocab_size, self.rank, self.world)
        if shard is None:
            if full_weights is None:
                raise ValueError("pass full_weights or shard")
            shard = full_weights[self.vocab_offset:self.vocab_offset + self.rows]
        if shard.shape[0] != self.rows:
            raise ValueError(f"shard has {shard.shape[0]} rows, expected {self.rows}")
        self.weights = shard.contiguous()

    def hidden_from_host(self, hidden_host: torch.Tensor) -> torch.Tensor:
        """Replicates host-resident hidden states (N, d) on every rank's GPU.

        Each rank copies only its 1/P slice of the rows from host memory
        and one all_gather over NVLink assembles the rest, so PCIe traffic
        per rank falls from N*d to N*d/P elements. The copy is asynchronous
        when ``hidden_host`` is pinned; a pageable tensor's slice is pinned
        here first (one extra host copy of the slice). Returns a device
        tensor (not a leaf of any graph).
        """
        dev = self.weights.device
        pin = dev.type == "cuda"  # pinned memory needs a CUDA driver
        if self.world == 1:
            src = hidden_host.pin_memory() if pin and not hidden_host.is_pinned() else hidden_host
            return src.to(dev, non_blocking=True)
        n, d = hidden_host.shape
        per = -(-n // self.world)
        lo, hi = min(self.rank * per, n), min((self.rank + 1) * per, n)
        rows = hidden_host[lo:hi]
        if pin and not rows.is_pinned():
            rows = rows.pin_memory()
        chunk = torch.zeros((per, d), dtype=hidden_host.dtype, device=dev)
        chunk[: hi - lo].copy_(rows, non_blocking=True)
        full = torch.empty((per * self.world, d), dtype=hidden_host.dtype, device=dev)
        dist.all_gather_into_tensor(full, chunk, group=self.group)
        return full[:n]

    def loss(self, hidden2d: torch.Tensor, labels: torch.Tensor, ignore_index: Optional[int] = None):
        from nimbleml_b200.losses.cross_entropy import tied_cross_entropy

        return tied_cross_entropy(hidden2d, self.weights, labels, ignore_index,
                                  vocab_offset=self.vocab_offset, vocab_size=self.vocab_size,
                                  group=self.group if self.world > 1 else None)
