"""The tied matrix's other grad and its update: embedding scatter-add and AdamW.

* ``embedding_scatter_add`` — grad_weights[ids] += grad_out, the input
  embedding's share of the tied matrix's grad
  (NimbleML/kernels/embedding_scatter.py:39-81), into an fp32 grad buffer,
  deterministically and for one vocab shard.
* ``AdamW`` — the reference's fused AdamW update (NimbleML/optimizers/adam.py:20-43,
  85-131, 295-312) over fp32 master weights, e.g. one rank's vocab shard of E,
  with an optional low-precision copy written in the same pass.
"""
from __future__ import annotations

from typing import Iterable, Optional

import torch

from nimbleml_b200.kernels.fused_tied_crossentropy import _TORCH_TO_NIMBLE, _stream_ptr, native, status_word


def embedding_scatter_add(grad_weights: torch.Tensor, ids: torch.Tensor, grad_out: torch.Tensor, *,
                          vocab_offset: int = 0, vocab_size: Optional[int] = None) -> torch.Tensor:
    """In-place ``grad_weights[ids[i] - vocab_offset] += grad_out[i]`` into an fp32 grad.

    ``grad_weights`` holds rows [vocab_offset, vocab_offset + rows) of a
    ``vocab_size`` vocabulary (default: all of it); ids of other rows are
    skipped, ids outside [0, vocab_size) set the status word's bad-label bit.
    Deterministic: each id's rows are added in ascending row order, the loop
    order of the reference's CPU scatter (native/src/scatter.cpp:6-15).
    """
    if grad_weights.dtype != torch.float32 or not grad_weights.is_contiguous():
        raise ValueError("grad_weights must be a contiguous float32 (vocab, d) tensor")
    v, d = grad_weights.shape
    vocab_size = v if vocab_size is None else int(vocab_size)
    flat_ids = ids.reshape(-1).to(torch.int64).contiguous()
    go = grad_out.reshape(-1, d).contiguous()
    n = go.shape[0]
    if n != flat_ids.numel():
        raise ValueError(f"ids length ({flat_ids.numel()}) must match grad_out rows ({n}).")
    if n == 0:
        return grad_weights
    ws_bytes = native.scatter_add_workspace_size(n, v)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=go.device)
    native.call("nimble_embedding_scatter_add", grad_weights.data_ptr(), flat_ids.data_ptr(), go.data_ptr(), n,
                int(vocab_offset), v, vocab_size, d, _TORCH_TO_NIMBLE[go.dtype], ws.data_ptr(), ws_bytes,
                status_word(go.device).data_ptr(), _stream_ptr(go.device))
    return grad_weights


class AdamW:
    """AdamW over fp32 master tensors (learning_rate, beta1, beta2, epsilon, weight_decay
    as in the reference's ``AdamW``); ``copies`` optionally receive the updated
    weights in their own dtype (e.g. the fp16 E used by the GEMMs)."""

    def __init__(self, params: Iterable[torch.Tensor], learning_rate=0.001, beta1=0.9, beta2=0.999,
                 epsilon=1e-8, weight_decay=0.01, copies: Optional[Iterable[Optional[torch.Tensor]]] = None):
        self.params = list(params)
        for p in self.params:
            if p.dtype != torch.float32 or not p.is_contiguous():
                raise ValueError("AdamW master weights must be contiguous float32 tensors")
        self.copies = list(copies) if copies is not None else [None] * len(self.params)
        self.lr, self.beta1, self.beta2 = float(learning_rate), float(beta1), float(beta2)
        self.epsilon, self.weight_decay = float(epsilon), float(weight_decay)
        self.m = [torch.zeros_like(p) for p in self.params]
        self.v = [torch.zeros_like(p) for p in self.params]
        self.t = 0

    @torch.no_grad()
    def step(self):
        self.t += 1
        bc1 = 1.0 - self.beta1 ** self.t
        bc2 = 1.0 - self.beta2 ** self.t
        for p, m, v, c in zip(self.params, self.m, self.v, self.copies):
            if p.grad is None:
                continue
            g = p.grad.contiguous()
            native.call("nimble_adamw_step", p.data_ptr(), g.data_ptr(), _TORCH_TO_NIMBLE[g.dtype], m.data_ptr(),
                        v.data_ptr(), p.numel(), self.lr, self.beta1, self.beta2, bc1, bc2, self.epsilon,
                        self.weight_decay, c.data_ptr() if c is not None else None,
                        _TORCH_TO_NIMBLE[c.dtype] if c is not None else 0, _stream_ptr(p.device))

    def zero_grad(self, set_to_none: bool = True):
        for p in self.params:
            p.grad = None if set_to_none else (torch.zeros_like(p) if p.grad is None else p.grad.zero_())


__all__ = ["embedding_scatter_add", "AdamW"]
