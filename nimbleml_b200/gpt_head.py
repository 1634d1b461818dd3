"""The rows either side of the tied head in a GPT: the final norm before it and
the tied matrix's other use, the input embedding.

* ``norm_tied_cross_entropy(x, gamma, weights, labels)`` — the last two steps
  of ``GPT.compute_loss``: the final RMSNorm (NimbleML/models/gpt.py:67,90,
  NimbleML/layers/rms_norm.py:25-95) and ``forward_tied``
  (NimbleML/losses/cross_entropy.py:109-192), as one autograd node. In the
  backward the hidden grad leaves the dh GEMM's epilogue in fp32 and the
  RMSNorm backward reads it as is: no 16-bit copy of dh is written and read
  back, and dh is not rounded before the norm's Jacobian. The forward still
  writes y = rmsnorm(x) (N x d) for the GEMM's TMA loads: normalising inside
  the operand load would need a transform stage between TMA and the tensor
  cores, and the norm's backward needs a dot product over each whole row of
  dh, which the dh GEMM spreads over d / 256 tiles.
* ``TiedEmbedding`` — one rank's vocab shard of the tied token-embedding /
  LM-head matrix E with fp32 master rows, the 16-bit (or TF32) copy the GEMMs
  read, ONE fp32 grad buffer that both uses of E add into, and the shard's
  AdamW state. The reference keeps one ``E.grad`` that the head's backward
  fills and the lookup's scatter-add then accumulates into
  (NimbleML/utils/tensor.py:334-350, NimbleML/layers/embedding.py:63-67,138-148);
  here the head's dE GEMM epilogue adds into the buffer and the deterministic
  scatter-add follows, in that order. ``step`` runs the reference's AdamW
  update (NimbleML/optimizers/adam.py:133-203, 295-312) over the shard and
  refreshes the compute copy in the same pass.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from nimbleml_b200 import vocab_parallel
from nimbleml_b200.embedding_grad import embedding_scatter_add
from nimbleml_b200.kernels.fused_tied_crossentropy import (
    _NO_IGNORE,
    _TORCH_TO_NIMBLE,
    _stream_ptr,
    as_label_indices,
    compute_dtype_of,
    native,
)
from nimbleml_b200.losses.cross_entropy import tied_backward_core, tied_cross_entropy, tied_forward_core
from nimbleml_b200.norm import rmsnorm_backward, rmsnorm_forward


class _NormTiedCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, weights, labels, ignore_index, eps, vocab_offset, vocab_size, group, grad_buffer):
        d = x.shape[-1]
        x2d = x.reshape(-1, d).contiguous()
        g = gamma.to(x.dtype).contiguous()
        y, ms, rms = rmsnorm_forward(x2d, g, eps)
        loss, saved = tied_forward_core(y, weights, labels, ignore_index, vocab_offset, vocab_size, group)
        ctx.saved = saved
        ctx.norm = (x2d, g, ms, rms, float(eps), gamma.dtype, x.shape)
        ctx.grad_buffer = grad_buffer
        return loss

    @staticmethod
    def backward(ctx, grad_out):
        saved, buf = ctx.saved, ctx.grad_buffer
        x2d, g, ms, rms, eps, gamma_dtype, x_shape = ctx.norm
        ctx.saved = ctx.grad_buffer = ctx.norm = None
        # fp32 grad_hidden straight from the head (at P > 1 the reduced partials).
        grad_y, grad_w = tied_backward_core(grad_out, saved, grad_buffer=buf, grad_hidden_dtype=torch.float32)
        gx, gg = rmsnorm_backward(grad_y, x2d, g, ms, rms, eps)
        return gx.view(x_shape), gg.to(gamma_dtype), grad_w, None, None, None, None, None, None, None


def norm_tied_cross_entropy(x: torch.Tensor, gamma: torch.Tensor, weights: torch.Tensor, labels,
                            ignore_index: Optional[int] = None, eps: float = 1e-5, *, vocab_offset: int = 0,
                            vocab_size: Optional[int] = None, group=None,
                            grad_weights_buffer: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Mean CE of ``rmsnorm(x, gamma) @ weights^T`` against ``labels`` (fp32 0-d loss).

    ``x`` is (..., d) pre-norm hidden states; sharding and
    ``grad_weights_buffer`` as in :func:`tied_cross_entropy`.
    """
    compute_dtype_of(x)
    if x.shape[-1] != gamma.shape[-1] or x.shape[-1] != weights.shape[-1]:
        raise ValueError("x, gamma and weights must share the last dimension")
    n = x.numel() // x.shape[-1]
    y = as_label_indices(labels, batch_size=n, device=x.device)
    ign = _NO_IGNORE if ignore_index is None else int(ignore_index)
    if vocab_size is None:
        vocab_size = weights.shape[0]
    return _NormTiedCE.apply(x, gamma, weights, y, ign, float(eps), int(vocab_offset), int(vocab_size), group,
                             grad_weights_buffer)


class _Lookup(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, anchor, emb):
        flat = ids.reshape(-1)
        lo, rows = emb.vocab_offset, emb.rows
        local = flat - lo
        mine = (local >= 0) & (local < rows)
        out = emb.weight[torch.where(mine, local, torch.zeros_like(local))]
        if emb.world > 1:
            # Vocab-parallel lookup: rows of other shards are zero here and
            # come from their owners in one all_reduce (exactly one nonzero
            # term per element, so the sum is exact).
            out = out * mine.unsqueeze(1).to(out.dtype)
            dist.all_reduce(out, group=emb.group)
        ctx.emb = emb
        ctx.save_for_backward(flat)
        return out.view(*ids.shape, emb.weight.shape[1])

    @staticmethod
    def backward(ctx, grad_out):
        (flat,) = ctx.saved_tensors
        emb = ctx.emb
        ctx.emb = None
        embedding_scatter_add(emb.grad, flat, grad_out, vocab_offset=emb.vocab_offset, vocab_size=emb.vocab_size)
        return None, None, None


class TiedEmbedding:
    """One rank's vocab shard of a tied embedding / LM-head matrix.

    Args:
        master: (rows, d) fp32 master rows [vocab_offset, vocab_offset + rows).
        vocab_size: the whole vocabulary V.
        compute_dtype: the dtype of the copy the lookup and the GEMMs read
            (float16, bfloat16, or float32 for TF32).
        group: torch.distributed group of the vocab split (None: one rank).
        AdamW hyper-parameters as the reference's ``AdamW``.
    """

    def __init__(self, master: torch.Tensor, vocab_size: int, *, vocab_offset: int = 0,
                 compute_dtype: torch.dtype = torch.float16, group=None, learning_rate: float = 1e-3,
                 beta1: float = 0.9, beta2: float = 0.999, epsilon: float = 1e-8, weight_decay: float = 0.01):
        if master.dtype != torch.float32 or master.ndim != 2:
            raise ValueError("master must be a (rows, d) float32 tensor")
        self.master = master.contiguous()
        self.vocab_size = int(vocab_size)
        self.vocab_offset = int(vocab_offset)
        self.rows = self.master.shape[0]
        self.group = group
        self.world = vocab_parallel.world_size(group)
        if self.vocab_offset < 0 or self.vocab_offset + self.rows > self.vocab_size:
            raise ValueError("the shard must lie inside the vocabulary")
        self.weight = self.master.to(compute_dtype)
        self.grad = torch.zeros_like(self.master)
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.lr, self.beta1, self.beta2 = float(learning_rate), float(beta1), float(beta2)
        self.epsilon, self.weight_decay = float(epsilon), float(weight_decay)
        self.t = 0
        # The lookup's inputs are integer ids; this empty tensor that requires
        # grad makes autograd run its backward (the scatter-add into grad).
        self._anchor = torch.empty(0, device=self.master.device, requires_grad=True)

    def lookup(self, ids: torch.Tensor) -> torch.Tensor:
        """Embedding rows of ``ids`` (any shape) in the compute dtype; the
        backward scatter-adds into ``grad`` (NimbleML/layers/embedding.py:23-67)."""
        return _Lookup.apply(ids.to(torch.int64), self._anchor, self)

    def loss(self, hidden: torch.Tensor, labels, ignore_index: Optional[int] = None, *,
             norm_gamma: Optional[torch.Tensor] = None, norm_eps: float = 1e-5) -> torch.Tensor:
        """Mean tied CE of ``hidden`` (..., d); with ``norm_gamma`` the final
        RMSNorm is applied first, in the same autograd node. The head's dE
        is added into ``grad``."""
        d = hidden.shape[-1]
        kw = dict(vocab_offset=self.vocab_offset, vocab_size=self.vocab_size,
                  group=self.group if self.world > 1 else None, grad_weights_buffer=self.grad)
        if norm_gamma is not None:
            return norm_tied_cross_entropy(hidden, norm_gamma, self.weight, labels, ignore_index, norm_eps, **kw)
        h2d = hidden.reshape(-1, d)
        y = as_label_indices(labels, batch_size=h2d.shape[0], device=hidden.device)
        return tied_cross_entropy(h2d, self.weight, y, ignore_index, **kw)

    def zero_grad(self) -> None:
        self.grad.zero_()

    @torch.no_grad()
    def step(self) -> None:
        """One AdamW step over the shard's master rows; the compute copy is
        rewritten in the same kernel pass."""
        self.t += 1
        bc1 = 1.0 - self.beta1 ** self.t
        bc2 = 1.0 - self.beta2 ** self.t
        native.call("nimble_adamw_step", self.master.data_ptr(), self.grad.data_ptr(), _TORCH_TO_NIMBLE[torch.float32],
                    self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(), self.master.numel(), self.lr, self.beta1,
                    self.beta2, bc1, bc2, self.epsilon, self.weight_decay, self.weight.data_ptr(),
                    _TORCH_TO_NIMBLE[self.weight.dtype], _stream_ptr(self.master.device))


__all__ = ["norm_tied_cross_entropy", "TiedEmbedding"]
